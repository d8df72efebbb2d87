"""Phenomenological noise for the rotated surface-code memory (synthetic inputs for the pre-decoder).

Per round t = 0 .. R - 1 every data qubit takes an X flip and a Z flip, each Bernoulli(p), and every stabilizer
measurement is flipped with probability q (default p).  Z checks see the accumulated X flips, X checks the accumulated
Z flips; the detector of check c at round t is the XOR of its measured parities at rounds t and t - 1 (parity 0 before
round 0).  Equivalently det[c, t] = (H flips[t])_c ^ m[c, t] ^ m[c, t - 1], which is how it is computed here.

Outputs follow the node order of geometry.RotatedSurface: det (shots, N_c) uint8 in check-node order and the data-qubit
error labels err (shots, N_d, 2) uint8 = (X flip, Z flip) of data node (t, q) at round t.  The reference draws its
shots from Stim circuits (cascade/d13/surface/surface_data.py), which are circuit-level and need Stim; this sampler is
the phenomenological model the pre-decoder workloads are specified with.
"""
from __future__ import annotations

import numpy as np

from .geometry import RotatedSurface


def _det_from_flips(geo: RotatedSurface, xf, zf, mx, mz, xp):
    """xf, zf: (S, T, d^2) 0/1; mx, mz: (S, T, nh) 0/1 -> det (S, N_c) uint8, err (S, N_d, 2) uint8."""
    S = xf.shape[0]
    if xp is np:
        hz = geo.hz.T.astype(np.float32)
        hx = geo.hx.T.astype(np.float32)
        sz = (xf.astype(np.float32) @ hz).astype(np.int64) & 1      # Z checks see X flips
        sx = (zf.astype(np.float32) @ hx).astype(np.int64) & 1
        mxp = np.concatenate([np.zeros_like(mx[:, :1]), mx[:, :-1]], 1)
        mzp = np.concatenate([np.zeros_like(mz[:, :1]), mz[:, :-1]], 1)
        dx = (sx ^ mx ^ mxp).astype(np.uint8)
        dz = (sz ^ mz ^ mzp).astype(np.uint8)
        det = np.concatenate([dx.reshape(S, -1), dz.reshape(S, -1)], 1)
        err = np.stack([xf.reshape(S, -1), zf.reshape(S, -1)], -1).astype(np.uint8)
        return det, err
    import torch
    dev = xf.device
    hz = torch.as_tensor(geo.hz.T, dtype=torch.float32, device=dev)
    hx = torch.as_tensor(geo.hx.T, dtype=torch.float32, device=dev)
    sz = (xf.float() @ hz).to(torch.int32) & 1
    sx = (zf.float() @ hx).to(torch.int32) & 1
    mx = mx.to(torch.int32)
    mz = mz.to(torch.int32)
    mxp = torch.cat([torch.zeros_like(mx[:, :1]), mx[:, :-1]], 1)
    mzp = torch.cat([torch.zeros_like(mz[:, :1]), mz[:, :-1]], 1)
    dx = (sx ^ mx ^ mxp).to(torch.uint8)
    dz = (sz ^ mz ^ mzp).to(torch.uint8)
    det = torch.cat([dx.reshape(S, -1), dz.reshape(S, -1)], 1)
    err = torch.stack([xf.reshape(S, -1), zf.reshape(S, -1)], -1).to(torch.uint8)
    return det, err


def sample(geo: RotatedSurface, p: float, shots: int, seed: int, q: float | None = None, chunk: int = 8192):
    """Seeded numpy sampler -> (det (shots, N_c) uint8, err (shots, N_d, 2) uint8)."""
    q = p if q is None else q
    rng = np.random.default_rng(seed)
    T, nq, nh = geo.T, geo.n_data_round, geo.nh
    dets, errs = [], []
    for s0 in range(0, shots, chunk):
        S = min(chunk, shots - s0)
        xf = (rng.random((S, T, nq), dtype=np.float32) < p)
        zf = (rng.random((S, T, nq), dtype=np.float32) < p)
        mx = (rng.random((S, T, nh), dtype=np.float32) < q).astype(np.int64)
        mz = (rng.random((S, T, nh), dtype=np.float32) < q).astype(np.int64)
        det, err = _det_from_flips(geo, xf, zf, mx, mz, np)
        dets.append(det)
        errs.append(err)
    if not dets:
        return np.zeros((0, geo.N_c), np.uint8), np.zeros((0, geo.N_d, 2), np.uint8)
    return np.concatenate(dets, 0), np.concatenate(errs, 0)


def sample_torch(geo: RotatedSurface, p: float, shots: int, seed: int, device="cpu", q: float | None = None,
                 chunk: int = 16384):
    """The same model drawn with torch's generator on `device` (large synthetic batches) -> (det, err) tensors."""
    import torch
    q = p if q is None else q
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    T, nq, nh = geo.T, geo.n_data_round, geo.nh
    det = torch.empty((shots, geo.N_c), dtype=torch.uint8, device=device)
    err = torch.empty((shots, geo.N_d, 2), dtype=torch.uint8, device=device)
    for s0 in range(0, shots, chunk):
        S = min(chunk, shots - s0)
        xf = torch.rand((S, T, nq), generator=g, device=device) < p
        zf = torch.rand((S, T, nq), generator=g, device=device) < p
        mx = torch.rand((S, T, nh), generator=g, device=device) < q
        mz = torch.rand((S, T, nh), generator=g, device=device) < q
        d_, e_ = _det_from_flips(geo, xf, zf, mx, mz, torch)
        det[s0:s0 + S] = d_
        err[s0:s0 + S] = e_
    return det, err


def sample_stream(geo: RotatedSurface, p: float, rounds: int, seed: int, q: float | None = None) -> np.ndarray:
    """A continuous phenomenological stream of `rounds` rounds for one memory experiment -> (rounds, 2 nh) uint8:
    per round the X checks' detectors then the Z checks' (the per-round order of RotatedSurface's check nodes)."""
    q = p if q is None else q
    rng = np.random.default_rng(seed)
    nq, nh = geo.n_data_round, geo.nh
    xf = (rng.random((rounds, nq), dtype=np.float32) < p).astype(np.float32)
    zf = (rng.random((rounds, nq), dtype=np.float32) < p).astype(np.float32)
    mx = (rng.random((rounds, nh), dtype=np.float32) < q).astype(np.int64)
    mz = (rng.random((rounds, nh), dtype=np.float32) < q).astype(np.int64)
    sz = (xf @ geo.hz.T.astype(np.float32)).astype(np.int64) & 1
    sx = (zf @ geo.hx.T.astype(np.float32)).astype(np.int64) & 1
    mxp = np.concatenate([np.zeros((1, nh), np.int64), mx[:-1]], 0)
    mzp = np.concatenate([np.zeros((1, nh), np.int64), mz[:-1]], 0)
    return np.concatenate([sx ^ mx ^ mxp, sz ^ mz ^ mzp], 1).astype(np.uint8)
