"""CPU oracle of the bipartite-conv pre-decoder path -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may import this module, and only to verify
results (or as the timed CPU baseline): the product path (codecoder_b200) never calls it.

What it restates:
  gather_mm      the reference's _GatherMM.forward (training/bb/ising_compare/bb/cascade_net.py:146-153): pad the
                 sources with a zero row, index_select by the (NT, K) table, one matmul with W^T (C_out, K C_in).
                 gather_mm_loop is the literal per-relation sum y = sum_r x[idx[:, r]] W_r^T of the Triton kernel's
                 docstring (cascade_triton.py:5,40) for small cases.
  gather_mm_dgrad / gather_mm_wgrad
                 the reference's _GatherMM.backward (cascade_net.py:155-171): the input gradient as the per-relation
                 sum gx[b, s] = sum_r gy[b, tgt[s, r]] W_r over the target table of the Triton backward
                 (cascade_triton.py:173-186), and the weight gradient gy^T gather(x) (cascade_triton.py:64-93).
  cascade_block  the reference's bottleneck residual Block in eval mode (cascade_net.py:195-210,236-259): BatchNorm
                 with running statistics, SiLU, bias-free down / up projections, the bipartite convolution, residual.
  bipartite_conv BipartiteConv.forward (cascade_net.py:228-233): check -> data for every data type, concatenated,
                 then data -> check for every check type.
  predecoder     the rotated-surface pre-decoder of codecoder_b200.params (embed, L x [c2d, GELU, residual;
                 d2c, GELU, residual], X / Z head, threshold, XOR cancellation).  Storage rounding is emulated: a
                 bf16 network rounds every stored activation to bf16 exactly where the device stores bf16, and
                 accumulates in float64 here (fp32 on the device).
  cancel         the GF(2) syndrome cancellation, integer numpy.
  route          the routing rule of the reference's decoder (|logit| < tau, here over the pre-decoder's data-qubit
                 logits, or a non-empty residual) and its ordered hand-off.
  parity_report / deep_parity
                 the parity figures of a GPU run against this oracle (logit error, band counts, residual bits);
                 deep_parity is the bar for deep bf16 networks, whose logits are chaotic in the bf16 rounding of the
                 stored activations, measured against the oracle's own float32-vs-float64 spread.
Parity pin: tests/golden/*.npz were produced by the reference's own gather_mm / BipartiteConv (imported from the
reference tree by tests/golden/make_golden.py); tests/test_oracle.py checks this module against them.
"""
from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F


def gather_mm(x: torch.Tensor, w: torch.Tensor, idx) -> torch.Tensor:
    """y[b, n] = W cat_r x[b, idx[n, r]], idx == NS reads a zero row (cascade_net.py:146-153)."""
    idx = torch.as_tensor(np.asarray(idx), dtype=torch.int64)
    B, N, C = x.shape
    nt, K = idx.shape
    xp = torch.cat([x, x.new_zeros(B, 1, C)], 1)
    g = xp.index_select(1, idx.reshape(-1)).view(B, nt, K * C)
    return g @ w.t()


def gather_mm_loop(x: np.ndarray, w: np.ndarray, idx: np.ndarray) -> np.ndarray:
    """Literal per-relation form in float64 (small cases only)."""
    B, N, C = x.shape
    nt, K = idx.shape
    co = w.shape[0]
    y = np.zeros((B, nt, co))
    x64 = x.astype(np.float64)
    w64 = w.astype(np.float64).reshape(co, K, C)
    for r in range(K):
        src = idx[:, r]
        ok = src < N
        y[:, ok] += x64[:, src[ok]] @ w64[:, r].T
    return y


def target_table(inv, NT: int, K: int) -> np.ndarray:
    """Inverse table (NS, K) of flat positions n K + r (NT K = none) -> target table, NT = none
    (cascade_triton.py:182)."""
    inv = np.asarray(inv, np.int64)
    return np.where(inv < NT * K, inv // K, NT)


def gather_mm_dgrad(gy: np.ndarray, w: np.ndarray, tgt: np.ndarray, Ci: int) -> np.ndarray:
    """gx (B, NS, Ci) float64 = sum_r gy[b, tgt[s, r]] W_r, tgt outside [0, NT) = none."""
    B, NT, Co = gy.shape
    NS, K = tgt.shape
    gy64 = np.asarray(gy, np.float64)
    w64 = np.asarray(w, np.float64).reshape(Co, K, Ci)
    gx = np.zeros((B, NS, Ci))
    for r in range(K):
        t = tgt[:, r]
        ok = (t >= 0) & (t < NT)
        gx[:, ok] += gy64[:, t[ok]] @ w64[:, r]
    return gx


def gather_mm_wgrad(x: np.ndarray, gy: np.ndarray, idx: np.ndarray) -> np.ndarray:
    """dW (Co, K Ci) float64 = sum_{b, n} gy[b, n]^T x[b, idx[n, r]] per relation r (pads contribute nothing)."""
    B, NS, Ci = x.shape
    _, NT, Co = gy.shape
    K = idx.shape[1]
    x64 = np.asarray(x, np.float64)
    gy64 = np.asarray(gy, np.float64)
    dw = np.zeros((Co, K, Ci))
    for r in range(K):
        src = idx[:, r]
        ok = (src >= 0) & (src < NS)
        dw[:, r] = np.tensordot(gy64[:, ok], x64[:, src[ok]], axes=([0, 1], [0, 1]))
    return dw.reshape(Co, K * Ci)


def bipartite_conv(x, w_c2d, w_d2c, c2d, d2c):
    """check features (B, N_c, C) -> check features (B, N_c, C), linear (cascade_net.py:228-233)."""
    data = torch.cat([gather_mm(x, w, t) for w, t in zip(w_c2d, c2d)], 1)
    return torch.cat([gather_mm(data, w, t) for w, t in zip(w_d2c, d2c)], 1)


def cascade_block(h, p: dict, c2d, d2c, L: int, res: str, eps: float = 1e-5, dtype=torch.float64):
    """h (B, N, H) -> h' in eval mode.  p: bn{1,2,3}_{weight,bias,mean,var}, down (H/4, H), up (H, H/4), w_c2d
    [(H/4, K H/4)] per data type, w_d2c [...] per check type (cascade_net.py:236-259)."""
    t = {k: torch.as_tensor(np.asarray(v)).to(dtype) for k, v in p.items() if not k.startswith("w_")}
    h = torch.as_tensor(np.asarray(h)).to(dtype)

    def bn(x, i):
        return (x - t[f"bn{i}_mean"]) / torch.sqrt(t[f"bn{i}_var"] + eps) * t[f"bn{i}_weight"] + t[f"bn{i}_bias"]

    u = F.silu(bn(h, 1)) @ t["down"].t()
    wc = [torch.as_tensor(np.asarray(w)).to(dtype) for w in p["w_c2d"]]
    wd = [torch.as_tensor(np.asarray(w)).to(dtype) for w in p["w_d2c"]]
    u = bipartite_conv(F.silu(bn(u, 2)), wc, wd, c2d, d2c)
    u = F.silu(bn(u, 3)) @ t["up"].t()
    scale = 1.0 / np.sqrt(2 * L)
    return h + scale * u if res == "branch" else scale * h + u


def _store(a: torch.Tensor, bf16: bool) -> torch.Tensor:
    return a.to(torch.bfloat16).to(a.dtype) if bf16 else a


def cancel(det: np.ndarray, e: np.ndarray, geo) -> np.ndarray:
    """residual[c] = det[c] ^ XOR over data nodes n with c in xor_nbr[n, j] of e[n, j] (uint8 in, uint8 out)."""
    det = np.asarray(det, np.uint8)
    res = det.copy()
    B = det.shape[0]
    nbr = geo.xor_nbr
    for j in range(2):
        for k in range(2):
            c = nbr[:, j, k]
            ok = c >= 0
            flips = e[:, ok, j].astype(np.uint8)             # (B, n_ok)
            np.bitwise_xor.at(res, (np.arange(B)[:, None], c[ok][None, :]), flips)
    return res


def predecoder(geo, cfg, params: dict, det: np.ndarray, dtype=torch.float64, return_features: bool = False):
    """Full forward -> (logits (B, N_d, 2) float64, residual (B, N_c) uint8[, h_c, h_d])."""
    bf16 = cfg.dtype == "bf16"
    det_t = torch.as_tensor(np.asarray(det, np.uint8)).long()
    tok = 2 * torch.as_tensor(geo.check_type) + det_t
    emb = torch.as_tensor(params["embed"]).to(dtype)
    hc = _store(emb[tok], bf16)
    B = det_t.shape[0]
    hd = None
    c2d = geo.c2d
    d2c = geo.d2c
    for layer in range(cfg.layers):
        wc = [_store(torch.as_tensor(w).to(dtype), bf16) for w in params["w_c2d"][layer]]
        wd = [_store(torch.as_tensor(w).to(dtype), bf16) for w in params["w_d2c"][layer]]
        acc = torch.cat([gather_mm(hc, w, t) for w, t in zip(wc, c2d)], 1)
        upd = F.gelu(acc, approximate="tanh")
        hd = _store(upd if hd is None else hd + upd, bf16)
        acc = torch.cat([gather_mm(hd, w, t) for w, t in zip(wd, d2c)], 1)
        hc = _store(hc + F.gelu(acc, approximate="tanh"), bf16)
    hw = torch.as_tensor(params["head_w"]).to(dtype)
    hb = torch.as_tensor(params["head_b"]).to(dtype)
    logits = hd @ hw.t() + hb
    e = (logits > 0).numpy().astype(np.uint8)
    residual = cancel(det, e, geo)
    if return_features:
        return logits.numpy(), residual, hc.numpy(), hd.numpy()
    return logits.numpy(), residual


def predecoder_batched(geo, cfg, params: dict, det: np.ndarray, dtype=torch.float64, batch: int = 64):
    """predecoder() over slices of `batch` shots (shots are independent), so the gathered (B, NT, K C) operand stays
    small at d = 13 -> (logits, residual) concatenated."""
    det = np.asarray(det, np.uint8)
    if len(det) == 0:
        return predecoder(geo, cfg, params, det, dtype=dtype)
    parts = [predecoder(geo, cfg, params, det[b:b + batch], dtype=dtype) for b in range(0, len(det), batch)]
    return np.concatenate([p[0] for p in parts]), np.concatenate([p[1] for p in parts])


def parity_report(geo, det, logits, residual, logits_ref, residual_ref, tol: float) -> dict:
    """The parity figures of a GPU run against the oracle on the same shots: max relative logit error, logits inside
    the band |logit| < tol rms (counted, and the shots that hold one), residual bits that differ at checks outside the
    band, residual bits that differ anywhere, and whether the residual is exactly the XOR of the run's own
    thresholded logits."""
    band = band_mask(logits_ref, tol)
    own = cancel(det, (np.asarray(logits) > 0).astype(np.uint8), geo)
    return {"shots": int(len(det)), "tol": tol, "logit_max_rel_err": logit_error(logits, logits_ref),
            "band_logits": int(band.sum()), "band_shots": int(band.reshape(len(det), -1).any(1).sum()),
            "logits": int(np.asarray(logits_ref).size),
            "residual_mismatch_outside_band": residual_mismatch_outside_band(residual, residual_ref, logits_ref, geo,
                                                                             tol),
            "residual_mismatch_total": int((np.asarray(residual) != np.asarray(residual_ref)).sum()),
            "residual_is_own_xor": bool(np.array_equal(own, residual))}


def _rel_err_stats(a, ref, rms):
    rel = np.abs(np.asarray(a) - ref) / np.maximum(np.abs(ref), max(rms, 1e-30))
    if rel.size == 0:
        return 0.0, 0.0, 0.0
    return (float(rel.max()), float(np.quantile(rel, 0.999)),
            float(np.sqrt(np.mean(np.square(np.asarray(a) - ref)))) / max(rms, 1e-30))


def deep_parity(geo, det, logits, residual, ref64, res64, ref32, tol: float = 2e-2) -> dict:
    """Parity of a deep bf16 network, whose logits are chaotic in the bf16 rounding of every stored activation: two
    correct restatements of the same arithmetic -- this oracle accumulating in float32 (ref32) and in float64 (ref64),
    both rounding stored activations to bf16 -- already differ by a few percent at the largest of ~10^6 logits
    (d = 13, 8 layers), because a rounding decision that tips the other way in an early layer propagates.  The bar,
    for each of the max, the 99.9th percentile and the RMS of the relative logit error against ref64:
      statistic <= max(floor, 2 x the same statistic of ref32 against ref64 on the same shots),
    floors tol (max, p99.9) and tol / 2 (RMS); and
      residual == XOR of the run's own thresholded logits (exact), and residual == the oracle's at every check none of
      whose cancelling data nodes has a logit inside the band of the observed error (outside it the sign cannot
      differ, so this checks the cancellation bit for bit).
    Band counts are reported at tol and at the observed error."""
    logits = np.asarray(logits)
    ref64 = np.asarray(ref64)
    rms = float(np.sqrt(np.mean(np.square(ref64)))) if ref64.size else 1.0
    err, p999, rrms = _rel_err_stats(logits, ref64, rms)
    s_max, s_p999, s_rms = _rel_err_stats(ref32, ref64, rms)
    band_tol = max(tol, err)
    own = cancel(det, (logits > 0).astype(np.uint8), geo)
    rep = {"shots": int(len(det)), "tol": tol, "logits": int(ref64.size),
           "logit_max_rel_err": err, "logit_p999_rel_err": p999, "logit_rms_rel_err": rrms,
           "oracle_spread_fp32_vs_fp64": {"max": s_max, "p999": s_p999, "rms": s_rms},
           "band_logits_at_tol": int(band_mask(ref64, tol).sum()),
           "band_logits_at_err": int(band_mask(ref64, band_tol).sum()),
           "band_shots_at_err": int(band_mask(ref64, band_tol).reshape(len(det), -1).any(1).sum()),
           "residual_mismatch_outside_band": residual_mismatch_outside_band(residual, res64, ref64, geo, band_tol),
           "residual_mismatch_total": int((np.asarray(residual) != np.asarray(res64)).sum()),
           "residual_is_own_xor": bool(np.array_equal(own, residual))}
    rep["pass"] = bool(err <= max(tol, 2 * s_max) and p999 <= max(tol, 2 * s_p999)
                       and rrms <= max(tol / 2, 2 * s_rms) and rep["residual_mismatch_outside_band"] == 0
                       and rep["residual_is_own_xor"])
    return rep


def band_mask(logits_ref: np.ndarray, tol: float) -> np.ndarray:
    """Data-node logits within tol x RMS of zero: their sign, and so the residual bits around them, may differ
    between two correct implementations."""
    rms = float(np.sqrt(np.mean(np.square(logits_ref)))) if logits_ref.size else 1.0
    return np.abs(logits_ref) < tol * max(rms, 1e-30)


def logit_error(logits: np.ndarray, logits_ref: np.ndarray) -> float:
    """max |a - b| / max(|b|, rms(b)) over all entries (a relative error that stays finite near zero)."""
    if logits_ref.size == 0:
        return 0.0
    rms = float(np.sqrt(np.mean(np.square(logits_ref))))
    den = np.maximum(np.abs(logits_ref), max(rms, 1e-30))
    return float(np.max(np.abs(logits - logits_ref) / den))


def residual_mismatch_outside_band(res, res_ref, logits_ref, geo, tol) -> int:
    """Residual bits that differ at checks none of whose cancelling data nodes lies in the band."""
    band = band_mask(logits_ref, tol)                     # (B, N_d, 2)
    B = res.shape[0]
    touched = np.zeros((B, geo.N_c), bool)
    nbr = geo.xor_nbr
    for j in range(2):
        for k in range(2):
            c = nbr[:, j, k]
            ok = c >= 0
            bi, ni = np.nonzero(band[:, ok, j])
            touched[bi, c[ok][ni]] = True
    diff = (np.asarray(res) != np.asarray(res_ref)) & ~touched
    return int(diff.sum())


def route(logits, residual, tau: float, route_residual: bool = True):
    """The routing rule restated (evaluation/convlines/decoder.py:116-142 `route`, with the pre-decoder's confidence):
    conf = min |logit| per shot, weight = set residual bits per shot, routed = conf < tau or (route_residual and
    weight > 0); the routed shots in ascending order and their residual rows -> (routed, index, handoff, conf,
    weight)."""
    lg = np.asarray(logits, np.float32)
    lg = lg.reshape(lg.shape[0], int(np.prod(lg.shape[1:])))
    rs = np.asarray(residual, np.uint8) & 1
    conf = np.abs(lg).min(1) if lg.shape[1] else np.full(len(lg), np.inf, np.float32)
    weight = rs.sum(1).astype(np.int32)
    routed = (conf < np.float32(tau)) | (bool(route_residual) & (weight > 0))
    index = np.flatnonzero(routed).astype(np.int64)
    return routed, index, np.asarray(residual, np.uint8)[index], conf.astype(np.float32), weight
