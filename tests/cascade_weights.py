"""Seeded weights for the Cascade network tests.

Every state_dict entry is drawn from numpy's default_rng seeded by (seed, CRC-32 of the entry's name), so the fixture
generator (tests/golden/make_golden.py, with the reference's CascadeBB) and the GPU test (with CascadeNet) rebuild the
same network without the fixture storing its weights.  Scales follow the modules' initialisations; the BatchNorm
statistics, the last MLP layer and a 4x larger scatter make the logits depend on the detectors (at initialisation
they barely do); the blocks' matrices are rounded to bf16, as the B200 path stores them."""
from __future__ import annotations

import zlib

import numpy as np


def _bf16(a: np.ndarray) -> np.ndarray:
    u = np.asarray(a, np.float32).view(np.uint32)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & np.uint32(0xFFFF0000)
    return u.view(np.float32)


def cascade_state(shapes: dict, seed: int) -> dict:
    """shapes: state_dict entry name -> shape (CascadeNet's or the reference CascadeBB's, the same names) ->
    name -> numpy array (float32; int64 for BatchNorm's num_batches_tracked)."""
    out = {}
    for name, shape in shapes.items():
        shape = tuple(int(s) for s in shape)
        rng = np.random.default_rng([seed, zlib.crc32(name.encode())])
        leaf = name.rsplit(".", 1)[-1]
        if leaf == "num_batches_tracked":
            out[name] = np.zeros(shape, np.int64)
            continue
        if leaf == "running_mean":
            v = rng.standard_normal(shape) * 0.1
        elif leaf == "running_var":
            v = rng.uniform(0.5, 2.0, shape)
        elif ".bn" in "." + name and leaf == "weight":
            v = rng.uniform(0.5, 1.5, shape)
        elif ".bn" in "." + name and leaf == "bias":
            v = rng.standard_normal(shape) * 0.1
        elif name == "embed.weight":
            v = rng.standard_normal(shape)
        elif name == "scatter":
            v = rng.standard_normal(shape) * 4.0 / np.sqrt(shape[1] / 2)
        elif name == "mlp2.weight":
            v = rng.standard_normal(shape)
        elif leaf == "bias":
            v = rng.standard_normal(shape) * 0.1
        else:                                       # linear and relation matrices: N(0, 1 / fan_in)
            v = rng.standard_normal(shape) / np.sqrt(shape[-1])
        v = np.asarray(v, np.float32)
        if name.startswith("blocks.") and len(shape) == 2:
            v = _bf16(v)
        out[name] = v
    return out
