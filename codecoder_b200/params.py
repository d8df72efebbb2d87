"""Pre-decoder configuration and seeded weights.

The network (a rotated-surface variant of the reference's bipartite convolution, cascade_net.py:213-233):
  tokens   tok[c] = 2 type(c) + det[c]           (the reference's detector tokens, cascade_net.py:44,310-312)
  embed    h_c = E[tok]  (4, C);  h_d = 0
  layer l  h_d <- h_d + GELU(gather_mm(h_c, Wc2d[l], c2d))                  check -> data, one data type
           h_c <- h_c + GELU(gather_mm(h_d, Wd2c[l, type], d2c[type]))      data -> check, per check type X / Z
           GELU is the tanh form, 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))) (torch's approximate='tanh')
  head     logits[n] = Wh h_d[n] + bh   (N_d, 2): predicted X / Z flip of data node n
  cancel   e = logits > 0;  residual[c] = det[c] ^ XOR of e[q, 1 - type(c)] over the data qubits q around c at
           the same round (geometry.RotatedSurface.xor_nbr)
Relation weights are (C_out, K C_in) as in the reference (cascade_net.py:221-222), bias-free.  The head reads h_d after
the last layer's check -> data step; the last data -> check step still runs and gives the final check features.

Weights are drawn from numpy's default_rng(seed) with torch's default Linear bound 1 / sqrt(fan_in) (uniform);
the embedding is N(0, 1) like nn.Embedding.
"""
from __future__ import annotations

import dataclasses
import math

import numpy as np


@dataclasses.dataclass(frozen=True)
class PreDecoderConfig:
    d: int
    rounds: int
    layers: int
    channels: int
    dtype: str = "bf16"          # "bf16" (bf16 storage, fp32 accumulate) or "f32"
    K: int = 8
    p: float = 0.005

    @property
    def name(self) -> str:
        return f"d{self.d}_R{self.rounds}_L{self.layers}_C{self.channels}_{self.dtype}"


# The workloads the path is specified on (rotated surface code, phenomenological noise).
CONFIGS = {
    "d5_fp32": PreDecoderConfig(d=5, rounds=5, layers=4, channels=32, dtype="f32", p=0.003),
    "d9_bf16": PreDecoderConfig(d=9, rounds=9, layers=6, channels=64, dtype="bf16", p=0.005),
    "d13_bf16": PreDecoderConfig(d=13, rounds=13, layers=8, channels=128, dtype="bf16", p=0.005),
    "d17_stream": PreDecoderConfig(d=17, rounds=3, layers=6, channels=64, dtype="bf16", p=0.003),
    "d11_train": PreDecoderConfig(d=11, rounds=11, layers=6, channels=96, dtype="bf16", p=0.005),
}

N_TOKENS = 4


def init_params(cfg: PreDecoderConfig, seed: int) -> dict:
    """Seeded float32 weights: embed (4, C), w_c2d (L, 1, C, K C), w_d2c (L, 2, C, K C), head_w (2, C), head_b (2,)."""
    rng = np.random.default_rng(seed)
    C, K, L = cfg.channels, cfg.K, cfg.layers
    b = 1.0 / math.sqrt(K * C)
    bh = 1.0 / math.sqrt(C)
    return {
        "embed": rng.standard_normal((N_TOKENS, C)).astype(np.float32),
        "w_c2d": rng.uniform(-b, b, (L, 1, C, K * C)).astype(np.float32),
        "w_d2c": rng.uniform(-b, b, (L, 2, C, K * C)).astype(np.float32),
        "head_w": rng.uniform(-bh, bh, (2, C)).astype(np.float32),
        "head_b": rng.uniform(-bh, bh, (2,)).astype(np.float32),
    }


def round_bf16(a: np.ndarray) -> np.ndarray:
    """Round float32 to the nearest bfloat16 (ties to even), returned as float32."""
    a = np.ascontiguousarray(a, np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    out = r.astype(np.uint32).view(np.float32)
    return np.where(np.isnan(a), a, out)


def storage_params(cfg: PreDecoderConfig, params: dict) -> dict:
    """The weights as the device holds them: relation weights and the embedding rounded to bf16 for a bf16 network
    (the head stays fp32)."""
    if cfg.dtype == "f32":
        return {k: np.asarray(v, np.float32) for k, v in params.items()}
    out = dict(params)
    for k in ("embed", "w_c2d", "w_d2c"):
        out[k] = round_bf16(params[k])
    return out


def flops_per_shot(cfg: PreDecoderConfig, N_c: int, N_d: int) -> float:
    """Algorithmic FLOPs per shot, every relation slot counted (pads included), as the reference's macs_per_shot
    convention (cascade_net.py:369-374): L 2 K C^2 (N_c + N_d) + the head 2 2 C N_d."""
    C, K, L = cfg.channels, cfg.K, cfg.layers
    return float(L * 2 * K * C * C * (N_c + N_d) + 2 * 2 * C * N_d)
