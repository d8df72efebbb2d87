"""Streaming pre-decoding: one new round of detectors per step, a sliding window of W rounds, batch 1.

Each step is one CUDA-graph replay on the decoder's stream:
  1. shift the device window one round (rounds 1 .. W-1 -> 0 .. W-2, for the X and the Z checks),
  2. copy the new round's detectors in from pinned host memory (nh X detectors, nh Z detectors),
  3. run the pre-decoder forward on the window (bpc_predecoder_forward: embed, 2L bipartite steps, head, residual),
  4. copy the window's residual syndrome and the newest round's X/Z logits out to pinned host memory.
The graph is captured once after a warm-up step, so a step costs one graph launch plus the device work.  A batch of
one shot runs the node-tiled kernels (the MMA rows are 128 target nodes, gmm_nodes.cu), which give the same bits as
the shot-tiled kernels of large batches.  The window keeps the model's time boundary: the oldest round is t = 0 and
the newest t = W - 1 (RotatedSurface(d, W)).
"""
from __future__ import annotations

import time

import numpy as np
import torch

from .geometry import RotatedSurface
from .modules import PreDecoder


class StreamingDecoder:
    def __init__(self, d: int, window: int, cfg, params, device="cuda"):
        self.geo = g = RotatedSurface(d, window)
        self.pd = PreDecoder(g, cfg, params, device=device, chunk_shots=256)
        self.device = dev = self.pd.device
        self.W, self.nh, self.nq = window, g.nh, g.n_data_round
        self.det = torch.zeros(1, g.N_c, dtype=torch.uint8, device=dev)
        self.det_next = torch.zeros_like(self.det)
        self.logits = torch.empty(1, g.N_d, 2, dtype=torch.float32, device=dev)
        self.residual = torch.empty(1, g.N_c, dtype=torch.uint8, device=dev)
        self.new_host = torch.zeros(2, self.nh, dtype=torch.uint8).pin_memory()
        self.new_dev = torch.zeros(2, self.nh, dtype=torch.uint8, device=dev)
        self.res_host = torch.zeros(1, g.N_c, dtype=torch.uint8).pin_memory()
        self.lg_host = torch.zeros(self.nq, 2, dtype=torch.float32).pin_memory()
        self.stream = torch.cuda.Stream(device=dev)
        self.graph = None

    def _work(self):
        W, nh = self.W, self.nh
        dn = self.det_next.view(2, W, nh)
        dc = self.det.view(2, W, nh)
        self.new_dev.copy_(self.new_host, non_blocking=True)
        dn[:, :W - 1].copy_(dc[:, 1:])
        dn[:, W - 1].copy_(self.new_dev)
        self.det.copy_(self.det_next)
        self.pd.forward_into(self.det, self.logits, self.residual)
        self.res_host.copy_(self.residual, non_blocking=True)
        self.lg_host.copy_(self.logits[0, (W - 1) * self.nq:], non_blocking=True)

    def capture(self):
        """Warm up (first launches configure the kernels) and capture one step as a CUDA graph."""
        with torch.cuda.device(self.device), torch.cuda.stream(self.stream):
            self._work()
            self.stream.synchronize()
            self.det.zero_()
            self.stream.synchronize()
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph, stream=self.stream):
                self._work()
        torch.cuda.synchronize(self.device)

    def reset(self):
        with torch.cuda.device(self.device):
            self.det.zero_()
            torch.cuda.synchronize(self.device)

    def step(self, new_round: np.ndarray):
        """new_round (2 nh,) uint8: this round's X then Z detectors -> (residual of the window (N_c,) uint8 view,
        logits of the newest round (d^2, 2) fp32 view), both in pinned host memory, valid until the next step."""
        if self.graph is None:
            self.capture()
        self.new_host.view(-1).copy_(torch.from_numpy(np.asarray(new_round, np.uint8)))
        self.graph.replay()
        self.stream.synchronize()
        return self.res_host[0], self.lg_host

    def latency(self, rounds: np.ndarray, warmup: int = 100):
        """Per-round latency in microseconds (host wall clock from handing the round over to having its results on
        the host) for rounds (R, 2 nh) uint8 -> np.ndarray (R - warmup,)."""
        if self.graph is None:
            self.capture()
        out = []
        for i, r in enumerate(rounds):
            t0 = time.perf_counter()
            self.step(r)
            if i >= warmup:
                out.append((time.perf_counter() - t0) * 1e6)
        return np.asarray(out)
