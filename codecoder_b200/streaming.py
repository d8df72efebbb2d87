"""Streaming pre-decoding: one new round of detectors per step, a sliding window of W rounds, batch 1.

Each step is one CUDA-graph replay on the decoder's stream:
  1. copy the new round's detectors in from pinned host memory (nh X detectors, nh Z detectors),
  2. form the next window: rounds 1 .. W-1 of the current window and the new round, one concatenation kernel into
     the other of two window buffers (two graphs, one per buffer, alternate),
  3. run the pre-decoder forward on the window (bpc_predecoder_forward: embed, 2L bipartite steps, head, residual),
  4. copy the newest round's X/Z logits and the window's residual syndrome out to pinned host memory in one copy
     (the forward writes them next to each other in one device buffer).
The graphs are captured once after a warm-up step, so a step costs one graph launch plus the device work.  A batch
of one shot runs the node-tiled kernels (gmm_nodes.cu: the MMA rows are target nodes; at C = 64 a cluster of 8
CTAs splits each 128-node tile by relation).  The window keeps the model's time boundary: the oldest round is t = 0
and the newest t = W - 1 (RotatedSurface(d, W)).
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
        self.win = [torch.zeros(1, g.N_c, dtype=torch.uint8, device=dev) for _ in range(2)]
        self.cur = 0                                     # which window buffer holds the current window
        # one device buffer: the logits (N_d x 2 fp32), then the residual (N_c bytes); its tail -- the newest round's
        # logits and the residual -- is one contiguous range, copied out in one piece
        nl = g.N_d * 2 * 4
        self._out = torch.empty(nl + g.N_c, dtype=torch.uint8, device=dev)
        self.logits = self._out[:nl].view(torch.float32).view(1, g.N_d, 2)
        self.residual = self._out[nl:].view(1, g.N_c)
        self._tail = self._out[(window - 1) * self.nq * 2 * 4:]
        self._tail_host = torch.zeros(self._tail.numel(), dtype=torch.uint8).pin_memory()
        self.lg_host = self._tail_host[:self.nq * 2 * 4].view(torch.float32).view(self.nq, 2)
        self.res_host = self._tail_host[self.nq * 2 * 4:].view(1, g.N_c)
        self.new_host = torch.zeros(2, 1, self.nh, dtype=torch.uint8).pin_memory()
        self.new_dev = torch.zeros(2, 1, self.nh, dtype=torch.uint8, device=dev)
        self.stream = torch.cuda.Stream(device=dev)
        self.graphs = None

    @property
    def det(self) -> torch.Tensor:
        """The current window (1, N_c) on the device."""
        return self.win[self.cur]

    def _round(self, src: int):
        W, nh = self.W, self.nh
        cur, nxt = self.win[src].view(2, W, nh), self.win[1 - src].view(2, W, nh)
        self.new_dev.copy_(self.new_host, non_blocking=True)
        torch.cat([cur[:, 1:], self.new_dev], dim=1, out=nxt)
        self.pd.forward_into(self.win[1 - src], self.logits, self.residual)
        self._tail_host.copy_(self._tail, non_blocking=True)

    def capture(self):
        """Warm up (first launches configure the kernels) and capture one graph per window buffer."""
        with torch.cuda.device(self.device), torch.cuda.stream(self.stream):
            self._round(0)
            self._round(1)
            self.stream.synchronize()
            for w in self.win:
                w.zero_()
            self.stream.synchronize()
            self.graphs = []
            for src in range(2):
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=self.stream):
                    self._round(src)
                self.graphs.append(g)
            self.stream.synchronize()            # this stream only: a resident kernel may run on another
        self.cur = 0

    def reset(self):
        with torch.cuda.device(self.device):
            for w in self.win:
                w.zero_()
            torch.cuda.synchronize(self.device)

    def step(self, new_round: np.ndarray):
        """new_round (2 nh,) uint8: this round's X then Z detectors -> (residual of the window (N_c,) uint8 view,
        logits of the newest round (d^2, 2) fp32 view), both in pinned host memory, valid until the next step."""
        if self.graphs is None:
            self.capture()
        self.new_host.view(-1).copy_(torch.from_numpy(np.asarray(new_round, np.uint8)))
        with torch.cuda.stream(self.stream):          # replay() launches on the current stream
            self.graphs[self.cur].replay()
        self.cur = 1 - self.cur
        self.stream.synchronize()
        return self.res_host[0], self.lg_host

    def latency(self, rounds: np.ndarray, warmup: int = 100):
        """Per-round latency in microseconds (host wall clock from handing the round over to having its results on
        the host) for rounds (R, 2 nh) uint8 -> np.ndarray (R - warmup,)."""
        if self.graphs is None:
            self.capture()
        out = []
        for i, r in enumerate(rounds):
            t0 = time.perf_counter()
            self.step(r)
            if i >= warmup:
                out.append((time.perf_counter() - t0) * 1e6)
        return np.asarray(out)


class PersistentStreamingDecoder:
    """The same sliding-window decoder served by one resident kernel (C ABI bpc_stream_*): rounds go in and results
    come out through a request line in mapped host memory, no launch per round.  bf16 networks with C = 64 and K = 8
    (the d = 17 streaming workload).  `layout`: "one_cluster" (one thread-block cluster of two CTAs per 128-node tile,
    16 SMs at d = 17, cluster barriers between the steps), "clusters" (8 clusters x 8 CTAs on 64 SMs, a grid barrier
    between the steps) or "auto" (the first where its cluster can be resident).  The kernel leaves after
    `idle_timeout_ms` without a request, on stop(), or when a wait inside a round exceeds its watchdog.  Same bits as StreamingDecoder
    (whose small-batch steps run the same relation-split arithmetic).  While it runs nothing may synchronise the
    whole device (torch.cuda.synchronize() would wait for the resident kernel until its idle limit): synchronise
    streams or events instead."""

    LAYOUTS = {"auto": 0, "clusters": 1, "one_cluster": 2}

    def __init__(self, d: int, window: int, cfg, params, device="cuda", idle_timeout_ms: int = 5000,
                 layout: str = "auto", trace: bool = False):
        import ctypes
        from . import _lib
        if layout not in self.LAYOUTS:
            raise ValueError(f"layout must be one of {sorted(self.LAYOUTS)}")
        self.geo = g = RotatedSurface(d, window)
        self.pd = PreDecoder(g, cfg, params, device=device, chunk_shots=256)
        self.device = self.pd.device
        self.W, self.nh, self.nq = window, g.nh, g.n_data_round
        h = ctypes.c_void_p()
        _lib.check(_lib.lib().bpc_stream_create_ex(self.pd._h, window, g.nh, g.n_data_round, int(idle_timeout_ms),
                                                   self.LAYOUTS[layout], ctypes.byref(h)), "bpc_stream_create_ex")
        self._s = h
        if trace:
            _lib.check(_lib.lib().bpc_stream_trace(h, 1), "bpc_stream_trace")
        self.residual = np.zeros(g.N_c, np.uint8)
        self.logits = np.zeros((self.nq, 2), np.float32)
        self.running = False

    def start(self):
        from . import _lib
        with torch.cuda.device(self.device):
            _lib.check(_lib.lib().bpc_stream_start(self._s), "bpc_stream_start")
        self.running = True

    def step(self, new_round: np.ndarray, timeout_us: int = 2_000_000):
        """new_round (2 nh,) uint8 -> (residual (N_c,) uint8, newest-round logits (nq, 2) fp32), host arrays valid
        until the next step."""
        from . import _lib
        if not self.running:
            self.start()
        r = np.ascontiguousarray(new_round, np.uint8)
        _lib.check(_lib.lib().bpc_stream_round(self._s, r.ctypes.data, self.residual.ctypes.data,
                                               self.logits.ctypes.data, int(timeout_us)), "bpc_stream_round")
        return self.residual, self.logits

    def latency(self, rounds: np.ndarray, warmup: int = 100, timeout_us: int = 2_000_000):
        """Per-round latency in microseconds (host wall clock in the library's own loop, from writing the request to
        reading the response) for rounds (R, 2 nh) uint8 -> np.ndarray (R - warmup,)."""
        from . import _lib
        if not self.running:
            self.start()
        rounds = np.ascontiguousarray(rounds, np.uint8)
        lat = np.zeros(len(rounds), np.int64)
        _lib.check(_lib.lib().bpc_stream_run(self._s, rounds.ctypes.data, len(rounds), None, None, lat.ctypes.data,
                                             int(timeout_us)), "bpc_stream_run")
        return lat[warmup:] / 1000.0

    def status(self) -> int:
        from . import _lib
        return int(_lib.lib().bpc_stream_status(self._s))

    def layout(self) -> str:
        """The layout of the kernel that runs or ran last ("clusters", "one_cluster"; "" before the first start)."""
        from . import _lib
        return {1: "clusters", 2: "one_cluster"}.get(int(_lib.lib().bpc_stream_layout(self._s)), "")

    PHASES = ("ready", "mma_issued", "accumulated", "exchanged", "epilogue", "barrier")

    def trace(self) -> np.ndarray:
        """After stop(), with trace=True: the global-timer stamps (ns) of the last round served, (64 CTAs, 16 slots,
        8) int64 -- slots 0 .. 2L - 2 the steps (start, weights / gathered rows ready, MMAs issued, accumulators
        ready, partials exchanged, epilogue done, past the barrier), slot 15 the round (waiting for the request,
        accepted, window embedded, past the barrier, published); 0 where a CTA did not pass."""
        from . import _lib
        out = np.zeros((64, 16, 8), np.uint64)
        _lib.check(_lib.lib().bpc_stream_trace_read(self._s, out.ctypes.data, out.size), "bpc_stream_trace_read")
        return out.astype(np.int64)

    def phase_table(self) -> dict:
        """Per step of the last round served, the median over the CTAs that worked on it of each phase's duration in
        ns (from the previous stamp; "barrier" from the end of the epilogue to past the barrier), and the step's
        critical path (start of the step to past its barrier, the same on every CTA)."""
        tr = self.trace()
        steps = []
        for st in range(2 * self.pd.cfg.layers - 1):
            x = tr[:, st]
            ok = (x[:, 0] > 0) & (x[:, 5] > 0) & (x[:, 3] > 0)
            if not ok.any():
                continue
            y = x[ok]
            d = np.diff(y[:, :7], axis=1)
            steps.append({"step": st, **{p: float(np.median(d[:, i])) for i, p in enumerate(self.PHASES)},
                          "total": float(np.median(y[:, 6] - y[:, 0])), "ctas": int(ok.sum())})
        r = tr[:, 15]
        r = r[r[:, 1] > 0]
        rnd = {"embed": float(np.median(r[:, 2] - r[:, 1]))}
        if (r[:, 3] > 0).all():                          # a barrier after the embedding (one-cluster layout)
            rnd["embed_barrier"] = float(np.median(r[:, 3] - r[:, 2]))
        r0 = tr[0, 15]
        if r0[4] > 0:
            rnd["publish"] = float(r0[4] - tr[0, 2 * self.pd.cfg.layers - 2, 6])
        return {"steps": steps, "round": rnd}

    def stop(self):
        from . import _lib
        if self.running:
            self.running = False
            _lib.check(_lib.lib().bpc_stream_stop(self._s), "bpc_stream_stop")

    def close(self):
        from . import _lib
        if getattr(self, "_s", None):
            try:
                self.stop()
            finally:
                _lib.lib().bpc_stream_destroy(self._s)
                self._s = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
