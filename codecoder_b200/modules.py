"""Modules on the B200 kernels: BipartiteConv (drop-in for the reference's module) and PreDecoder.

CascadeBlock(H, geo, L, res, impl) is the reference's bottleneck residual block (cascade_net.py:236-259) on the same op.

BipartiteConv(C, geo, impl) keeps the reference's constructor, parameter names (w_c2d, w_d2c: one (C, K C) matrix per
target type), registered tables (c2d{k}, inv_c2d{k}, d2c{k}, inv_d2c{k}) and forward (cascade_net.py:213-233).  It
takes the reference's Geometry (BB codes, K = 12) or geometry.RotatedSurface (K = 8).

PreDecoder(geo, cfg, params) runs the whole rotated-surface pre-decoder (params.py) in one C-ABI call per batch:
forward(det) -> (logits (B, N_d, 2) fp32, residual (B, N_c) uint8).
"""
from __future__ import annotations

import ctypes
import math

import numpy as np
import torch
import torch.nn.functional as F
from torch import nn

from . import _lib
from .ops import gather_mm, residual_affine_silu


class BipartiteConv(nn.Module):
    """check -> data -> check at width C, linear and bias-free (cascade_net.py:213-233).  impl is kept for the
    reference's signature; every impl runs the B200 kernels."""

    def __init__(self, C, geo, impl="b200"):
        super().__init__()
        self.C, self.impl = C, impl
        K = int(np.asarray(geo.c2d[0]).shape[1])
        self.K = K
        std = 1 / math.sqrt(K * C)
        self.w_c2d = nn.ParameterList([nn.Parameter(torch.randn(C, K * C) * std) for _ in range(len(geo.c2d))])
        self.w_d2c = nn.ParameterList([nn.Parameter(torch.randn(C, K * C) * std) for _ in range(len(geo.d2c))])
        for name in ("c2d", "d2c"):
            for k in range(len(getattr(geo, name))):
                self.register_buffer(f"{name}{k}", torch.as_tensor(np.asarray(getattr(geo, name)[k])),
                                     persistent=False)
                self.register_buffer(f"inv_{name}{k}", torch.as_tensor(np.asarray(getattr(geo, "inv_" + name)[k])),
                                     persistent=False)

    def forward(self, x):                               # (B, N checks, C) -> (B, N checks, C)
        data = torch.cat([gather_mm(x, self.w_c2d[d], getattr(self, f"c2d{d}"), getattr(self, f"inv_c2d{d}"))
                          for d in range(len(self.w_c2d))], 1)
        return torch.cat([gather_mm(data, self.w_d2c[c], getattr(self, f"d2c{c}"), getattr(self, f"inv_d2c{c}"))
                          for c in range(len(self.w_d2c))], 1)


class PreDecoder:
    """The rotated-surface pre-decoder on one GPU through libbpc.so (bpc_predecoder_*).

    geo: geometry.RotatedSurface; cfg: params.PreDecoderConfig; params: params.init_params-style dict (fp32 numpy).
    chunk_shots: shots per pass through the network (sets the workspace: 2 x (N_c + N_d) x C activations)."""

    def __init__(self, geo, cfg, params, device=None, chunk_shots: int = 16384):
        self.geo, self.cfg = geo, cfg
        self.device = torch.device(device if device is not None else "cuda")
        if self.device.type != "cuda":
            raise RuntimeError("PreDecoder runs on a CUDA device only (no CPU path)")
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        if cfg.K != geo.K or cfg.d != geo.d or cfg.rounds != geo.R:
            raise ValueError("configuration and geometry disagree")
        self.dtype = _lib.BPC_DTYPE_BF16 if cfg.dtype == "bf16" else _lib.BPC_DTYPE_F32
        L = _lib.lib()
        c = _lib.PredecoderConfig(cfg.layers, cfg.channels, cfg.K, self.dtype, geo.N_c, geo.N_d, geo.T * geo.nh)
        self._keep = {
            "c2d": np.ascontiguousarray(geo.c2d[0], np.int32),
            "d2c": np.ascontiguousarray(geo.d2c_all, np.int32),
            "xor": np.ascontiguousarray(geo.xor_nbr, np.int32),
            "ctype": np.ascontiguousarray(geo.check_type, np.uint8),
            "order": np.ascontiguousarray(geo.check_round_order, np.int32),
        }
        h = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            _lib.check(L.bpc_predecoder_create(ctypes.byref(c), *(a.ctypes.data for a in self._keep.values()),
                                               ctypes.byref(h)), "bpc_predecoder_create")
        self._h = h
        self.set_weights(params)
        self.chunk_shots = int(chunk_shots)
        self._ws = None

    def set_weights(self, params: dict) -> None:
        cfg = self.cfg

        def conv(a):
            t = torch.as_tensor(np.ascontiguousarray(a, np.float32))
            if cfg.dtype == "bf16":
                return t.to(torch.bfloat16).contiguous()
            return t.contiguous()

        emb = conv(params["embed"])
        wc = conv(np.asarray(params["w_c2d"]).reshape(cfg.layers, cfg.channels, cfg.K * cfg.channels))
        wd = conv(np.asarray(params["w_d2c"]).reshape(cfg.layers, 2, cfg.channels, cfg.K * cfg.channels))
        hw = np.ascontiguousarray(params["head_w"], np.float32)
        hb = np.ascontiguousarray(params["head_b"], np.float32)
        with torch.cuda.device(self.device):
            _lib.check(_lib.lib().bpc_predecoder_set_weights(self._h, emb.data_ptr(), wc.data_ptr(), wd.data_ptr(),
                                                             hw.ctypes.data, hb.ctypes.data),
                       "bpc_predecoder_set_weights")

    def workspace_bytes(self, shots: int) -> int:
        return int(_lib.lib().bpc_predecoder_workspace_size(self._h, int(shots)))

    def _workspace(self, B: int) -> torch.Tensor:
        want = self.workspace_bytes(min(max(B, 1), self.chunk_shots))
        if self._ws is None or self._ws.numel() < want:
            self._ws = torch.empty(want, dtype=torch.uint8, device=self.device)
        return self._ws

    def forward_into(self, det: torch.Tensor, logits: torch.Tensor, residual: torch.Tensor) -> None:
        """det (B, N_c) uint8 -> logits (B, N_d, 2) fp32, residual (B, N_c) uint8, all on this device."""
        B = det.shape[0]
        for t, shape, dt in ((det, (B, self.geo.N_c), torch.uint8), (logits, (B, self.geo.N_d, 2), torch.float32),
                             (residual, (B, self.geo.N_c), torch.uint8)):
            if t.device != self.device or tuple(t.shape) != shape or t.dtype != dt or not t.is_contiguous():
                raise ValueError(f"expected a contiguous {dt} tensor {shape} on {self.device}")
        if B == 0:
            return
        ws = self._workspace(B)
        rc = _lib.lib().bpc_predecoder_forward(self._h, det.data_ptr(), logits.data_ptr(), residual.data_ptr(), B,
                                               ws.data_ptr(), ws.numel(),
                                               torch.cuda.current_stream(self.device).cuda_stream)
        _lib.check(rc, "bpc_predecoder_forward")

    def forward(self, det: torch.Tensor):
        """det (B, N_c) uint8 on this device -> (logits (B, N_d, 2) fp32, residual (B, N_c) uint8)."""
        det = det.to(self.device, torch.uint8).contiguous()
        B = det.shape[0]
        logits = torch.empty(B, self.geo.N_d, 2, dtype=torch.float32, device=self.device)
        residual = torch.empty(B, self.geo.N_c, dtype=torch.uint8, device=self.device)
        self.forward_into(det, logits, residual)
        return logits, residual

    __call__ = forward

    def forward_host(self, det_host: torch.Tensor, logits_host: torch.Tensor, residual_host: torch.Tensor,
                     slice_shots: int | None = None) -> None:
        """Host buffers in, host buffers out (pinned memory): det (B, N_c) uint8 -> logits (B, N_d, 2) fp32,
        residual (B, N_c) uint8.  The batch goes through in slices of `slice_shots` (default: the pass size) with two
        device buffer sets: the next slice's detectors go up on one copy stream while the current slice runs, and the
        finished slice's results come down on another, so the forward passes follow one another without waiting for
        the copies.  Synchronises before returning."""
        B = det_host.shape[0]
        if B == 0:
            return
        for t in (det_host, logits_host, residual_host):
            if t.device.type != "cpu" or not t.is_contiguous():
                raise ValueError("forward_host takes contiguous host tensors (pinned for overlap)")
        S = int(slice_shots or self.chunk_shots)
        S = max(256, (S // 256) * 256)
        dev = self.device
        bufs = getattr(self, "_host_bufs", None)
        if bufs is None or bufs[0][0].shape[0] < S:
            bufs = [(torch.empty(S, self.geo.N_c, dtype=torch.uint8, device=dev),
                     torch.empty(S, self.geo.N_d, 2, dtype=torch.float32, device=dev),
                     torch.empty(S, self.geo.N_c, dtype=torch.uint8, device=dev)) for _ in range(2)]
            self._host_bufs = bufs
            self._copy_streams = (torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev))
        comp = torch.cuda.current_stream(dev)
        up, down = self._copy_streams
        starts = list(range(0, B, S))
        ready = [None, None]                    # event: the slice's detectors are on the device
        done = [None, None]                     # event: the slice buffers are free again (results copied out)

        def upload(i):
            b0, k = starts[i], i % 2
            n = min(S, B - b0)
            with torch.cuda.stream(up):
                if done[k] is not None:
                    up.wait_event(done[k])
                bufs[k][0][:n].copy_(det_host[b0:b0 + n], non_blocking=True)
                ready[k] = torch.cuda.Event()
                ready[k].record(up)

        with torch.cuda.device(dev):
            upload(0)
            for i, b0 in enumerate(starts):
                n = min(S, B - b0)
                k = i % 2
                d_det, d_lg, d_rs = (t[:n] for t in bufs[k])
                comp.wait_event(ready[k])
                self.forward_into(d_det, d_lg, d_rs)
                computed = torch.cuda.Event()
                computed.record(comp)
                if i + 1 < len(starts):
                    upload(i + 1)               # overlaps this slice's forward pass
                with torch.cuda.stream(down):
                    down.wait_event(computed)
                    logits_host[b0:b0 + n].copy_(d_lg, non_blocking=True)
                    residual_host[b0:b0 + n].copy_(d_rs, non_blocking=True)
                    done[k] = torch.cuda.Event()
                    done[k].record(down)
            comp.wait_stream(down)
        torch.cuda.synchronize(dev)

    def record_step_events(self, pairs) -> None:
        """pairs: list of (start, end) torch.cuda.Event(enable_timing=True); the next forward calls record them
        around their bipartite-step launches in launch order (empty list: off)."""
        flat = [e for pr in pairs for e in pr]
        for e in flat:
            e.record()                                   # make torch create the underlying CUDA event
        torch.cuda.synchronize(self.device)
        arr = (ctypes.c_void_p * max(1, len(flat)))(*[e.cuda_event for e in flat])
        _lib.check(_lib.lib().bpc_predecoder_record_step_events(self._h, arr, len(pairs)),
                   "bpc_predecoder_record_step_events")
        self._step_events = flat

    def status(self) -> int:
        """Device watchdog status (0 = every wait completed); synchronises the current stream, raises otherwise."""
        s = ctypes.c_int(0)
        rc = _lib.lib().bpc_predecoder_status(self._h, torch.cuda.current_stream(self.device).cuda_stream,
                                              ctypes.byref(s))
        _lib.check(rc, "bpc_predecoder_status")
        return s.value

    def close(self) -> None:
        if getattr(self, "_h", None):
            _lib.lib().bpc_predecoder_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def _fold_bn(bn: nn.BatchNorm1d):
    """Inference BatchNorm as a per-channel affine map: (scale, shift) fp32 with bn(x) = scale x + shift."""
    scale = bn.weight.float() / torch.sqrt(bn.running_var.float() + bn.eps)
    return scale, bn.bias.float() - bn.running_mean.float() * scale


class CascadeBlock(nn.Module):
    """The reference's bottleneck residual block (cascade_net.py:236-259) on the B200 op, with its parameter names
    (bn1, bn2, bn3, down, conv, up) so its state_dicts load unchanged:
        u = up(SiLU(BN3(conv(SiLU(BN2(down(SiLU(BN1(h)))))))));  h' = h + u / sqrt(2L) (res 'branch') or
        h / sqrt(2L) + u (res 'skip'),  H -> H / 4 in the bottleneck.
    Training: the reference's composition (batch statistics over every node of every shot, cascade_net.py:195-210),
    the convolution through gather_mm (forward and backward on the B200 kernels).
    Eval: the fused inference path on the folded BatchNorms --
        BN1 + SiLU: one elementwise pass;  down + BN2 + SiLU: the op with K = 1 (identity table) and the affine + SiLU
        epilogue;  conv: two launches, each covering both target types (stacked relation matrices, the targets are
        type-major);  BN3 + SiLU: the epilogue of the second;  up and the residual: one bf16 GEMM and one fp32 add.
    The bottleneck activations are bf16 (the reference's bf16 autocast), the residual stream keeps h's dtype."""

    def __init__(self, H, geo, L, res="branch", impl="b200"):
        super().__init__()
        Hb = H // 4
        self.bn1, self.bn2, self.bn3 = nn.BatchNorm1d(H), nn.BatchNorm1d(Hb), nn.BatchNorm1d(Hb)
        self.down = nn.Linear(H, Hb, bias=False)
        self.conv = BipartiteConv(Hb, geo, impl)
        self.up = nn.Linear(Hb, H, bias=False)
        for lin in (self.down, self.up):
            nn.init.normal_(lin.weight, std=1 / math.sqrt(lin.in_features))
        self.res, self.scale = res, 1 / math.sqrt(2 * L)
        n_data = int(np.asarray(geo.c2d[0]).shape[0])
        n_chk = int(np.asarray(geo.d2c[0]).shape[0])
        self._splits = (n_data, n_chk)
        self.register_buffer("c2d_all", torch.as_tensor(np.concatenate([np.asarray(t) for t in geo.c2d]), dtype=torch.int32),
                             persistent=False)
        self.register_buffer("d2c_all", torch.as_tensor(np.concatenate([np.asarray(t) for t in geo.d2c]), dtype=torch.int32),
                             persistent=False)
        self._cache = None

    def _bn(self, mod, x):
        C = x.shape[-1]
        return mod(x.reshape(-1, C)).view(x.shape)

    def branch(self, h):
        u = self.down(F.silu(self._bn(self.bn1, h)))
        u = self.conv(F.silu(self._bn(self.bn2, u)))
        return self.up(F.silu(self._bn(self.bn3, u)))

    def prepare_inference(self):
        """Fold the BatchNorms and cast the weights once (call again after changing weights or statistics)."""
        with torch.no_grad():
            a1, b1 = _fold_bn(self.bn1)
            a2, b2 = _fold_bn(self.bn2)
            a3, b3 = _fold_bn(self.bn3)
            bf = torch.bfloat16
            self._cache = dict(a1=a1, b1=b1, a2=a2, b2=b2, a3=a3, b3=b3,
                               down=self.down.weight.to(bf).contiguous(), up=self.up.weight.to(bf).contiguous(),
                               wc=torch.stack([w.to(bf) for w in self.conv.w_c2d]).contiguous(),
                               wd=torch.stack([w.to(bf) for w in self.conv.w_d2c]).contiguous(),
                               ident=torch.zeros(0, dtype=torch.int32))
        return self

    def _fused(self, h, x1=None, nxt=None):
        """h (B, N, H) fp32 -> (h', SiLU(BN1 of `nxt`)(h') bf16 or None).  x1: this block's SiLU(BN1(h)) if the
        previous block already produced it."""
        from .ops import gmm_ex, residual_affine_silu
        c = self._cache
        B, N, H = h.shape
        if c["ident"].numel() != N or c["ident"].device != h.device:
            c["ident"] = torch.arange(N, dtype=torch.int32, device=h.device).view(N, 1)
        if x1 is None:
            _, x1 = residual_affine_silu(h, None, 1.0, 0.0, c["a1"], c["b1"], want_out=False)
        x2 = gmm_ex(x1, c["ident"], c["down"], scale=c["a2"], shift=c["b2"])
        d = gmm_ex(x2, self.c2d_all, c["wc"], type_split=self._splits[0])
        x3 = gmm_ex(d, self.d2c_all, c["wd"], type_split=self._splits[1], scale=c["a3"], shift=c["b3"])
        u = torch.matmul(x3, c["up"].t())
        sh, su = (1.0, self.scale) if self.res == "branch" else (self.scale, 1.0)
        a_n = b_n = None
        if nxt is not None:
            if nxt._cache is None or nxt._cache["a1"].device != h.device:
                nxt.prepare_inference()
            a_n, b_n = nxt._cache["a1"], nxt._cache["b1"]
        return residual_affine_silu(h, u, sh, su, a_n, b_n)

    def forward(self, h):
        if not self.training and h.is_cuda and h.dtype == torch.float32:
            if self._cache is None or self._cache["a1"].device != h.device:
                self.prepare_inference()
            return self._fused(h)[0]
        u = self.branch(h)
        if self.res == "branch":
            return h + self.scale * u
        return self.scale * h + u


class CascadeStack(nn.Module):
    """A sequence of CascadeBlocks (the reference CascadeBB's `blocks`, cascade_net.py:319-343).  In eval mode on the
    GPU the blocks hand over their fp32 residual stream and the next block's SiLU(BN1(.)) input in one pass each."""

    def __init__(self, blocks):
        super().__init__()
        self.blocks = nn.ModuleList(blocks)

    def forward(self, h):
        if self.training or not h.is_cuda or h.dtype != torch.float32:
            for b in self.blocks:
                h = b(h)
            return h
        return CascadeStack.forward_blocks(self.blocks, h)[0]

    @staticmethod
    def boundary_path(blocks) -> bool:
        """Blocks of H = 512 with a 128-channel bottleneck (the reference's C14 and C6 blocks) take the one-launch
        block boundary."""
        return all(tuple(b.up.weight.shape) == (512, 128) for b in blocks)

    @staticmethod
    def forward_blocks(blocks, h, final=None, tokens=None):
        """The fused inference path over a sequence of CascadeBlocks (eval mode, fp32 h on the GPU) -> (h, x): the
        residual stream after the last block, and with `final` = (scale, shift) of a folded BatchNorm, x =
        bf16(SiLU(scale h + shift)) (then h is None: a caller that asks for x needs only x).
        Blocks of H = 512 with a 128-channel bottleneck (the reference's C14 blocks) hand over in one launch per block
        boundary (bpc_cascade_boundary: up, residual, the next block's BN1 + SiLU, down and BN2 + SiLU); other sizes
        run the block-by-block fused path."""
        dev = h.device if h is not None else tokens[3].device
        for b in blocks:
            if b._cache is None or b._cache["a1"].device != dev:
                b.prepare_inference()
        if CascadeStack.boundary_path(blocks):
            return CascadeStack._forward_boundaries(blocks, h, final, tokens)
        if h is None:
            raise ValueError("forward_blocks: the token source needs blocks of the boundary path")
        x = None
        for i, b in enumerate(blocks):
            nxt = blocks[i + 1] if i + 1 < len(blocks) else None
            h, x = b._fused(h, x, nxt)
        if final is None:
            return h, None
        _, x = residual_affine_silu(h.contiguous(), None, 1.0, 0.0, final[0], final[1], want_out=False)
        return None, x

    @staticmethod
    def _forward_boundaries(blocks, h, final, tokens=None):
        """tokens = (det (B, D) uint8, gidx (N), tbase (N), E (5, H)): the stream before the first block is the
        embedding of the detector tokens, which the first block's kernels compute where they read it (bpc_cascade_stem,
        bpc_cascade_boundary_tokens) instead of it being written and read back."""
        from .ops import cascade_boundary, cascade_boundary_tokens, cascade_stem, gmm_ex
        c = blocks[0]._cache
        if tokens is None:
            h = h.contiguous()
            N, dev = h.shape[1], h.device
            _, x1 = residual_affine_silu(h, None, 1.0, 0.0, c["a1"], c["b1"], want_out=False)
        else:
            det, gidx, tbase, E = tokens
            N, dev = gidx.shape[0], E.device
            x1 = cascade_stem(det, gidx, tbase, E, c["a1"], c["b1"])
        if c["ident"].numel() != N or c["ident"].device != dev:
            c["ident"] = torch.arange(N, dtype=torch.int32, device=dev).view(N, 1)
        x2 = gmm_ex(x1, c["ident"], c["down"], scale=c["a2"], shift=c["b2"])
        stream, x = h, None
        for i, b in enumerate(blocks):
            c = b._cache
            d = gmm_ex(x2, b.c2d_all, c["wc"], type_split=b._splits[0])
            x3 = gmm_ex(d, b.d2c_all, c["wd"], type_split=b._splits[1], scale=c["a3"], shift=c["b3"])
            sh, su = (1.0, b.scale) if b.res == "branch" else (b.scale, 1.0)
            if i == 0 and tokens is not None:
                last = len(blocks) == 1
                n = None if last else blocks[1]._cache
                if not last:
                    stream, x2 = cascade_boundary_tokens(x3, c["up"], *tokens, sh, su, n["a1"], n["b1"], n["down"],
                                                         n["a2"], n["b2"])
                elif final is None:
                    stream, _ = cascade_boundary_tokens(x3, c["up"], *tokens, sh, su, want_y=False)
                else:
                    _, x = cascade_boundary_tokens(x3, c["up"], *tokens, sh, su, final[0], final[1], want_h=False)
                continue
            out = torch.empty_like(h) if stream is h else stream      # the caller's h is never written
            if i + 1 < len(blocks):
                n = blocks[i + 1]._cache
                stream, x2 = cascade_boundary(x3, c["up"], stream, sh, su, n["a1"], n["b1"], n["down"], n["a2"],
                                              n["b2"], h_out=out)
            elif final is None:
                stream, _ = cascade_boundary(x3, c["up"], stream, sh, su, h_out=out, want_y=False)
            else:
                _, x = cascade_boundary(x3, c["up"], stream, sh, su, final[0], final[1], h_out=None)
                stream = None
        return stream, x


class CascadeNet(nn.Module):
    """The reference's whole Cascade network for a BB code memory, CascadeBB (cascade_net.py:262-343): detector bits
    (B, D) -> one logit per observable (B, k), with its parameter names (embed, blocks.*, bn_out, scatter, mlp1,
    mlp2) so its state_dicts load unchanged.

    geo: the code's Tanner-graph tables with T, n2, N, c2d / d2c (per data / check type, (T n2, 12)) and their
    inverses, as the reference's Geometry gives them; det_t / det_typ / det_site: each detector's place; logicals
    (k, 2 n2): the observables' supports on the data qubits.
      stem      token = 2 type + bit at every detector's node, 4 at nodes without a detector; Embedding(5, H)
      blocks    L CascadeBlocks (the fused inference path of CascadeStack in eval mode on the GPU)
      read-out  SiLU(bn_out(h)); per observable the pooled sources of its support's check -> data relations
                (a fixed (24 k, N) pooling matrix), the scatter projection (24 H -> H), mlp1, SiLU, mlp2
    Eval on the GPU: the blocks on the B200 kernels (with C14-size blocks the embedded stream is never written: the
    stem and the first block's kernels read the embedding table by token, and the last block boundary writes
    SiLU(bn_out(h))); the read-out's pooling and scatter are plain dense GEMMs (cuBLAS) in bf16 as under the
    reference's autocast, its MLP in fp32."""

    def __init__(self, geo, H, L, det_t, det_typ, det_site, logicals, res="branch"):
        super().__init__()
        if H % 4:
            raise ValueError("H must be a multiple of 4")
        self.H, self.L = H, L
        T, n2, N = int(geo.T), int(geo.n2), int(geo.N)
        det_t, det_typ, det_site = (np.asarray(a, np.int64) for a in (det_t, det_typ, det_site))
        self.D = D = len(det_t)
        node = (det_typ * T + det_t) * n2 + det_site
        if len(np.unique(node)) != D or node.max() >= N:
            raise ValueError("detector places collide or fall outside the grid")
        gidx = np.full(N, D, np.int64)
        gidx[node] = np.arange(D)
        tbase = np.full(N, 4, np.int64)               # the "absent" token
        tbase[node] = 2 * det_typ
        self.register_buffer("gidx", torch.as_tensor(gidx), persistent=False)
        self.register_buffer("tbase", torch.as_tensor(tbase), persistent=False)
        self.embed = nn.Embedding(5, H)
        self.blocks = nn.ModuleList([CascadeBlock(H, geo, L, res) for _ in range(L)])
        self.bn_out = nn.BatchNorm1d(H)
        logicals = np.asarray(logicals, np.int64)
        self.k = k = len(logicals)
        self.support = [np.flatnonzero(r) for r in logicals]      # each observable's data qubits, d n2 + s
        K = int(np.asarray(geo.c2d[0]).shape[1])
        pool = np.zeros((k, 2, K, N + 1))
        for o in range(k):
            sup = np.flatnonzero(logicals[o])
            w = 1.0 / (T * len(sup))
            for q in sup:
                d, s = divmod(int(q), n2)
                for t in range(T):
                    np.add.at(pool[o, d], (np.arange(K), np.asarray(geo.c2d[d])[t * n2 + s]), w)
        self.register_buffer("pool", torch.as_tensor(pool[..., :N].reshape(k * 2 * K, N), dtype=torch.float32),
                             persistent=False)
        self.scatter = nn.Parameter(torch.randn(H, 2 * K * H) / math.sqrt(K * H))
        self.mlp1 = nn.Linear(H, 2 * H)
        self.mlp2 = nn.Linear(2 * H, 1)
        self._tables = None                         # int32 copies of gidx / tbase for the kernels

    def tokens(self, det: torch.Tensor) -> torch.Tensor:
        det = F.pad(det.to(torch.uint8), (0, 1))
        return self.tbase + det[:, self.gidx].long()

    def readout(self, x: torch.Tensor, dt: torch.dtype | None = None) -> torch.Tensor:
        """x = SiLU(bn_out(h)) (B, N, H) -> (B, k): the pooling and scatter GEMMs in dt (x's dtype by default), the
        observables' MLP (k rows per shot, a negligible share of the work) in fp32."""
        B, dt = x.shape[0], dt or x.dtype
        pooled = torch.matmul(self.pool.to(dt), x.to(dt))                      # (B, 24 k, H)
        z = (pooled.view(B, self.k, self.scatter.shape[1]) @ self.scatter.t().to(dt)).float()     # (B, k, H)
        return self.mlp2(F.silu(self.mlp1(z))).squeeze(-1)

    def forward(self, det: torch.Tensor) -> torch.Tensor:
        if self.training or not det.is_cuda:
            h = self.embed(self.tokens(det))
            for b in self.blocks:
                h = b(h)
            return self.readout(F.silu(self.bn_out(h.reshape(-1, self.H)).view(h.shape)))
        if CascadeStack.boundary_path(self.blocks):
            # the stem's embedding is computed by the first block's kernels, never written
            if self._tables is None or self._tables[0].device != det.device:
                self._tables = (self.gidx.to(torch.int32), self.tbase.to(torch.int32))
            tokens = (det.to(torch.uint8).contiguous(), *self._tables, self.embed.weight.float().contiguous())
            _, x = CascadeStack.forward_blocks(self.blocks, None, final=_fold_bn(self.bn_out), tokens=tokens)
        else:
            h = self.embed(self.tokens(det))
            _, x = CascadeStack.forward_blocks(self.blocks, h.float().contiguous(), final=_fold_bn(self.bn_out))
        return self.readout(x, torch.bfloat16)
