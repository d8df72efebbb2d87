"""Training step of the rotated-surface pre-decoder on the B200 gather_mm op (forward and backward kernels).

PreDecoderNet is the network of params.py as an nn.Module over (B, N, C) row-layout features:
  h_c = E[2 type + det];  per layer  h_d (+)= GELU(gather_mm(h_c, Wc2d[l], c2d, inv_c2d))
                                     h_c += GELU(cat_type gather_mm(h_d, Wd2c[l, type], d2c[type], inv_d2c[type]))
  logits = h_d Wh^T + bh  (B, N_d, 2): predicted X / Z flip of every data node
with gather_mm the autograd Function of ops.py (cascade_net.py:140-175 / cascade_triton.py:161-186): its forward,
input gradient and weight gradient all run on the tcgen05 kernels under bf16 autocast.

Trainer.step is the reference's optimisation step (training/bb/ising_compare/bb/cascade_train.py:292-320), with the
optimiser of the training workload (Adam) in place of the reference's Muon / Lion pair: bf16 autocast forward,
binary cross-entropy with logits against the sampled data-qubit error labels, backward, gradient-norm clipping,
optimiser step.  With world > 1 the model is wrapped in DistributedDataParallel(broadcast_buffers=False) (NCCL
all-reduce of the gradients, cascade_train.py:243-245), and Trainer.agree takes the MAX of the per-rank
stop / non-finite flags so that every rank takes the same decision (cascade_train.py:387-391).
"""
from __future__ import annotations

import math
from contextlib import nullcontext

import numpy as np
import torch
import torch.nn.functional as F
from torch import nn

from .ops import bipartite_step, embed_tokens, gather_mm, head_bce, target_table
from .params import N_TOKENS


class PreDecoderNet(nn.Module):
    """geo: geometry.RotatedSurface; cfg: params.PreDecoderConfig; params: optional init_params-style dict (fp32
    numpy) to start from, else a seeded init with the same bounds.  `gmm` is the bipartite-conv op with the
    reference's signature gmm(x, w, idx, inv) (default: the B200 op)."""

    def __init__(self, geo, cfg, params: dict | None = None, gmm=gather_mm, seed: int = 0, fused: bool = True):
        super().__init__()
        self.fused = fused
        if cfg.K != geo.K or cfg.d != geo.d or cfg.rounds != geo.R:
            raise ValueError("configuration and geometry disagree")
        self.cfg, self.gmm = cfg, gmm
        C, K, L = cfg.channels, cfg.K, cfg.layers
        if params is None:
            from .params import init_params
            params = init_params(cfg, seed)
        self.embed = nn.Parameter(torch.as_tensor(np.asarray(params["embed"], np.float32)).clone())
        self.w_c2d = nn.ParameterList([nn.Parameter(torch.as_tensor(params["w_c2d"][l][0]).clone()) for l in range(L)])
        self.w_d2c = nn.ParameterList([nn.Parameter(torch.as_tensor(params["w_d2c"][l][c]).clone())
                                       for l in range(L) for c in range(2)])
        self.head_w = nn.Parameter(torch.as_tensor(params["head_w"]).clone())
        self.head_b = nn.Parameter(torch.as_tensor(params["head_b"]).clone())
        assert self.embed.shape == (N_TOKENS, C) and self.w_c2d[0].shape == (C, K * C)
        buf = {"check_type": geo.check_type.astype(np.int64), "c2d": geo.c2d[0],
               "inv_c2d": geo.inverse(geo.c2d[0], geo.N_c)}
        for c in range(2):
            buf[f"d2c{c}"] = geo.d2c[c]
            buf[f"inv_d2c{c}"] = geo.inverse(geo.d2c[c], geo.N_d)
        for k, v in buf.items():
            self.register_buffer(k, torch.as_tensor(np.asarray(v, np.int64)), persistent=False)
        # int32 gather and target tables of the fused steps (checks are type-major: X checks, then Z checks)
        K = cfg.K
        i32 = {"c2d_i32": geo.c2d[0], "c2d_tgt": target_table(torch.as_tensor(buf["inv_c2d"]), geo.N_d, K)}
        for c in range(2):
            i32[f"d2c{c}_i32"] = geo.d2c[c]
            i32[f"d2c{c}_tgt"] = target_table(torch.as_tensor(buf[f"inv_d2c{c}"]), geo.d2c[c].shape[0], K)
        for k, v in i32.items():
            self.register_buffer(k, torch.as_tensor(np.asarray(v), dtype=torch.int32), persistent=False)
        self.register_buffer("check_type_u8", torch.as_tensor(geo.check_type.astype(np.uint8)), persistent=False)
        self._fused_ok = (geo.d2c[0].shape[0] == geo.d2c[1].shape[0] and
                          np.array_equal(np.concatenate([np.flatnonzero(geo.check_type == 0),
                                                         np.flatnonzero(geo.check_type == 1)]), np.arange(geo.N_c)))
        # the logits read h_d after the last check -> data step: the last data -> check step does not reach the
        # loss, so its weights take no gradient (kept for the inference weight set)
        for c in range(2):
            self.w_d2c[2 * (L - 1) + c].requires_grad_(False)

    def forward(self, det: torch.Tensor, labels: torch.Tensor | None = None) -> torch.Tensor:
        """det (B, N_c) uint8 -> logits (B, N_d, 2) (bf16 under autocast); with labels (B, N_d, 2) 0/1 -> the mean
        BCE-with-logits loss of those logits (the training step's loss, cascade_train.py:292-320)."""
        if (self.fused and self._fused_ok and self.gmm is gather_mm and det.is_cuda and
                torch.is_autocast_enabled("cuda") and torch.get_autocast_dtype("cuda") == torch.bfloat16 and
                self.cfg.channels % 8 == 0):
            return self._forward_fused(det, labels)
        z = self._forward_unfused(det)
        if labels is None:
            return z
        return F.binary_cross_entropy_with_logits(z.float(), labels.float())

    def _forward_unfused(self, det: torch.Tensor) -> torch.Tensor:
        tok = 2 * self.check_type + det.long()
        hc = F.embedding(tok, self.embed)
        hd = None
        for l in range(self.cfg.layers):
            u = F.gelu(self.gmm(hc, self.w_c2d[l], self.c2d, self.inv_c2d), approximate="tanh")
            hd = u if hd is None else hd + u
            if l == self.cfg.layers - 1:
                break
            a = torch.cat([self.gmm(hd, self.w_d2c[2 * l + c], getattr(self, f"d2c{c}"), getattr(self, f"inv_d2c{c}"))
                           for c in range(2)], 1)
            hc = hc + F.gelu(a, approximate="tanh")
        return F.linear(hd, self.head_w, self.head_b)

    def _forward_fused(self, det: torch.Tensor, labels: torch.Tensor | None = None) -> torch.Tensor:
        """The same network under bf16 autocast through ops.bipartite_step: each step is the op's forward kernels
        plus one GELU + residual pass (forward) and one GELU-gradient pass (backward), the check stream fp32 with its
        bf16 copy made in the same pass, the data stream bf16."""
        hc, hc16 = embed_tokens(det.to(torch.uint8), self.check_type_u8, self.embed)
        c2d = ((self.c2d_i32, self.c2d_tgt),)
        d2c = ((self.d2c0_i32, self.d2c0_tgt), (self.d2c1_i32, self.d2c1_tgt))
        hd = None
        carry = {}                              # h_d's two gradients summed in the dgrad epilogue (see bipartite_step)
        for l in range(self.cfg.layers):
            hd = bipartite_step(hc16, hd, c2d, self.w_c2d[l], carry=(carry, l - 1 if l > 0 else None, None))
            if l == self.cfg.layers - 1:
                break
            hc, hc16 = bipartite_step(hd, hc, d2c, self.w_d2c[2 * l], self.w_d2c[2 * l + 1], carry=(carry, None, l))
        if labels is not None and self.cfg.channels <= 128:
            # head and loss in one pass each way, the logits never materialised (ops.HeadBCEB200)
            return head_bce(hd, self.head_w, self.head_b, labels)
        z = F.linear(hd, self.head_w, self.head_b)
        return z if labels is None else F.binary_cross_entropy_with_logits(z.float(), labels.float())


class Trainer:
    """One process per GPU.  model: PreDecoderNet on `device`; with an initialised process group of world > 1 the
    model is wrapped in DDP (NCCL on GPUs, gloo on CPU).  graph=True (one GPU): step_graphed replays the whole step
    from a CUDA graph (the optimiser then keeps its step count on the device)."""

    def __init__(self, model: PreDecoderNet, lr: float = 1e-3, clip: float = 1.0, autocast: bool = True,
                 graph: bool = False):
        import torch.distributed as dist
        self.model = model
        self.device = next(model.parameters()).device
        self.world = dist.get_world_size() if dist.is_available() and dist.is_initialized() else 1
        self.net = model
        if self.world > 1:
            from torch.nn.parallel import DistributedDataParallel as DDP
            ids = [self.device.index] if self.device.type == "cuda" else None
            # ~5 MB of gradients in ~1 MB buckets: the all-reduce of the last layers' buckets runs while the
            # backward of the earlier layers still computes, instead of one bucket after the whole backward
            self.net = DDP(model, device_ids=ids, broadcast_buffers=False, bucket_cap_mb=1,
                           gradient_as_bucket_view=True)
        self.params = [p for p in model.parameters() if p.requires_grad]
        self.graphable = graph and self.world == 1 and self.device.type == "cuda"
        if graph and not self.graphable:
            raise ValueError("graphed training steps run on one GPU (DDP's all-reduce is not captured)")
        self.opt = torch.optim.Adam(self.params, lr=lr, capturable=self.graphable)
        self.clip = clip
        self.autocast = autocast and self.device.type == "cuda"
        self._graph = None

    def step(self, det: torch.Tensor, err: torch.Tensor) -> torch.Tensor:
        """det (B, N_c) uint8, err (B, N_d, 2) 0/1 labels -> the batch loss (a device scalar, not synchronised)."""
        loss = self._forward_backward(det, err)
        self.opt.zero_grad(set_to_none=True)
        return loss

    def _forward_backward(self, det: torch.Tensor, err: torch.Tensor, cache: bool = True) -> torch.Tensor:
        ctx = torch.autocast("cuda", dtype=torch.bfloat16, cache_enabled=cache) if self.autocast else nullcontext()
        with ctx:
            loss = self.net(det, err)            # logits and loss (fused on the GPU path)
        loss.backward()
        torch.nn.utils.clip_grad_norm_(self.params, self.clip)
        self.opt.step()
        return loss.detach()

    def step_graphed(self, det: torch.Tensor, err: torch.Tensor, warmup: int = 2) -> torch.Tensor:
        """The same step replayed from one CUDA graph (forward, backward, clipping, optimiser step), so that the ~230
        launches of a step no longer wait on the host.  The first call runs `warmup` eager steps on det / err on a side
        stream, captures the step over static copies of the inputs and replays it; later calls copy det / err into
        those and replay.  The gradients live in the graph's memory between replays."""
        if not self.graphable:
            raise RuntimeError("graphed steps need Trainer(..., graph=True) on one GPU")
        if self._graph is None:
            self._det, self._err = det.clone(), err.clone()
            side = torch.cuda.Stream(self.device)
            side.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(side):
                for _ in range(warmup):
                    self.step(self._det, self._err)
            torch.cuda.current_stream(self.device).wait_stream(side)
            self.opt.zero_grad(set_to_none=True)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self._loss = self._forward_backward(self._det, self._err, cache=False)
            self._graph = g
        else:
            self._det.copy_(det)
            self._err.copy_(err)
        self._graph.replay()
        return self._loss.clone()

    def agree(self, stop: bool, bad: bool) -> tuple[bool, bool]:
        """Every rank takes the same decision: MAX over ranks of the stop / non-finite flags."""
        if self.world == 1:
            return stop, bad
        import torch.distributed as dist
        fl = torch.tensor([float(stop), float(bad)], device=self.device)
        dist.all_reduce(fl, op=dist.ReduceOp.MAX)
        return bool(fl[0].item()), bool(fl[1].item())


def train_flops_per_shot(geo, cfg) -> float:
    """Algorithmic FLOPs of one training shot: forward + input gradient + weight gradient of every bipartite step
    that reaches the loss (3 x 2 K C^2 per target node and step, all K slots counted; L check -> data steps and
    L - 1 data -> check steps) plus the head."""
    C, K, L = cfg.channels, cfg.K, cfg.layers
    return 3.0 * 2 * K * C * C * (L * geo.N_d + (L - 1) * geo.N_c) + 3.0 * 2 * 2 * C * geo.N_d


def bce_at_init(err_rate: float) -> float:
    """Loss of a predictor that outputs the label frequency (a reference point for the loss curve)."""
    p = min(max(err_rate, 1e-12), 1 - 1e-12)
    return -(p * math.log(p) + (1 - p) * math.log(1 - p))
