"""Routing pre-decoded shots to a fallback decoder (C ABI bpc_route), the hand-off of the reference's decoder.

The reference trusts its network where the network is confident and sends the other shots to PyMatching:
`route(c, tau)` marks shots whose logit is within tau of zero and `decode(model, cfg, det, matcher=...)` decides the
marked shots with the matcher, the rest by the network's sign (evaluation/convlines/decoder.py:116-142; the
deployed router hands the fired detectors to the matcher, evaluation/timing/d7/router.cc:142-168).  For the
pre-decoder the shot's confidence is its least confident data-qubit logit, and a shot whose residual syndrome is not
empty is also routed (the pre-decoder left detectors for the global decoder to explain):

    route(logits, residual, tau)      -> Routing(routed, index, handoff, conf, weight) on the device
    decode(pd, det, tau, matcher)     -> (logits, residual, routed, correction)

`matcher` is any callable taking the hand-off (R, N_c) uint8 residual rows (numpy) and returning the data-qubit flips
(R, N_d, 2) uint8 that explain them (e.g. a PyMatching wrapper where PyMatching is installed; it is not a dependency
here).  The correction of a routed shot is the network's thresholded flips XOR the matcher's; without a matcher the
routed shots keep the network's flips and the hand-off is returned for the caller's decoder.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from . import _lib


@dataclass
class Routing:
    routed: torch.Tensor        # (B,) bool: the shot goes to the fallback decoder
    index: torch.Tensor         # (R,) int64: routed shots in ascending order
    handoff: torch.Tensor       # (R, N_c) uint8: their residual syndromes, the fallback decoder's input
    conf: torch.Tensor          # (B,) fp32: least |logit| of the shot
    weight: torch.Tensor        # (B,) int32: set bits of the shot's residual


def route(logits: torch.Tensor, residual: torch.Tensor, tau: float, route_residual: bool = True) -> Routing:
    """logits (B, N_d, 2) fp32 and residual (B, N_c) uint8 on a CUDA device -> Routing (device tensors)."""
    if not (logits.is_cuda and residual.is_cuda) or logits.device != residual.device:
        raise RuntimeError("route runs on CUDA tensors of one device (no CPU path)")
    if logits.dtype != torch.float32 or residual.dtype != torch.uint8 or logits.dim() != 3 or logits.shape[2] != 2:
        raise TypeError("route: logits (B, N_d, 2) fp32 and residual (B, N_c) uint8")
    B, N_d, _ = logits.shape
    if residual.dim() != 2 or residual.shape[0] != B:
        raise ValueError("route: logits and residual disagree on the batch")
    N_c = residual.shape[1]
    dev = logits.device
    logits, residual = logits.contiguous(), residual.contiguous()
    routed = torch.empty(B, dtype=torch.uint8, device=dev)
    index = torch.empty(max(B, 1), dtype=torch.int64, device=dev)
    handoff = torch.empty(max(B, 1), N_c, dtype=torch.uint8, device=dev)
    n = torch.zeros(1, dtype=torch.int64, device=dev)
    conf = torch.empty(B, dtype=torch.float32, device=dev)
    weight = torch.empty(B, dtype=torch.int32, device=dev)
    L = _lib.lib()
    ws = torch.empty(max(int(L.bpc_route_workspace_size(B)), 8), dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        rc = L.bpc_route(logits.data_ptr(), residual.data_ptr(), B, N_d, N_c, float(tau), int(bool(route_residual)),
                         routed.data_ptr(), index.data_ptr(), handoff.data_ptr(), n.data_ptr(), conf.data_ptr(),
                         weight.data_ptr(), ws.data_ptr(), ws.numel(), torch.cuda.current_stream(dev).cuda_stream)
    _lib.check(rc, "bpc_route")
    R = int(n.item())
    return Routing(routed.bool(), index[:R], handoff[:R], conf, weight)


def decode(pd, det: torch.Tensor, tau: float, matcher=None, route_residual: bool = True):
    """The pre-decoder `pd` (modules.PreDecoder) on det (B, N_c) uint8, then the routing and, where a matcher is
    given, the fallback decoding of the routed shots' residuals -> (logits, residual, routing, correction (B, N_d, 2)
    uint8 on the device)."""
    logits, residual = pd(det)
    r = route(logits, residual, tau, route_residual)
    corr = (logits > 0).to(torch.uint8)
    if matcher is not None and r.index.numel() > 0:
        fix = np.asarray(matcher(r.handoff.cpu().numpy()), np.uint8)
        if fix.shape != (r.index.numel(), logits.shape[1], 2):
            raise ValueError("matcher must return (R, N_d, 2) data-qubit flips for the R routed residuals")
        corr[r.index] ^= torch.as_tensor(fix, device=corr.device)
    return logits, residual, r, corr
