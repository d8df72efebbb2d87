"""The allocation-free forward entry point (bpc_predecoder_forward_noalloc), called through the C ABI.

It serves callers that cannot allocate device memory -- a host whose memory pool owns the device heap, a real-time
loop that must not enter the CUDA allocator, a plugin handed only its input and output pointers -- by running the
forward pass on a scratch array built into the library.  Its results must equal those of the workspace entry point
(bpc_predecoder_forward, the same kernels), on two calls in a row (the array keeps the previous call's contents),
and a network too large for the built-in scratch must be refused with a clear error.  This file is collected last.
"""
import ctypes
from dataclasses import replace

import numpy as np
import pytest
import torch

from codecoder_b200 import _lib
from codecoder_b200.geometry import RotatedSurface
from codecoder_b200.modules import PreDecoder
from codecoder_b200.params import CONFIGS, init_params
from codecoder_b200.sampler import sample

pytestmark = pytest.mark.gpu
DEV = "cuda"


def noalloc(pd, det):
    B = det.shape[0]
    logits = torch.empty(B, pd.geo.N_d, 2, dtype=torch.float32, device=pd.device)
    residual = torch.empty(B, pd.geo.N_c, dtype=torch.uint8, device=pd.device)
    rc = _lib.lib().bpc_predecoder_forward_noalloc(pd._h, det.data_ptr(), logits.data_ptr(), residual.data_ptr(), B,
                                                   torch.cuda.current_stream(pd.device).cuda_stream)
    _lib.check(rc, "bpc_predecoder_forward_noalloc")
    return logits, residual


@pytest.mark.parametrize("name,B", [("d9_bf16", 600), ("d5_fp32", 1000)])
def test_noalloc_matches_workspace_entry_point(name, B):
    cfg = CONFIGS[name] if name != "d9_bf16" else replace(CONFIGS[name], layers=3)
    g = RotatedSurface(cfg.d, cfg.rounds)
    params = init_params(cfg, 808)
    pd = PreDecoder(g, cfg, params, device=DEV)
    assert pd.workspace_bytes(256) <= _lib.lib().bpc_noalloc_scratch_bytes()
    for call in range(2):                                   # two calls in a row share the scratch array
        det, _ = sample(g, 0.02, B, 809 + call)
        d = torch.as_tensor(det).to(DEV)
        ref_lg, ref_rs = pd(d)
        lg, rs = noalloc(pd, d)
        torch.cuda.synchronize()
        assert pd.status() == 0
        tol = 1e-4 if cfg.dtype == "f32" else 2e-2
        scale = max(float(ref_lg.abs().max()), 1e-30)
        assert float((lg - ref_lg).abs().max()) <= tol * scale
        assert torch.equal(rs, ref_rs)


def test_noalloc_refuses_networks_larger_than_its_scratch():
    cfg = CONFIGS["d13_bf16"]
    g = RotatedSurface(cfg.d, cfg.rounds)
    pd = PreDecoder(g, replace(cfg, layers=1), init_params(replace(cfg, layers=1), 1), device=DEV)
    assert pd.workspace_bytes(256) > _lib.lib().bpc_noalloc_scratch_bytes()
    det = torch.zeros(256, g.N_c, dtype=torch.uint8, device=DEV)
    lg = torch.empty(256, g.N_d, 2, dtype=torch.float32, device=DEV)
    rs = torch.empty(256, g.N_c, dtype=torch.uint8, device=DEV)
    rc = _lib.lib().bpc_predecoder_forward_noalloc(pd._h, det.data_ptr(), lg.data_ptr(), rs.data_ptr(), 256, None)
    assert rc == 6 and "built-in scratch" in _lib.last_error()
