"""The allocation-free forward entry point (bpc_predecoder_forward_noalloc), called through the C ABI.

It serves callers that cannot allocate device memory -- a host whose memory pool owns the device heap, a real-time
loop that must not enter the CUDA allocator, a plugin handed only its input and output pointers -- by running the
forward pass on a scratch array built into the library.  Its results must equal those of the workspace entry point
(bpc_predecoder_forward, the same kernels) bit for bit, on two calls in a row (the array keeps the previous call's
contents); after the first call's set-up a call must leave the device's free memory unchanged; a network too large
for the built-in scratch, and a handle of another device, must be refused with a clear error.  This file is
collected last.
"""
import ctypes
from dataclasses import replace

import pytest
import torch

from codecoder_b200 import _lib
from codecoder_b200.geometry import RotatedSurface
from codecoder_b200.modules import PreDecoder
from codecoder_b200.params import CONFIGS, init_params
from codecoder_b200.sampler import sample

pytestmark = pytest.mark.gpu
DEV = "cuda"


def noalloc_into(pd, det, logits, residual):
    rc = _lib.lib().bpc_predecoder_forward_noalloc(pd._h, det.data_ptr(), logits.data_ptr(), residual.data_ptr(),
                                                   det.shape[0], torch.cuda.current_stream(pd.device).cuda_stream)
    _lib.check(rc, "bpc_predecoder_forward_noalloc")


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
        lg = torch.empty(B, g.N_d, 2, dtype=torch.float32, device=DEV)
        rs = torch.empty(B, g.N_c, dtype=torch.uint8, device=DEV)
        torch.cuda.synchronize()
        before = (torch.cuda.memory_allocated(), torch.cuda.mem_get_info()[0])
        noalloc_into(pd, d, lg, rs)
        torch.cuda.synchronize()
        after = (torch.cuda.memory_allocated(), torch.cuda.mem_get_info()[0])
        assert pd.status() == 0
        # the same kernels on a different pass size: chunking does not change a bit
        assert torch.equal(lg, ref_lg) and torch.equal(rs, ref_rs)
        if call == 1:                                       # after the first call's set-up: nothing is allocated
            assert after == before, f"device memory changed across a call: {before} -> {after}"


def test_noalloc_refuses_a_handle_of_another_device():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    cfg = replace(CONFIGS["d9_bf16"], layers=1)
    g = RotatedSurface(cfg.d, cfg.rounds)
    pd = PreDecoder(g, cfg, init_params(cfg, 3), device="cuda:0")
    with torch.cuda.device(1):
        det = torch.zeros(8, g.N_c, dtype=torch.uint8, device="cuda:1")
        lg = torch.empty(8, g.N_d, 2, dtype=torch.float32, device="cuda:1")
        rs = torch.empty(8, g.N_c, dtype=torch.uint8, device="cuda:1")
        rc = _lib.lib().bpc_predecoder_forward_noalloc(pd._h, det.data_ptr(), lg.data_ptr(), rs.data_ptr(), 8, None)
    assert rc == 2 and "created on device 0" in _lib.last_error()


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
