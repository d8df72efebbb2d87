"""The C-ABI library loads here (no GPU) and exports exactly what include/bpc.h declares; argument errors come back
as error codes with a message, before any device work."""
import ctypes
import os
import re
import subprocess

import pytest

from codecoder_b200 import _lib

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared():
    src = open(os.path.join(REPO, "include", "bpc.h")).read()
    return sorted(set(re.findall(r"BPC_API\s+[\w\s\*]+?\b(bpc_\w+)\s*\(", src)))


@pytest.fixture(scope="module")
def lib():
    from codecoder_b200.build import build
    build()
    return _lib.lib()


def test_header_and_binding_agree():
    assert declared() == sorted(_lib.SIGNATURES)


def test_library_exports_every_declared_symbol(lib):
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True).stdout
    exported = set(re.findall(r" T (bpc_\w+)", out))
    assert set(declared()) <= exported
    for name in declared():
        assert getattr(lib, name) is not None


def test_version_and_errors(lib):
    assert lib.bpc_version() >= 1
    rc = lib.bpc_gather_mm_fwd(None, None, None, None, 4, 0, 4, 8, 64, 64, 1, None)
    assert rc == 2
    assert "shape" in _lib.last_error()
    rc = lib.bpc_gather_mm_fwd(None, None, None, None, 4, 10, 4, 8, 64, 64, 7, None)
    assert rc == 2 and "dtype" in _lib.last_error()
    rc = lib.bpc_gather_mm_fwd(None, None, None, None, 4, 10, 4, 8, 64, 64, 1, None)
    assert rc == 2 and "null" in _lib.last_error()
    # an empty batch is a no-op
    assert lib.bpc_gather_mm_fwd(None, None, None, None, 0, 10, 4, 8, 64, 64, 1, None) == 0


def test_predecoder_argument_checks(lib):
    cfg = _lib.PredecoderConfig(0, 64, 8, 1, 10, 10, 5)
    h = ctypes.c_void_p()
    z = (ctypes.c_int32 * 100)()
    rc = lib.bpc_predecoder_create(ctypes.byref(cfg), z, z, z, z, None, ctypes.byref(h))
    assert rc == 2 and "configuration" in _lib.last_error()
    assert lib.bpc_predecoder_forward(None, None, None, None, 1, None, 0, None) == 2
    assert lib.bpc_predecoder_workspace_size(None, 128) == 0


def test_ops_refuse_cpu_tensors():
    import torch
    from codecoder_b200.ops import gmm
    with pytest.raises(RuntimeError, match="CUDA"):
        gmm(torch.zeros(1, 4, 64, dtype=torch.bfloat16), torch.zeros(2, 8, dtype=torch.int32),
            torch.zeros(64, 512, dtype=torch.bfloat16))


def test_training_entry_points_check_arguments_first(lib):
    """The training network's passes reject bad shapes and null buffers with BPC_ERR_ARG before any device work, and
    an empty batch is a no-op."""
    bf16, f32 = _lib.BPC_DTYPE_BF16, _lib.BPC_DTYPE_F32
    # NT not a multiple of the type count, C not a multiple of 8
    assert lib.bpc_gelu_residual_fwd(None, None, None, None, 4, 7, 64, 2, bf16, None) == 2
    assert "multiple" in _lib.last_error()
    assert lib.bpc_gelu_residual_fwd(None, None, None, None, 4, 8, 60, 2, bf16, None) == 2
    # null buffers
    assert lib.bpc_gelu_residual_fwd(None, None, None, None, 4, 8, 64, 2, bf16, None) == 2
    assert "null" in _lib.last_error()
    # the bf16 stream takes neither a second gradient nor gh
    assert lib.bpc_gelu_residual_bwd(16, 16, 16, 16, 16, 4, 8, 64, 2, bf16, None) == 2
    assert lib.bpc_gelu_residual_bwd(None, None, None, None, None, 4, 8, 64, 2, f32, None) == 2
    # empty batches
    assert lib.bpc_gelu_residual_fwd(None, None, None, None, 0, 8, 64, 2, bf16, None) == 0
    assert lib.bpc_gelu_residual_bwd(None, None, None, None, None, 0, 8, 64, 2, f32, None) == 0
    # embedding: C limits, null buffers, workspace size
    assert lib.bpc_embed_tokens_fwd(None, None, None, None, None, 4, 10, 60, None) == 2
    assert lib.bpc_embed_tokens_fwd(None, None, None, None, None, 4, 10, 64, None) == 2
    assert lib.bpc_embed_tokens_fwd(None, None, None, None, None, 0, 10, 64, None) == 0
    assert lib.bpc_embed_tokens_bwd_workspace_size(96) >= 4 * 96 * 4
    assert lib.bpc_embed_tokens_bwd(None, None, None, None, 16, None, 0, 4, 10, 300, None) == 2
    assert lib.bpc_embed_tokens_bwd(None, None, None, None, 16, None, 0, 4, 10, 96, None) == 2
    # accumulating input gradient: shape and dtype checks
    assert lib.bpc_gather_mm_dgrad_ex(None, None, None, None, None, 4, 0, 10, 8, 64, 64, 1, bf16, None) == 2
    assert lib.bpc_gather_mm_dgrad_ex(None, None, None, None, None, 4, 10, 10, 8, 64, 64, 1, 9, None) == 2
    assert lib.bpc_gather_mm_dgrad_ex(None, None, None, None, None, 4, 10, 10, 8, 64, 64, 1, bf16, None) == 2
    assert "null" in _lib.last_error()
    # the one-launch residual step: shape, stream dtype, stream rows that overlap, null buffers
    gelu = lib.bpc_gather_mm_fwd_gelu
    assert gelu(None, None, None, None, 4, 0, 10, 8, 96, 96, None, bf16, None, None, 960, None) == 2
    assert gelu(None, None, None, None, 4, 20, 10, 8, 96, 96, 16, 9, None, None, 960, None) == 2
    assert gelu(None, None, None, None, 4, 20, 10, 8, 96, 96, None, bf16, None, None, 959, None) == 2
    assert "overlap" in _lib.last_error()
    assert gelu(None, None, None, None, 4, 20, 10, 8, 96, 96, None, bf16, None, None, 960, None) == 2
    assert "null" in _lib.last_error()
