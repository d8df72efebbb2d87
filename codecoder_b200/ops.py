"""The bipartite-convolution op with the reference's signatures, on libbpc.so's kernels.

Drop-ins (training/bb/ising_compare/bb/cascade_net.py and cascade_triton.py):
  gather_mm(x, w, idx, inv)                  cascade_net.py:174-175
  GatherMMB200.apply(x, w, idx, inv)         the autograd Function, as GatherMMTriton (cascade_triton.py:161-171)
  torch.ops.cascade.gmm(a, idx, w, transposed)   cascade_triton.py:139-148 (transposed=False)
Everything runs on the GPU: a CPU tensor raises, there is no CPU path.  bf16 inputs run on the tcgen05 tensor
cores (C_in >= 64, C_out % 32 == 0, C_out <= 256) or the CUDA-core kernel; fp32 inputs on the CUDA-core kernel.
"""
from __future__ import annotations

import torch

from . import _lib

_DTYPES = {torch.bfloat16: _lib.BPC_DTYPE_BF16, torch.float32: _lib.BPC_DTYPE_F32}


def _stream_ptr(device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def gmm(a: torch.Tensor, idx: torch.Tensor, w: torch.Tensor, transposed: bool = False) -> torch.Tensor:
    """a (B, NS, C_in), idx (NT, K) int32, w (C_out, K C_in) -> y (B, NT, C_out), y[b, n] = sum_r a[b, idx[n, r]] W_r^T
    (idx outside [0, NS) reads zeros).  Same contract as cascade_triton.gmm with transposed=False."""
    if transposed:
        raise NotImplementedError("the input-gradient form (transposed=True) of cascade::gmm is not built yet")
    if not (a.is_cuda and idx.is_cuda and w.is_cuda):
        raise RuntimeError("codecoder_b200.gmm runs on CUDA tensors only (no CPU path)")
    if a.dtype not in _DTYPES or w.dtype != a.dtype:
        raise TypeError(f"gmm needs bf16 or fp32 a and w of the same dtype, got {a.dtype} / {w.dtype}")
    if a.dim() != 3 or idx.dim() != 2 or w.dim() != 2:
        raise ValueError("gmm expects a (B, NS, C), idx (NT, K), w (C_out, K C_in)")
    B, NS, Ci = a.shape
    NT, K = idx.shape
    Co, KC = w.shape
    if KC != K * Ci:
        raise ValueError(f"w has {KC} columns, expected K * C_in = {K * Ci}")
    a = a.contiguous()
    w = w.contiguous()
    idx = idx.to(torch.int32).contiguous()
    y = torch.empty(B, NT, Co, device=a.device, dtype=a.dtype)
    if B == 0 or NT == 0:
        return y
    rc = _lib.lib().bpc_gather_mm_fwd(a.data_ptr(), w.data_ptr(), idx.data_ptr(), y.data_ptr(), B, NS, NT, K, Ci,
                                      Co, _DTYPES[a.dtype], _stream_ptr(a.device))
    _lib.check(rc, "bpc_gather_mm_fwd")
    return y


@torch.library.custom_op("cascade::gmm", mutates_args=())
def gmm_op(a: torch.Tensor, idx: torch.Tensor, w: torch.Tensor, transposed: bool) -> torch.Tensor:
    """gmm as an opaque operator (the reference registers the same name, cascade_triton.py:139-142)."""
    return gmm(a, idx, w, transposed)


@gmm_op.register_fake
def _(a, idx, w, transposed):
    K = idx.shape[1]
    return a.new_empty(a.shape[0], idx.shape[0], w.shape[1] // K if transposed else w.shape[0])


class GatherMMB200(torch.autograd.Function):
    """Drop-in for cascade_net._GatherMM / cascade_triton.GatherMMTriton (same signature; idx and the inverse table
    as int64 on the device).  Forward only: the backward kernels are not built yet and raise."""

    @staticmethod
    @torch.amp.custom_fwd(device_type="cuda", cast_inputs=torch.bfloat16)
    def forward(ctx, x, w, idx, inv):
        return gmm_op(x.contiguous(), idx.to(torch.int32), w.contiguous(), False)

    @staticmethod
    @torch.amp.custom_bwd(device_type="cuda")
    def backward(ctx, gy):
        raise NotImplementedError("backward of the B200 gather_mm (dgrad / wgrad kernels) is not built yet")


def gather_mm(x, w, idx, inv):
    """y[b, n] = W cat_r x[b, idx[n, r]] (cascade_net.py:174-175), on the B200 kernels."""
    return GatherMMB200.apply(x, w, idx, inv)
