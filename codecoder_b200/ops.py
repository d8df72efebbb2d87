"""The bipartite-convolution op with the reference's signatures, on libbpc.so's kernels.

Drop-ins (training/bb/ising_compare/bb/cascade_net.py and cascade_triton.py):
  gather_mm(x, w, idx, inv)                  cascade_net.py:174-175
  GatherMMB200.apply(x, w, idx, inv)         the autograd Function, as GatherMMTriton (cascade_triton.py:161-186)
  torch.ops.cascade.gmm(a, idx, w, transposed)   cascade_triton.py:100-117,139-148
  torch.ops.cascade.gmm_wgrad(x, gy, idx)        cascade_triton.py:120-136,151-158 (fp32 result)
Everything runs on the GPU: a CPU tensor raises, there is no CPU path.  bf16 inputs run on the tcgen05 tensor
cores (forward: C_in >= 64, C_out % 32 == 0, C_out <= 256; weight gradient: C_in % 16 == 0, C_out % 8 == 0) or
the CUDA-core kernels; fp32 inputs on the CUDA-core kernels.  The weight gradient is deterministic (fixed split of
the rows, partial sums added in a fixed order), as the reference's is.
"""
from __future__ import annotations

import torch

from . import _lib

_DTYPES = {torch.bfloat16: _lib.BPC_DTYPE_BF16, torch.float32: _lib.BPC_DTYPE_F32}


# True: the fused steps' forward runs the op and its GELU / residual pass in one launch where the wide-tile kernel
# takes the shape (bpc_gather_mm_fwd_gelu); False (default): the op, then the pass.  Both give the same bits; on a
# B200 the one-launch form measured slower (d = 11 training step 146 against 139 ms on the same box: the stream's
# loads and stores in the epilogue slow the L2-bound op by more than the separate pass costs).
_FUSED_GELU = False


def _stream_ptr(device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _check_cuda(*ts):
    if not all(t.is_cuda for t in ts):
        raise RuntimeError("codecoder_b200 ops run on CUDA tensors only (no CPU path)")


def gmm(a: torch.Tensor, idx: torch.Tensor, w: torch.Tensor, transposed: bool = False) -> torch.Tensor:
    """Same contract as cascade_triton.gmm (cascade_triton.py:100-117).
    transposed=False: a (B, NS, C_in), idx (NT, K), w (C_out, K C_in) -> (B, NT, C_out),
                      y[b, n] = sum_r a[b, idx[n, r]] W_r^T (idx outside [0, NS) reads zeros).
    transposed=True:  a = gy (B, NT, C_out), idx = the target table tgt (NS, K) -> gx (B, NS, C_in),
                      gx[b, s] = sum_r gy[b, tgt[s, r]] W_r (tgt outside [0, NT) = none)."""
    _check_cuda(a, idx, w)
    if a.dtype not in _DTYPES or w.dtype != a.dtype:
        raise TypeError(f"gmm needs bf16 or fp32 a and w of the same dtype, got {a.dtype} / {w.dtype}")
    if a.dim() != 3 or idx.dim() != 2 or w.dim() != 2:
        raise ValueError("gmm expects a (B, N, C), idx (N_out, K), w (C_out, K C_in)")
    B, NA, CA = a.shape
    NY, K = idx.shape
    Co, KC = w.shape
    if KC % K:
        raise ValueError(f"w has {KC} columns, not a multiple of K = {K}")
    Ci = KC // K
    if CA != (Co if transposed else Ci):
        raise ValueError(f"a has {CA} channels, expected {Co if transposed else Ci}")
    a = a.contiguous()
    w = w.contiguous()
    idx = idx.to(torch.int32).contiguous()
    CY = Ci if transposed else Co
    y = torch.empty(B, NY, CY, device=a.device, dtype=a.dtype)
    if B == 0 or NY == 0:
        return y
    L = _lib.lib()
    if transposed:
        w_t = torch.empty_like(w)
        rc = L.bpc_gather_mm_dgrad(a.data_ptr(), w.data_ptr(), idx.data_ptr(), y.data_ptr(), w_t.data_ptr(), B, NA,
                                   NY, K, Ci, Co, _DTYPES[a.dtype], _stream_ptr(a.device))
        _lib.check(rc, "bpc_gather_mm_dgrad")
    else:
        rc = L.bpc_gather_mm_fwd(a.data_ptr(), w.data_ptr(), idx.data_ptr(), y.data_ptr(), B, NA, NY, K, Ci, Co,
                                 _DTYPES[a.dtype], _stream_ptr(a.device))
        _lib.check(rc, "bpc_gather_mm_fwd")
    return y


def gmm_ex(a: torch.Tensor, idx: torch.Tensor, w: torch.Tensor, type_split: int | None = None,
           scale: torch.Tensor | None = None, shift: torch.Tensor | None = None) -> torch.Tensor:
    """Forward with one or two weight sets and an optional affine + SiLU epilogue (C ABI bpc_gather_mm_fwd_ex).
    a (B, NS, C_in); idx (NT, K); w (C_out, K C_in) or (2, C_out, K C_in) with targets >= type_split using w[1];
    scale / shift fp32 (C_out,): y = SiLU(scale * acc + shift) per output channel (an inference BatchNorm + SiLU)."""
    _check_cuda(a, idx, w)
    if a.dtype not in _DTYPES or w.dtype != a.dtype:
        raise TypeError(f"gmm_ex needs bf16 or fp32 a and w of the same dtype, got {a.dtype} / {w.dtype}")
    B, NS, Ci = a.shape
    NT, K = idx.shape
    n_w = 1 if w.dim() == 2 else w.shape[0]
    Co, KC = w.shape[-2:]
    if KC != K * Ci or n_w not in (1, 2):
        raise ValueError("gmm_ex: w must be (C_out, K C_in) or (2, C_out, K C_in)")
    split = NT if type_split is None else int(type_split)
    if (scale is None) != (shift is None):
        raise ValueError("gmm_ex: give both scale and shift, or neither")
    a = a.contiguous()
    w = w.contiguous()
    idx = idx.to(torch.int32).contiguous()
    y = torch.empty(B, NT, Co, device=a.device, dtype=a.dtype)
    if B == 0 or NT == 0:
        return y
    epi = _lib.BPC_EPILOGUE_STORE
    sp = hp = None
    if scale is not None:
        epi = _lib.BPC_EPILOGUE_AFFINE_SILU
        scale = scale.to(a.device, torch.float32).contiguous()
        shift = shift.to(a.device, torch.float32).contiguous()
        sp, hp = scale.data_ptr(), shift.data_ptr()
    rc = _lib.lib().bpc_gather_mm_fwd_ex(a.data_ptr(), w.data_ptr(), idx.data_ptr(), y.data_ptr(), B, NS, NT, K, Ci,
                                         Co, n_w, split, epi, sp, hp, _DTYPES[a.dtype], _stream_ptr(a.device))
    _lib.check(rc, "bpc_gather_mm_fwd_ex")
    return y


def cascade_boundary(x3: torch.Tensor, w_up: torch.Tensor, h: torch.Tensor, scale_h: float, scale_u: float,
                     a1: torch.Tensor | None = None, b1: torch.Tensor | None = None, w_down: torch.Tensor | None = None,
                     a2: torch.Tensor | None = None, b2: torch.Tensor | None = None, h_out="new", want_y: bool = True):
    """The boundary between two Cascade bottleneck blocks in one launch (C ABI bpc_cascade_boundary; H = 512, a
    128-channel bottleneck): x3 (..., 128) bf16, w_up (512, 128) bf16, h (..., 512) fp32 ->
    (h' = scale_h h + scale_u bf16(x3 w_up^T) fp32 or None,
     y = bf16(SiLU(a2 (x1 w_down^T) + b2)) (..., 128) with w_down, else x1 = bf16(SiLU(a1 h' + b1)) (..., 512), or None).
    h_out: "new" (allocate), a tensor to write (h itself updates in place), or None (h' not written)."""
    _check_cuda(x3, w_up, h)
    if x3.dtype != torch.bfloat16 or w_up.dtype != torch.bfloat16 or h.dtype != torch.float32:
        raise TypeError("cascade_boundary: bf16 x3 and w_up, fp32 h")
    H, Hb = w_up.shape
    if x3.shape[-1] != Hb or h.shape[-1] != H or x3.shape[:-1] != h.shape[:-1]:
        raise ValueError("cascade_boundary: x3 (..., Hb), w_up (H, Hb), h (..., H) with the same rows")
    x3, w_up, h = x3.contiguous(), w_up.contiguous(), h.contiguous()
    rows = h.numel() // H
    out = torch.empty_like(h) if isinstance(h_out, str) else h_out
    if out is not None and (out.shape != h.shape or out.dtype != torch.float32 or not out.is_contiguous()):
        raise ValueError("cascade_boundary: h_out must be a contiguous fp32 tensor of h's shape")
    vec = lambda t: None if t is None else t.to(h.device, torch.float32).contiguous()
    a1, b1, a2, b2 = vec(a1), vec(b1), vec(a2), vec(b2)
    y = None
    if w_down is not None:
        w_down = w_down.to(torch.bfloat16).contiguous()
        y = torch.empty(*h.shape[:-1], w_down.shape[0], device=h.device, dtype=torch.bfloat16)
    elif want_y and a1 is not None:
        y = torch.empty(h.shape, device=h.device, dtype=torch.bfloat16)
    ptr = lambda t: None if t is None else t.data_ptr()
    rc = _lib.lib().bpc_cascade_boundary(x3.data_ptr(), w_up.data_ptr(), h.data_ptr(), ptr(out), float(scale_h),
                                         float(scale_u), ptr(a1), ptr(b1), ptr(w_down), ptr(a2), ptr(b2), ptr(y),
                                         rows, H, Hb, _stream_ptr(h.device))
    _lib.check(rc, "bpc_cascade_boundary")
    return out, y


def cascade_boundary_tokens(x3: torch.Tensor, w_up: torch.Tensor, det: torch.Tensor, gidx: torch.Tensor,
                            tbase: torch.Tensor, E: torch.Tensor, scale_h: float, scale_u: float,
                            a1: torch.Tensor | None = None, b1: torch.Tensor | None = None,
                            w_down: torch.Tensor | None = None, a2: torch.Tensor | None = None,
                            b2: torch.Tensor | None = None, want_h: bool = True, want_y: bool = True):
    """cascade_boundary for the first block of a network (C ABI bpc_cascade_boundary_tokens): the stream h is the
    embedding E (5, 512) of the detector tokens (det (B, D) uint8, gidx / tbase (N) int32), never materialised.
    x3 (B, N, 128) -> (h' (B, N, 512) fp32 or None, y or None) as cascade_boundary."""
    _check_cuda(x3, w_up, det, gidx, tbase, E)
    B, D = det.shape
    N = gidx.shape[0]
    H, Hb = w_up.shape
    if x3.shape != (B, N, Hb) or E.shape != (5, H):
        raise ValueError("cascade_boundary_tokens: x3 (B, N, Hb), E (5, H)")
    dev = x3.device
    x3, w_up = x3.contiguous(), w_up.contiguous()
    det = det.to(torch.uint8).contiguous()
    gidx, tbase = gidx.to(torch.int32).contiguous(), tbase.to(torch.int32).contiguous()
    E = E.to(torch.float32).contiguous()
    vec = lambda t: None if t is None else t.to(dev, torch.float32).contiguous()
    a1, b1, a2, b2 = vec(a1), vec(b1), vec(a2), vec(b2)
    out = torch.empty(B, N, H, device=dev, dtype=torch.float32) if want_h else None
    y = None
    if w_down is not None:
        w_down = w_down.to(torch.bfloat16).contiguous()
        y = torch.empty(B, N, w_down.shape[0], device=dev, dtype=torch.bfloat16)
    elif want_y and a1 is not None:
        y = torch.empty(B, N, H, device=dev, dtype=torch.bfloat16)
    ptr = lambda t: None if t is None else t.data_ptr()
    rc = _lib.lib().bpc_cascade_boundary_tokens(x3.data_ptr(), w_up.data_ptr(), det.data_ptr(), gidx.data_ptr(),
                                                tbase.data_ptr(), E.data_ptr(), D, N, ptr(out), float(scale_h),
                                                float(scale_u), ptr(a1), ptr(b1), ptr(w_down), ptr(a2), ptr(b2),
                                                ptr(y), B, H, Hb, _stream_ptr(dev))
    _lib.check(rc, "bpc_cascade_boundary_tokens")
    return out, y


def cascade_stem(det: torch.Tensor, gidx: torch.Tensor, tbase: torch.Tensor, E: torch.Tensor, a1: torch.Tensor,
                 b1: torch.Tensor) -> torch.Tensor:
    """The Cascade network's stem and first BN1 + SiLU (C ABI bpc_cascade_stem): det (B, D) uint8 ->
    x1 = bf16(SiLU(a1 E[token] + b1)) (B, N, H), the embedded stream itself not written."""
    _check_cuda(det, gidx, tbase, E)
    B, D = det.shape
    N = gidx.shape[0]
    H = E.shape[1]
    dev = E.device
    det = det.to(torch.uint8).contiguous()
    gidx, tbase = gidx.to(torch.int32).contiguous(), tbase.to(torch.int32).contiguous()
    E = E.to(torch.float32).contiguous()
    a1, b1 = a1.to(dev, torch.float32).contiguous(), b1.to(dev, torch.float32).contiguous()
    x1 = torch.empty(B, N, H, device=dev, dtype=torch.bfloat16)
    rc = _lib.lib().bpc_cascade_stem(det.data_ptr(), gidx.data_ptr(), tbase.data_ptr(), E.data_ptr(), D, N,
                                     a1.data_ptr(), b1.data_ptr(), x1.data_ptr(), B, H, _stream_ptr(dev))
    _lib.check(rc, "bpc_cascade_stem")
    return x1


def residual_affine_silu(h: torch.Tensor, u: torch.Tensor | None, scale_h: float, scale_u: float,
                         a: torch.Tensor | None = None, b: torch.Tensor | None = None, want_out: bool = True):
    """One pass over an fp32 (..., H) stream (C ABI bpc_residual_affine_silu): v = scale_h h + scale_u u (u bf16 or
    None) -> (v fp32 or None, SiLU(a v + b) bf16 or None)."""
    _check_cuda(h)
    if h.dtype != torch.float32 or (u is not None and (u.dtype != torch.bfloat16 or u.shape != h.shape)):
        raise TypeError("residual_affine_silu: h fp32, u bf16 of h's shape")
    h = h.contiguous()
    H = h.shape[-1]
    rows = h.numel() // H
    out = torch.empty_like(h) if want_out else None
    x = torch.empty(h.shape, dtype=torch.bfloat16, device=h.device) if a is not None else None
    u = u.contiguous() if u is not None else None
    rc = _lib.lib().bpc_residual_affine_silu(
        h.data_ptr(), u.data_ptr() if u is not None else None, out.data_ptr() if out is not None else None,
        x.data_ptr() if x is not None else None, rows, H, float(scale_h), float(scale_u),
        a.data_ptr() if a is not None else None, b.data_ptr() if b is not None else None, _stream_ptr(h.device))
    _lib.check(rc, "bpc_residual_affine_silu")
    return out, x


def gmm_wgrad(x: torch.Tensor, gy: torch.Tensor, idx: torch.Tensor) -> torch.Tensor:
    """x (B, NS, C_in), gy (B, NT, C_out), idx (NT, K) -> dW (C_out, K C_in) fp32,
    dW[o, r C_in + i] = sum_{b, n} gy[b, n, o] x[b, idx[n, r], i] (cascade_triton.py:120-136)."""
    _check_cuda(x, gy, idx)
    if x.dtype not in _DTYPES or gy.dtype != x.dtype:
        raise TypeError(f"gmm_wgrad needs bf16 or fp32 x and gy of the same dtype, got {x.dtype} / {gy.dtype}")
    B, NS, Ci = x.shape
    B2, NT, Co = gy.shape
    NT2, K = idx.shape
    if B2 != B or NT2 != NT:
        raise ValueError("gmm_wgrad: x, gy and idx disagree on B or NT")
    x = x.contiguous()
    gy = gy.contiguous()
    idx = idx.to(torch.int32).contiguous()
    dw = torch.empty(Co, K * Ci, device=x.device, dtype=torch.float32)
    L = _lib.lib()
    dt = _DTYPES[x.dtype]
    nbytes = int(L.bpc_gather_mm_wgrad_workspace_size(B, NS, NT, K, Ci, Co, dt))
    ws = torch.empty(max(nbytes, 16), device=x.device, dtype=torch.uint8)
    rc = L.bpc_gather_mm_wgrad(x.data_ptr(), gy.data_ptr(), idx.data_ptr(), dw.data_ptr(), ws.data_ptr(), ws.numel(),
                               B, NS, NT, K, Ci, Co, dt, _stream_ptr(x.device))
    _lib.check(rc, "bpc_gather_mm_wgrad")
    return dw


def op_status(device=None) -> int:
    """Synchronise the current stream and read (and clear) the gather_mm kernels' watchdog word; raises if set."""
    import ctypes
    s = ctypes.c_int(0)
    with torch.cuda.device(device if device is not None else torch.cuda.current_device()):
        rc = _lib.lib().bpc_gather_mm_status(_stream_ptr(torch.cuda.current_device()), ctypes.byref(s))
    _lib.check(rc, "bpc_gather_mm_status")
    return s.value


@torch.library.custom_op("cascade::gmm", mutates_args=())
def gmm_op(a: torch.Tensor, idx: torch.Tensor, w: torch.Tensor, transposed: bool) -> torch.Tensor:
    """gmm as an opaque operator (the reference registers the same name, cascade_triton.py:139-142)."""
    return gmm(a, idx, w, transposed)


@gmm_op.register_fake
def _(a, idx, w, transposed):
    K = idx.shape[1]
    return a.new_empty(a.shape[0], idx.shape[0], w.shape[1] // K if transposed else w.shape[0])


@torch.library.custom_op("cascade::gmm_wgrad", mutates_args=())
def gmm_wgrad_op(x: torch.Tensor, gy: torch.Tensor, idx: torch.Tensor) -> torch.Tensor:
    """gmm_wgrad as an opaque operator (cascade_triton.py:151-153)."""
    return gmm_wgrad(x, gy, idx)


@gmm_wgrad_op.register_fake
def _(x, gy, idx):
    return x.new_empty(gy.shape[2], idx.shape[1] * x.shape[2], dtype=torch.float32)


def target_table(inv: torch.Tensor, NT: int, K: int) -> torch.Tensor:
    """Inverse table (NS, K), value n K + r or NT K = none -> int32 target table, NT = none
    (cascade_triton.py:182)."""
    return torch.where(inv < NT * K, inv // K, torch.full_like(inv, NT)).to(torch.int32)


class GatherMMB200(torch.autograd.Function):
    """Drop-in for cascade_net._GatherMM / cascade_triton.GatherMMTriton (same signature; idx and the inverse table
    as int64 on the device).  Forward and backward on the B200 kernels (cascade_triton.py:161-186)."""

    @staticmethod
    @torch.amp.custom_fwd(device_type="cuda", cast_inputs=torch.bfloat16)
    def forward(ctx, x, w, idx, inv):
        x = x.contiguous()
        w = w.contiguous()
        idx32 = idx.to(torch.int32)
        ctx.save_for_backward(x, w, idx32, inv)
        return gmm_op(x, idx32, w, False)

    @staticmethod
    @torch.amp.custom_bwd(device_type="cuda")
    def backward(ctx, gy):
        x, w, idx32, inv = ctx.saved_tensors
        gy = gy.contiguous().to(x.dtype)
        NT, K = idx32.shape
        gx = gw = None
        if ctx.needs_input_grad[0]:
            gx = gmm_op(gy, target_table(inv, NT, K), w, True)
        if ctx.needs_input_grad[1]:
            gw = gmm_wgrad_op(x, gy, idx32).to(w.dtype)
        return gx, gw, None, None


def _gmm_into(a: torch.Tensor, idx32: torch.Tensor, w: torch.Tensor, out: torch.Tensor) -> None:
    """Forward into a caller's contiguous bf16 (B, NT, C_out) block (the op with an output argument)."""
    B, NS, Ci = a.shape
    NT, K = idx32.shape
    Co = w.shape[0]
    rc = _lib.lib().bpc_gather_mm_fwd(a.data_ptr(), w.data_ptr(), idx32.data_ptr(), out.data_ptr(), B, NS, NT, K, Ci,
                                      Co, _DTYPES[a.dtype], _stream_ptr(a.device))
    _lib.check(rc, "bpc_gather_mm_fwd")


def _dgrad_into(gy: torch.Tensor, tgt32: torch.Tensor, w: torch.Tensor, gx: torch.Tensor, accumulate: bool) -> None:
    """gx (=|+=) the input gradient of one weight set (bpc_gather_mm_dgrad_ex)."""
    B, NT, Co = gy.shape
    NS, K = tgt32.shape
    Ci = w.shape[1] // K
    w_t = torch.empty_like(w)
    rc = _lib.lib().bpc_gather_mm_dgrad_ex(gy.data_ptr(), w.data_ptr(), tgt32.data_ptr(), gx.data_ptr(), w_t.data_ptr(),
                                           B, NT, NS, K, Ci, Co, int(accumulate), _DTYPES[gy.dtype],
                                           _stream_ptr(gy.device))
    _lib.check(rc, "bpc_gather_mm_dgrad_ex")


class BipartiteStepB200(torch.autograd.Function):
    """One residual bipartite step of the training network, y = h + GELU(gather_mm(x, W_t, idx_t)) over T target
    types (targets of type t are the rows [t NT / T, (t + 1) NT / T) of y), as the reference composes it under bf16
    autocast from per-type gather_mm calls, a concatenation, GELU and an add (cascade_net.py:140-175,228-233):
      x (B, NS, C_in) bf16; h (B, NT, C_out) bf16 (-> y bf16), fp32 (-> y fp32 and its bf16 copy, returned as a
      pair: the copy is the next op's input) or None (y = bf16 GELU); ws: T fp32 master weights (C_out, K C_in),
      cast to bf16 here; tables: per type (idx (NT / T, K), target table (NS, K)) int32 on the device.
    The T forwards write one type-major pre-activation block (T, B, NT / T, C_out) that is kept for the backward;
    GELU, the add and the cast run as one pass (bpc_gelu_residual_fwd), the GELU gradient and the residual sum as
    one pass back (bpc_gelu_residual_bwd); the input gradients of the T types accumulate in the second dgrad's
    epilogue, and the weight gradients are fp32 from the deterministic wgrad kernel.

    carry: None, or (dict, give, take) linking two steps of one forward that share a bf16 tensor (the data stream
    h_d, the residual input h of a check -> data step and the input x of the data -> check step before it).  The
    step with give = k hands the residual gradient (its output's gradient, passed through) to dict[k] instead of
    returning it; the step with take = k starts its input gradient from dict[k] and accumulates both types' dgrads into
    it in the kernel's add epilogue, so the two gradients of h_d are summed without a separate add.  The giving step's
    backward always runs first: the taking step's output feeds the giving step's x."""

    @staticmethod
    def forward(ctx, x, h, tables, carry, *ws):
        T = len(ws)
        B, NS, Ci = x.shape
        NTt = tables[0][0].shape[0]
        NT = T * NTt
        w16 = [w.to(torch.bfloat16).contiguous() for w in ws]
        Co = w16[0].shape[0]
        a = torch.empty(T, B, NTt, Co, device=x.device, dtype=torch.bfloat16)
        L = _lib.lib()
        st = _stream_ptr(x.device)
        f32 = h is not None and h.dtype == torch.float32
        y = torch.empty(B, NT, Co, device=x.device, dtype=torch.float32 if f32 else torch.bfloat16)
        y16 = torch.empty(B, NT, Co, device=x.device, dtype=torch.bfloat16) if f32 else None
        hdt = _lib.BPC_DTYPE_F32 if f32 else _lib.BPC_DTYPE_BF16
        K = tables[0][0].shape[1]
        if _FUSED_GELU and x.is_cuda and x.dtype == torch.bfloat16 and Ci in (64, 96, 128) and \
                Co in (64, 96, 128) and K <= 16:
            # the op and the GELU / residual pass in one launch per target type (bpc_gather_mm_fwd_gelu): the
            # epilogue writes the kept pre-activation and this type's block of the residual stream
            x = x.contiguous()
            h = h.contiguous() if h is not None else None
            for t in range(T):
                off = t * NTt * Co
                rc = L.bpc_gather_mm_fwd_gelu(
                    x.data_ptr(), w16[t].data_ptr(), tables[t][0].data_ptr(), a[t].data_ptr(), B, NS, NTt, K, Ci, Co,
                    h.data_ptr() + off * h.element_size() if h is not None else None, hdt,
                    y.data_ptr() + off * y.element_size(), y16.data_ptr() + off * 2 if f32 else None, NT * Co, st)
                _lib.check(rc, "bpc_gather_mm_fwd_gelu")
        else:
            for t in range(T):
                _gmm_into(x, tables[t][0], w16[t], a[t])
            rc = L.bpc_gelu_residual_fwd(a.data_ptr(), h.data_ptr() if h is not None else None, y.data_ptr(),
                                         y16.data_ptr() if f32 else None, B, NT, Co, T, hdt, st)
            _lib.check(rc, "bpc_gelu_residual_fwd")
        ctx.save_for_backward(x, a, *w16)
        ctx.set_materialize_grads(False)     # an unused output's gradient stays None, not a zero-filled tensor
        ctx.tables, ctx.f32, ctx.has_h, ctx.carry = tables, f32, h is not None, carry
        return (y, y16) if f32 else y

    @staticmethod
    def backward(ctx, gy, gy16=None):
        x, a, *w16 = ctx.saved_tensors
        T, B, NTt, Co = a.shape
        NT = T * NTt
        L = _lib.lib()
        st = _stream_ptr(x.device)
        if gy is None and gy16 is None:
            return (None, None, None, None, *([None] * T))
        gh = None
        ga = torch.empty_like(a)
        if ctx.f32:
            gy = gy.float().contiguous() if gy is not None else None
            g16 = gy16.to(torch.bfloat16).contiguous() if gy16 is not None else None
            gh = torch.empty(B, NT, Co, device=x.device, dtype=torch.float32) if ctx.needs_input_grad[1] else None
            rc = L.bpc_gelu_residual_bwd(gy.data_ptr() if gy is not None else None,
                                         g16.data_ptr() if g16 is not None else None, a.data_ptr(),
                                         gh.data_ptr() if gh is not None else None, ga.data_ptr(), B, NT, Co, T,
                                         _lib.BPC_DTYPE_F32, st)
        else:
            gy = gy.to(torch.bfloat16).contiguous()
            rc = L.bpc_gelu_residual_bwd(gy.data_ptr(), None, a.data_ptr(), None, ga.data_ptr(), B, NT, Co, T,
                                         _lib.BPC_DTYPE_BF16, st)
            gh = gy if ctx.has_h and ctx.needs_input_grad[1] else None
        _lib.check(rc, "bpc_gelu_residual_bwd")
        carry = ctx.carry
        if carry is not None and carry[1] is not None and gh is not None and gh.dtype == torch.bfloat16:
            carry[0][carry[1]] = gh                # the taking step adds its input gradient to it
            gh = None
        gx = None
        if ctx.needs_input_grad[0]:
            base = carry[0].pop(carry[2], None) if carry is not None and carry[2] is not None else None
            if base is not None and base.shape == x.shape and base.dtype == x.dtype and base.is_contiguous():
                gx = base
                for t in range(T):
                    _dgrad_into(ga[t], ctx.tables[t][1], w16[t], gx, accumulate=True)
            else:
                gx = torch.empty_like(x)
                for t in range(T):
                    _dgrad_into(ga[t], ctx.tables[t][1], w16[t], gx, accumulate=t > 0)
        gws = [gmm_wgrad(x, ga[t], ctx.tables[t][0]) if ctx.needs_input_grad[4 + t] else None for t in range(T)]
        return (gx, gh, None, None, *gws)


class EmbedTokensB200(torch.autograd.Function):
    """Detector tokens -> the fp32 check stream and its bf16 copy (C ABI bpc_embed_tokens_fwd / _bwd):
    det (B, N) uint8, check_type (N) uint8, E (4, C) fp32 -> (E[2 type + det] fp32, the same in bf16).  The weight
    gradient sums both outputs' gradients per token, deterministically (cascade_net.py:279-285,310-312)."""

    @staticmethod
    def forward(ctx, det, check_type, E):
        B, N = det.shape
        C = E.shape[1]
        det = det.contiguous()
        E = E.float().contiguous()
        h = torch.empty(B, N, C, device=det.device, dtype=torch.float32)
        h16 = torch.empty(B, N, C, device=det.device, dtype=torch.bfloat16)
        rc = _lib.lib().bpc_embed_tokens_fwd(det.data_ptr(), check_type.data_ptr(), E.data_ptr(), h.data_ptr(),
                                             h16.data_ptr(), B, N, C, _stream_ptr(det.device))
        _lib.check(rc, "bpc_embed_tokens_fwd")
        ctx.save_for_backward(det, check_type)
        ctx.set_materialize_grads(False)     # an unused output's gradient stays None
        ctx.C = C
        return h, h16

    @staticmethod
    def backward(ctx, g, g16):
        det, check_type = ctx.saved_tensors
        B, N = det.shape
        C = ctx.C
        L = _lib.lib()
        dE = torch.empty(4, C, device=det.device, dtype=torch.float32)
        ws = torch.empty(max(int(L.bpc_embed_tokens_bwd_workspace_size(C)), 16), device=det.device, dtype=torch.uint8)
        g = g.float().contiguous() if g is not None else None
        g16 = g16.to(torch.bfloat16).contiguous() if g16 is not None else None
        if g is None and g16 is None:
            return None, None, torch.zeros_like(dE)
        rc = L.bpc_embed_tokens_bwd(det.data_ptr(), check_type.data_ptr(), g.data_ptr() if g is not None else None,
                                    g16.data_ptr() if g16 is not None else None, dE.data_ptr(), ws.data_ptr(),
                                    ws.numel(), B, N, C, _stream_ptr(det.device))
        _lib.check(rc, "bpc_embed_tokens_bwd")
        return None, None, dE


class HeadBCEB200(torch.autograd.Function):
    """The training network's head and loss (C ABI bpc_head_bce_fwd / _bwd): hd (..., C) bf16 data stream, W (2, C)
    and b (2) fp32, labels (..., 2) 0/1 -> the mean BCE-with-logits of the bf16 logits linear(hd, W, b), the value
    and the gradients of torch's bf16 autocast composition (F.linear, then binary_cross_entropy_with_logits on the
    logits in fp32) without the logits tensor or the head GEMMs."""

    @staticmethod
    def forward(ctx, hd, W, b, labels):
        C = hd.shape[-1]
        hd = hd.to(torch.bfloat16).contiguous()
        labels = labels.to(torch.uint8).contiguous()
        Wf, bf = W.float().contiguous(), b.float().contiguous()
        rows = hd.numel() // C
        L = _lib.lib()
        ws = torch.empty(int(L.bpc_head_bce_workspace_size(C)), device=hd.device, dtype=torch.uint8)
        loss = torch.empty((), device=hd.device, dtype=torch.float32)
        rc = L.bpc_head_bce_fwd(hd.data_ptr(), Wf.data_ptr(), bf.data_ptr(), labels.data_ptr(), loss.data_ptr(),
                                ws.data_ptr(), ws.numel(), rows, C, _stream_ptr(hd.device))
        _lib.check(rc, "bpc_head_bce_fwd")
        ctx.save_for_backward(hd, Wf, bf, labels)
        ctx.dtypes = (W.dtype, b.dtype)
        return loss

    @staticmethod
    def backward(ctx, go):
        hd, Wf, bf, labels = ctx.saved_tensors
        C = hd.shape[-1]
        rows = hd.numel() // C
        L = _lib.lib()
        ws = torch.empty(int(L.bpc_head_bce_workspace_size(C)), device=hd.device, dtype=torch.uint8)
        go = go.float().contiguous()
        dh = torch.empty_like(hd)
        dW = torch.empty_like(Wf)
        db = torch.empty_like(bf)
        rc = L.bpc_head_bce_bwd(hd.data_ptr(), Wf.data_ptr(), bf.data_ptr(), labels.data_ptr(), go.data_ptr(),
                                dh.data_ptr(), dW.data_ptr(), db.data_ptr(), ws.data_ptr(), ws.numel(), rows, C,
                                _stream_ptr(hd.device))
        _lib.check(rc, "bpc_head_bce_bwd")
        return dh, dW.to(ctx.dtypes[0]), db.to(ctx.dtypes[1]), None


def head_bce(hd, W, b, labels):
    """HeadBCEB200.apply (see there)."""
    return HeadBCEB200.apply(hd, W, b, labels)


def embed_tokens(det, check_type, E):
    """EmbedTokensB200.apply (see there)."""
    return EmbedTokensB200.apply(det, check_type, E)


def bipartite_step(x, h, tables, *ws, carry=None):
    """BipartiteStepB200.apply (see there)."""
    return BipartiteStepB200.apply(x, h, tables, carry, *ws)


def gather_mm(x, w, idx, inv):
    """y[b, n] = W cat_r x[b, idx[n, r]] (cascade_net.py:174-175), on the B200 kernels."""
    return GatherMMB200.apply(x, w, idx, inv)
