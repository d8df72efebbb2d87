"""ctypes binding of libbpc.so, the C-ABI library that holds every kernel of this package.

The library must exist (codecoder_b200.build); there is no fallback: a missing library raises at first use."""
from __future__ import annotations

import ctypes
import os

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("BPC_LIB", os.path.join(_PKG, "libbpc.so"))

BPC_DTYPE_F32 = 0
BPC_DTYPE_BF16 = 1
BPC_EPILOGUE_STORE = 0
BPC_EPILOGUE_AFFINE_SILU = 1
BPC_EPILOGUE_ADD = 2

c_i32 = ctypes.c_int32
c_i64 = ctypes.c_int64
c_vp = ctypes.c_void_p


class PredecoderConfig(ctypes.Structure):
    _fields_ = [("layers", c_i32), ("channels", c_i32), ("K", c_i32), ("dtype", c_i32), ("n_checks", c_i32),
                ("n_data", c_i32), ("z_check_begin", c_i32)]


# name -> (restype, argtypes), in the order include/bpc.h declares them
SIGNATURES = {
    "bpc_version": (ctypes.c_int, []),
    "bpc_last_error": (ctypes.c_int, [ctypes.c_char_p, ctypes.c_int]),
    "bpc_gather_mm_fwd": (ctypes.c_int, [c_vp, c_vp, c_vp, c_vp, c_i64, c_i32, c_i32, c_i32, c_i32, c_i32, c_i32,
                                         c_vp]),
    "bpc_gather_mm_fwd_ex": (ctypes.c_int, [c_vp, c_vp, c_vp, c_vp, c_i64, c_i32, c_i32, c_i32, c_i32, c_i32, c_i32,
                                            c_i32, c_i32, c_vp, c_vp, c_i32, c_vp]),
    "bpc_route": (ctypes.c_int, [c_vp, c_vp, c_i64, c_i32, c_i32, ctypes.c_float, c_i32, c_vp, c_vp, c_vp, c_vp, c_vp,
                                 c_vp, c_vp, ctypes.c_size_t, c_vp]),
    "bpc_route_workspace_size": (ctypes.c_size_t, [c_i64]),
    "bpc_cascade_boundary": (ctypes.c_int, [c_vp, c_vp, c_vp, c_vp, ctypes.c_float, ctypes.c_float, c_vp, c_vp, c_vp,
                                            c_vp, c_vp, c_vp, c_i64, c_i32, c_i32, c_vp]),
    "bpc_cascade_boundary_tokens": (ctypes.c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_i32, c_i32, c_vp,
                                                   ctypes.c_float, ctypes.c_float, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp,
                                                   c_i64, c_i32, c_i32, c_vp]),
    "bpc_cascade_stem": (ctypes.c_int, [c_vp, c_vp, c_vp, c_vp, c_i32, c_i32, c_vp, c_vp, c_vp, c_i64, c_i32, c_vp]),
    "bpc_residual_affine_silu": (ctypes.c_int, [c_vp, c_vp, c_vp, c_vp, c_i64, c_i32, ctypes.c_float, ctypes.c_float,
                                                c_vp, c_vp, c_vp]),
    "bpc_gelu_residual_fwd": (ctypes.c_int, [c_vp, c_vp, c_vp, c_vp, c_i64, c_i32, c_i32, c_i32, c_i32, c_vp]),
    "bpc_gelu_residual_bwd": (ctypes.c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_i64, c_i32, c_i32, c_i32, c_i32, c_vp]),
    "bpc_embed_tokens_fwd": (ctypes.c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_i64, c_i32, c_i32, c_vp]),
    "bpc_embed_tokens_bwd_workspace_size": (ctypes.c_size_t, [c_i32]),
    "bpc_head_bce_workspace_size": (ctypes.c_size_t, [c_i32]),
    "bpc_head_bce_fwd": (ctypes.c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, ctypes.c_size_t, c_i64, c_i32, c_vp]),
    "bpc_head_bce_bwd": (ctypes.c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, ctypes.c_size_t, c_i64,
                                        c_i32, c_vp]),
    "bpc_embed_tokens_bwd": (ctypes.c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, ctypes.c_size_t, c_i64, c_i32, c_i32,
                                            c_vp]),
    "bpc_gather_mm_fwd_gelu": (ctypes.c_int, [c_vp, c_vp, c_vp, c_vp, c_i64, c_i32, c_i32, c_i32, c_i32, c_i32, c_vp,
                                              c_i32, c_vp, c_vp, c_i64, c_vp]),
    "bpc_gather_mm_dgrad": (ctypes.c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_i64, c_i32, c_i32, c_i32, c_i32, c_i32,
                                           c_i32, c_vp]),
    "bpc_gather_mm_dgrad_ex": (ctypes.c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_i64, c_i32, c_i32, c_i32, c_i32, c_i32,
                                              c_i32, c_i32, c_vp]),
    "bpc_gather_mm_wgrad": (ctypes.c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, ctypes.c_size_t, c_i64, c_i32, c_i32, c_i32,
                                           c_i32, c_i32, c_i32, c_vp]),
    "bpc_gather_mm_wgrad_workspace_size": (ctypes.c_size_t, [c_i64, c_i32, c_i32, c_i32, c_i32, c_i32, c_i32]),
    "bpc_gather_mm_status": (ctypes.c_int, [c_vp, ctypes.POINTER(ctypes.c_int)]),
    "bpc_predecoder_create": (ctypes.c_int, [ctypes.POINTER(PredecoderConfig), c_vp, c_vp, c_vp, c_vp, c_vp,
                                             ctypes.POINTER(c_vp)]),
    "bpc_predecoder_set_weights": (ctypes.c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_vp]),
    "bpc_predecoder_workspace_size": (ctypes.c_size_t, [c_vp, c_i64]),
    "bpc_predecoder_forward": (ctypes.c_int, [c_vp, c_vp, c_vp, c_vp, c_i64, c_vp, ctypes.c_size_t, c_vp]),
    "bpc_predecoder_record_step_events": (ctypes.c_int, [c_vp, ctypes.POINTER(c_vp), ctypes.c_int]),
    "bpc_predecoder_status": (ctypes.c_int, [c_vp, c_vp, ctypes.POINTER(ctypes.c_int)]),
    "bpc_predecoder_destroy": (None, [c_vp]),
    "bpc_predecoder_forward_noalloc": (ctypes.c_int, [c_vp, c_vp, c_vp, c_vp, c_i64, c_vp]),
    "bpc_stream_create": (ctypes.c_int, [c_vp, c_i32, c_i32, c_i32, c_i32, ctypes.POINTER(c_vp)]),
    "bpc_stream_create_ex": (ctypes.c_int, [c_vp, c_i32, c_i32, c_i32, c_i32, c_i32, ctypes.POINTER(c_vp)]),
    "bpc_stream_start": (ctypes.c_int, [c_vp]),
    "bpc_stream_round": (ctypes.c_int, [c_vp, c_vp, c_vp, c_vp, c_i64]),
    "bpc_stream_run": (ctypes.c_int, [c_vp, c_vp, c_i64, c_vp, c_vp, c_vp, c_i64]),
    "bpc_stream_stop": (ctypes.c_int, [c_vp]),
    "bpc_stream_status": (ctypes.c_int, [c_vp]),
    "bpc_stream_layout": (ctypes.c_int, [c_vp]),
    "bpc_stream_trace": (ctypes.c_int, [c_vp, c_i32]),
    "bpc_stream_trace_read": (ctypes.c_int, [c_vp, c_vp, c_i64]),
    "bpc_stream_destroy": (None, [c_vp]),
    "bpc_noalloc_scratch_bytes": (ctypes.c_size_t, []),
}

_lib = None


def lib() -> ctypes.CDLL:
    """The loaded library (loaded once, with argument types set)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m codecoder_b200.build`")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def last_error() -> str:
    buf = ctypes.create_string_buffer(1024)
    lib().bpc_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(rc: int, what: str) -> None:
    if rc != 0:
        raise RuntimeError(f"{what} failed ({rc}): {last_error()}")
