"""ctypes binding of the tread_b200 C ABI (`include/tread_b200.h`).

The library is loaded from the package tree (`tread_b200/_lib/libtread_b200.so`). There is
no fallback: if the library is missing or a call fails, a RuntimeError says why.
"""
import ctypes
import os

import torch

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_lib", "libtread_b200.so")

TREAD_F32, TREAD_F16, TREAD_BF16 = 0, 1, 2
_DTYPE = {torch.float32: TREAD_F32, torch.float16: TREAD_F16, torch.bfloat16: TREAD_BF16}

P = ctypes.c_void_p
I32 = ctypes.c_int32
I64 = ctypes.c_int64
F32 = ctypes.c_float
PP = ctypes.POINTER(ctypes.c_void_p)
PI32 = ctypes.POINTER(ctypes.c_int32)
PI64 = ctypes.POINTER(ctypes.c_int64)
PF32 = ctypes.POINTER(ctypes.c_float)

# name -> (restype, argtypes), mirroring include/tread_b200.h
SIGNATURES = {
    "tread_last_error": (ctypes.c_char_p, []),
    "tread_abi_version": (ctypes.c_int, []),
    "tread_rope_gather_append": (
        ctypes.c_int,
        [PP, PP, PI32, PI64, PI64, ctypes.c_int, P, P, ctypes.c_int, ctypes.c_int, ctypes.c_int, I64, PF32,
         F32, ctypes.c_int, P],
    ),
    "tread_deviation_topk": (
        ctypes.c_int,
        [P, P, I64, I64, P, P, I64, I64, I64, P, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
         ctypes.c_int, P, P, P, P, P],
    ),
    "tread_deviation_topk_noalloc": (
        ctypes.c_int,
        [P, P, I64, I64, P, P, I64, I64, I64, P, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
         ctypes.c_int, P, P, P, P],
    ),
    "tread_deviation_head_norms": (
        ctypes.c_int,
        [P, P, I64, I64, P, P, I64, I64, I64, P, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, P, P, P],
    ),
    "tread_select_head_norms": (
        ctypes.c_int,
        [P, ctypes.c_int, ctypes.c_int, ctypes.c_int, P, P, P, P, P, P],
    ),
    "tread_rope_rows": (
        ctypes.c_int,
        [P, I64, P, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, P, P, P, I64, I64, ctypes.c_int, PF32,
         F32, ctypes.c_int, P, P],
    ),
    "tread_attn_rows_workspace_bytes": (ctypes.c_size_t, []),
    "tread_attn_rows": (
        ctypes.c_int,
        [P, P, P, I64, I64, P, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, F32, P, ctypes.c_int,
         ctypes.c_int, P, P, ctypes.c_size_t, P],
    ),
    "tread_rows_gemm_workspace_bytes": (ctypes.c_size_t, []),
    "tread_rows_gemm": (
        ctypes.c_int,
        [P, I64, P, I64, P, P, I64, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, P, P,
         ctypes.c_size_t, P],
    ),
    "tread_rmsnorm": (ctypes.c_int, [P, I64, P, P, I64, I64, ctypes.c_int, F32, ctypes.c_int, P]),
    "tread_silu_mul": (ctypes.c_int, [P, I64, P, I64, I64, ctypes.c_int, ctypes.c_int, P]),
    "tread_kv_fetch": (ctypes.c_int, [P, P, ctypes.c_size_t, P]),
    "tread_kv_spill": (ctypes.c_int, [P, P, ctypes.c_size_t, P]),
    "tread_kv_fetch_rows": (ctypes.c_int, [P, ctypes.c_size_t, P, ctypes.c_size_t, ctypes.c_size_t,
                                           ctypes.c_size_t, P]),
    "tread_kv_spill_rows": (ctypes.c_int, [P, ctypes.c_size_t, P, ctypes.c_size_t, ctypes.c_size_t,
                                           ctypes.c_size_t, P]),
}

_lib = None


def lib():
    """Load the library once and attach the declared signatures."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"tread_b200 CUDA library not built ({LIB_PATH} missing); run `python -m tread_b200.build`")
        handle = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def check(rc, what):
    if rc != 0:
        msg = lib().tread_last_error().decode(errors="replace")
        raise RuntimeError(f"{what} failed (status {rc}): {msg}")


def dtype_code(dtype):
    try:
        return _DTYPE[dtype]
    except KeyError:
        raise TypeError(f"unsupported dtype {dtype}; expected float32, float16 or bfloat16") from None


def stream_ptr(device=None):
    return P(torch.cuda.current_stream(device).cuda_stream)


def ptr_array(ptrs):
    return (ctypes.c_void_p * len(ptrs))(*ptrs)


def i32_array(vals):
    return (ctypes.c_int32 * len(vals))(*vals)


def i64_array(vals):
    return (ctypes.c_int64 * len(vals))(*vals)


def f32_array(vals):
    return (ctypes.c_float * len(vals))(*vals)


def require_cuda(t, name):
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (got {t.device}); tread_b200 has no CPU path")


def same_device(ref, **tensors):
    """Every tensor given (None skips) must sit on ref's device: the kernels dereference them all
    there, so a host or other-GPU tensor is refused before anything launches."""
    for name, t in tensors.items():
        if t is not None and t.device != ref.device:
            raise ValueError(f"{name} is on {t.device}, the call's other tensors on {ref.device}")
