"""TEST INFRASTRUCTURE ONLY: Python side of the CPU oracle for tread's hot path.

Restates the reference's algorithms on the CPU (numpy, plus the C library built from
`oracle/oracle_tread.c`) so that tests can check the CUDA kernels of `tread_b200` on the
same seeded inputs. Only `tests/`, `__graft_entry__.smoke()` and bench.py's CPU-baseline
leg use this module; the product never imports it.

Pinning: every function here is checked against golden vectors produced by the reference
itself (tests/golden/make_golden.py, imported from the unmodified tread sources) in
tests/test_oracle_golden.py.

bf16 arrays are carried as numpy uint16 bit patterns.
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_lib", "liboracle_tread.so")
F32, F16, BF16 = 0, 1, 2

_lib = None


def build():
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        h = ctypes.CDLL(LIB_PATH)
        P, PP = ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p)
        h.oracle_rope_cos_sin.argtypes = [ctypes.c_int64, P, ctypes.c_int, ctypes.c_float, P, P]
        h.oracle_rope_cos_sin.restype = None
        h.oracle_rope_gather_append.argtypes = [
            PP, PP, P, P, P, ctypes.c_int, P, P, ctypes.c_int, ctypes.c_int, ctypes.c_int64, P, ctypes.c_float,
            ctypes.c_int, ctypes.c_int, ctypes.c_int]
        h.oracle_rope_gather_append.restype = None
        h.oracle_max_threads.restype = ctypes.c_int
        h.oracle_deviation.argtypes = [P, P, ctypes.c_int64, ctypes.c_int64, P, P, ctypes.c_int64, ctypes.c_int64, P,
                                       ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, P]
        h.oracle_deviation.restype = None
        _lib = h
    return _lib


def max_threads():
    return lib().oracle_max_threads()


# ---- bf16 helpers ------------------------------------------------------------------------

def bf16_to_f32(bits):
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(x):
    """Round-to-nearest-even fp32 -> bf16 bit pattern."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def bf16_ulp(x):
    """Spacing of bf16 numbers at |x| (for normal numbers: 2^(exponent-7))."""
    x = np.abs(np.asarray(x, dtype=np.float32))
    e = np.floor(np.log2(np.maximum(x, np.float32(2.0 ** -126))))
    return np.float32(2.0) ** (e - 7)


def _np_code(a):
    if a.dtype == np.float32:
        return F32
    if a.dtype == np.float16:
        return F16
    if a.dtype == np.uint16:
        return BF16
    raise TypeError(a.dtype)


# ---- A1/A2: rotate_keys + assembly (tread/blend.py:22-39, tread/engine.py:108-120) --------

def rope_cos_sin(delta, inv_freq, scale=1.0):
    inv = np.ascontiguousarray(inv_freq, dtype=np.float32)
    half = inv.shape[0]
    c = np.empty(half, np.float32)
    s = np.empty(half, np.float32)
    lib().oracle_rope_cos_sin(int(delta), inv.ctypes.data, half, float(scale), c.ctypes.data, s.ctypes.data)
    return c, s


def rope_gather_append(segments, T_out, inv_freq, scale=1.0, out_dtype=None, nthreads=0, out=None):
    """segments: list of (K, V, delta, dst_tok0) with K, V numpy arrays [..., n, D] (same leading
    dims for all segments). Returns (out_k, out_v) with shape [..., T_out, D].
    out_dtype: F32 / F16 / BF16 code (default: the input type)."""
    K0 = segments[0][0]
    lead = K0.shape[:-2]
    D = K0.shape[-1]
    LH = int(np.prod(lead)) if lead else 1
    in_code = _np_code(K0)
    out_code = in_code if out_dtype is None else out_dtype
    np_out = {F32: np.float32, F16: np.float16, BF16: np.uint16}[out_code]
    if out is None:
        out_k = np.zeros(lead + (T_out, D), np_out)
        out_v = np.zeros(lead + (T_out, D), np_out)
    else:
        out_k, out_v = out
    ks = [np.ascontiguousarray(s[0]) for s in segments]
    vs = [np.ascontiguousarray(s[1]) for s in segments]
    for k, v in zip(ks, vs):
        assert k.shape[:-2] == lead and k.shape[-1] == D and _np_code(k) == in_code and v.shape == k.shape
    kp = (ctypes.c_void_p * len(ks))(*[k.ctypes.data for k in ks])
    vp = (ctypes.c_void_p * len(vs))(*[v.ctypes.data for v in vs])
    n = np.array([k.shape[-2] for k in ks], np.int32)
    delta = np.array([s[2] for s in segments], np.int64)
    dst0 = np.array([s[3] for s in segments], np.int64)
    inv = np.ascontiguousarray(inv_freq, dtype=np.float32)
    lib().oracle_rope_gather_append(kp, vp, n.ctypes.data, delta.ctypes.data, dst0.ctypes.data, len(ks),
                                    out_k.ctypes.data, out_v.ctypes.data, LH, D, T_out, inv.ctypes.data,
                                    float(scale), in_code, out_code, int(nthreads))
    return out_k, out_v


def inv_freq(head_dim, theta):
    """HF default RoPE inverse frequencies (transformers Qwen2RotaryEmbedding
    .compute_default_rope_parameters): 1 / theta ** (arange(0, D, 2) / D), in fp32."""
    import torch

    return (1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64).to(torch.float) / head_dim))).numpy()


# ---- A4: deviation + selection (tread/blend.py:117-130, 145, 158-169) -----------------------

def deviation(k1, v1, K1, V1, cand_pos):
    """dev[t] in the kernel's fixed fp32 order. k1, v1: [H, n, D] fresh layer-1 rows; K1, V1:
    [H, T, D] layer-1 cache; cand_pos: [n] positions. Arrays: float32 / float16 / uint16 (bf16)."""
    k1, v1, K1, V1 = (np.ascontiguousarray(a) for a in (k1, v1, K1, V1))
    H, n, D = k1.shape
    T = K1.shape[1]
    pos = np.ascontiguousarray(cand_pos, dtype=np.int64)
    assert v1.shape == k1.shape and K1.shape == V1.shape == (H, T, D) and pos.shape == (n,)
    assert ((pos >= 0) & (pos < T)).all()
    dev = np.empty(n, np.float32)
    lib().oracle_deviation(k1.ctypes.data, v1.ctypes.data, D, n * D, K1.ctypes.data, V1.ctypes.data, D, T * D,
                           pos.ctypes.data, n, H, D, _np_code(k1), dev.ctypes.data)
    return dev


def head_norms(k1, v1, K1, V1, cand_pos):
    """Per-head terms of tread/blend.py:129 in the kernel's fixed order: [2, H, n] fp32 with
    [0, h, t] = ||k1[h,t] - K1[h,pos_t]|| and [1, h, t] the same for V. Each term is the
    single-head `deviation` with the other side's rows set equal (so that side adds an exact 0)."""
    k1, v1, K1, V1 = (np.ascontiguousarray(a) for a in (k1, v1, K1, V1))
    H, n, D = k1.shape
    zf = np.zeros((1, n, D), k1.dtype)
    zc = np.zeros((1, K1.shape[1], D), K1.dtype)
    out = np.empty((2, H, n), np.float32)
    for h in range(H):
        out[0, h] = deviation(k1[h:h + 1], zf, K1[h:h + 1], zc, cand_pos)
        out[1, h] = deviation(zf, v1[h:h + 1], zc, V1[h:h + 1], cand_pos)
    return out


def dev_from_head_norms(norms):
    """dev[t] = (((nk_0 + nk_1) + ...) + ((nv_0 + nv_1) + ...)) in fp32, the fused kernel's order
    (tread/blend.py:129 sums K and V norms over heads)."""
    a = np.zeros(norms.shape[2], np.float32)
    b = np.zeros(norms.shape[2], np.float32)
    for h in range(norms.shape[1]):
        a = (a + norms[0, h]).astype(np.float32)
    for h in range(norms.shape[1]):
        b = (b + norms[1, h]).astype(np.float32)
    return (a + b).astype(np.float32)


def order_key(dev):
    """Order-preserving uint32 image of fp32 values (NaN above +inf, as torch.topk ranks it)."""
    u = np.ascontiguousarray(dev, dtype=np.float32).view(np.uint32)
    return np.where(u & 0x80000000, ~u, u | 0x80000000).astype(np.uint32)


def select_topk(dev, budget):
    """Indices of the `budget` largest values, ties toward the lower index, returned ascending
    (the set sort(topk(dev, budget).indices), tread/blend.py:160,165)."""
    key = order_key(dev).astype(np.int64)
    order = np.argsort(-key, kind="stable")
    return np.sort(order[:budget])


def budget_for(ratio, n):
    """tread/blend.py:145: int(round(ratio * n)) with Python's round-half-to-even."""
    return int(round(ratio * n))
