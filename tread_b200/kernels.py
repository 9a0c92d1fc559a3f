"""Torch-facing wrappers of the C-ABI kernels (device pointers in, stream-ordered, no host sync).

Each wrapper validates shapes/dtypes/devices on the host and calls the library; there is no
PyTorch fallback path.
"""
import torch

from tread_b200 import _capi as C


def _flat_kv(t, name):
    """A block tensor [L, 1, Hkv, n, D] (tread/store.py layout) or [L, Hkv, n, D] as (LH, n, D)."""
    C.require_cuda(t, name)
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    return t.shape[-2], t.shape[-1]


class RopeAppendPlan:
    """Validated, pre-marshalled arguments of one tread_rope_gather_append call.

    Building the plan checks every segment once; `launch()` then costs one C call, which keeps
    the host far ahead of the GPU when the same assembly is replayed. The plan keeps references
    to its tensors so their memory stays valid.

    segments: iterable of (K, V, delta, dst_tok0); K, V contiguous CUDA tensors whose leading
      dims flatten to the same (layers * kv_heads) as the outputs, shape [..., n, D].
    out_k, out_v: contiguous [..., T_out, D] CUDA tensors of the same dtype.
    inv_freq: D/2 fp32 inverse frequencies (host list or tensor).
    """

    def __init__(self, segments, out_k, out_v, inv_freq, attn_scaling=1.0):
        segs = list(segments)
        for t, nm in ((out_k, "out_k"), (out_v, "out_v")):
            C.require_cuda(t, nm)
            if not t.is_contiguous():
                raise ValueError(f"{nm} must be contiguous")
        if out_k.shape != out_v.shape or out_k.dtype != out_v.dtype:
            raise ValueError("out_k and out_v must have the same shape and dtype")
        C.same_device(out_k, out_v=out_v)
        D = out_k.shape[-1]
        T_out = out_k.shape[-2]
        LH = out_k.numel() // (T_out * D) if T_out * D else 0
        kp, vp, n, dl, d0 = [], [], [], [], []
        for K, V, delta, dst0 in segs:
            nk, dk = _flat_kv(K, "K")
            _flat_kv(V, "V")
            if K.shape != V.shape or dk != D or K.numel() != LH * nk * D:
                raise ValueError(f"segment K/V shape {tuple(K.shape)} does not match output {tuple(out_k.shape)}")
            if K.dtype != out_k.dtype or V.dtype != out_k.dtype:
                raise TypeError("segment dtype differs from the output dtype")
            C.same_device(out_k, K=K, V=V)
            if K.device != out_k.device or V.device != out_k.device:
                raise ValueError("segment and output on different devices")
            kp.append(K.data_ptr())
            vp.append(V.data_ptr())
            n.append(nk)
            dl.append(int(delta))
            d0.append(int(dst0))
        inv = inv_freq.tolist() if isinstance(inv_freq, torch.Tensor) else [float(x) for x in inv_freq]
        if len(inv) != D // 2:
            raise ValueError(f"inv_freq has {len(inv)} entries, expected {D // 2}")
        self.device = out_k.device
        self.nseg = len(segs)
        self._keep = (segs, out_k, out_v)
        self._args = (C.ptr_array(kp), C.ptr_array(vp), C.i32_array(n), C.i64_array(dl), C.i64_array(d0),
                      len(segs), out_k.data_ptr(), out_v.data_ptr(), LH, 1, D, T_out, C.f32_array(inv),
                      float(attn_scaling), C.dtype_code(out_k.dtype))

    def launch(self, stream=None):
        if self.nseg == 0:
            return
        st = C.stream_ptr(self.device) if stream is None else C.P(stream.cuda_stream)
        rc = C.lib().tread_rope_gather_append(*self._args, st)
        C.check(rc, "tread_rope_gather_append")


def rope_gather_append(segments, out_k, out_v, inv_freq, attn_scaling=1.0, stream=None):
    """Assemble cached blocks into out_k/out_v with RoPE re-rotation of K (one launch).
    See RopeAppendPlan for the argument layout."""
    RopeAppendPlan(segments, out_k, out_v, inv_freq, attn_scaling).launch(stream)
    return out_k, out_v


def _stream_arg(stream, device):
    if stream is None:
        return C.stream_ptr(device)
    return C.P(stream.cuda_stream)


def kv_fetch(dst, src, stream=None):
    """Pinned host tensor `src` -> device tensor `dst` (same byte size), async on `stream`."""
    C.require_cuda(dst, "dst")
    if src.is_cuda or not src.is_pinned():
        raise ValueError("kv_fetch source must be a pinned (page-locked) CPU tensor")
    if not (dst.is_contiguous() and src.is_contiguous()) or dst.nbytes != src.nbytes:
        raise ValueError("kv_fetch needs contiguous tensors of equal byte size")
    with torch.cuda.device(dst.device):
        C.check(C.lib().tread_kv_fetch(dst.data_ptr(), src.data_ptr(), dst.nbytes, _stream_arg(stream, dst.device)),
                "tread_kv_fetch")


def kv_spill(dst, src, stream=None):
    """Device tensor `src` -> pinned host tensor `dst` (same byte size), async on `stream`."""
    C.require_cuda(src, "src")
    if dst.is_cuda or not dst.is_pinned():
        raise ValueError("kv_spill destination must be a pinned (page-locked) CPU tensor")
    if not (dst.is_contiguous() and src.is_contiguous()) or dst.nbytes != src.nbytes:
        raise ValueError("kv_spill needs contiguous tensors of equal byte size")
    with torch.cuda.device(src.device):
        C.check(C.lib().tread_kv_spill(dst.data_ptr(), src.data_ptr(), src.nbytes, _stream_arg(stream, src.device)),
                "tread_kv_spill")


def _rows(t, tok0, n):
    """(base pointer, pitch, row bytes, rows) of tokens [tok0, tok0+n) of a [..., T, D] tensor."""
    T, D = t.shape[-2], t.shape[-1]
    es = t.element_size()
    return t.data_ptr() + tok0 * D * es, T * D * es, n * D * es, t.numel() // (T * D)


def kv_spill_rows(dst_host, src_dev, tok0, n, stream=None):
    """Copy tokens [tok0, tok0+n) of every (layer, head) row of a device [..., T, D] cache into the
    same tokens of a pinned host tensor of the same shape."""
    C.require_cuda(src_dev, "src")
    if dst_host.is_cuda or not dst_host.is_pinned() or dst_host.shape != src_dev.shape:
        raise ValueError("kv_spill_rows needs a pinned host tensor of the source's shape")
    if not (dst_host.is_contiguous() and src_dev.is_contiguous()) or tok0 < 0 or tok0 + n > src_dev.shape[-2]:
        raise ValueError("kv_spill_rows: bad token range or non-contiguous tensors")
    d, pitch, rb, rows = _rows(dst_host, tok0, n)
    s, _, _, _ = _rows(src_dev, tok0, n)
    with torch.cuda.device(src_dev.device):
        C.check(C.lib().tread_kv_spill_rows(d, pitch, s, pitch, rb, rows, _stream_arg(stream, src_dev.device)),
                "tread_kv_spill_rows")


# ---- deviation + top-k ----------------------------------------------------------------------

WORKSPACE_BYTES = 256
_workspaces = {}


def workspace(device, stream=None):
    """Zeroed scratch for tread_deviation_topk, one per (device, stream): calls that share one
    must be ordered (the kernel's last CTA resets the ticket counter for the next call)."""
    key = (torch.device(device).index, None if stream is None else stream.cuda_stream)
    ws = _workspaces.get(key)
    if ws is None:
        ws = torch.zeros(WORKSPACE_BYTES // 4, dtype=torch.int32, device=device)
        _workspaces[key] = ws
    return ws


def selector_flags(device):
    """Word 1 of the default-stream selector workspace of `device` (a one-element int32 view): the
    sticky flag the selector kernels set when a candidate position lies outside the cache."""
    return workspace(device)[1:2]


def _rows_view(t, name):
    """(tensor, token stride, head stride) of a [H, n, D] or [1, H, n, D] view with unit last stride."""
    C.require_cuda(t, name)
    if t.dim() == 4:
        if t.shape[0] != 1:
            raise ValueError(f"{name}: leading dim must be 1")
        t = t[0]
    if t.dim() != 3 or t.stride(-1) != 1:
        raise ValueError(f"{name} must be [H, n, D] with contiguous rows")
    return t, t.stride(1), t.stride(0)


def deviation_topk(k1, v1, K1, V1, cand_pos, budget, dev_out=None, sel_idx=None, sel_pos=None, ws=None,
                   stream=None):
    """Layer-1 KV deviation of every candidate and the top-`budget` selection.

    k1, v1: fresh layer-1 K/V rows of the candidates, [H, n, D] (or [1, H, n, D]) views;
    K1, V1: the layer-1 assembled cache [H, T, D] (or [1, H, T, D]);
    cand_pos: int64 CUDA tensor [n], cache position of each candidate.
    Returns (dev fp32 [n], sel_idx int64 [budget] ascending candidate indices,
             sel_pos int64 [budget] = cand_pos[sel_idx]).
    """
    k1, f_st, f_sh = _rows_view(k1, "k1")
    v1, f_st2, f_sh2 = _rows_view(v1, "v1")
    K1, c_st, c_sh = _rows_view(K1, "K1")
    V1, c_st2, c_sh2 = _rows_view(V1, "V1")
    if (f_st, f_sh) != (f_st2, f_sh2) or (c_st, c_sh) != (c_st2, c_sh2):
        raise ValueError("k1/v1 (and K1/V1) must share strides")
    C.same_device(k1, v1=v1, K1=K1, V1=V1, cand_pos=cand_pos, ws=ws)
    H, n, D = k1.shape
    if v1.shape != k1.shape or K1.shape[0] != H or K1.shape[2] != D or V1.shape != K1.shape:
        raise ValueError("shape mismatch between fresh rows and cache")
    if not (k1.dtype == v1.dtype == K1.dtype == V1.dtype):
        raise TypeError("k1, v1, K1, V1 must share a dtype")
    if cand_pos.dtype != torch.int64 or not cand_pos.is_cuda or cand_pos.numel() != n or not cand_pos.is_contiguous():
        raise ValueError("cand_pos must be a contiguous int64 CUDA tensor of length n")
    budget = int(budget)
    if not 0 <= budget <= n:
        raise ValueError(f"budget {budget} outside [0, {n}]")
    dev = k1.device
    if dev_out is None:
        dev_out = torch.empty(n, dtype=torch.float32, device=dev)
    if sel_idx is None:
        sel_idx = torch.empty(budget, dtype=torch.int64, device=dev)
    if sel_pos is None:
        sel_pos = torch.empty(budget, dtype=torch.int64, device=dev)
    C.same_device(k1, dev_out=dev_out, sel_idx=sel_idx, sel_pos=sel_pos)
    if ws is None:
        ws = workspace(dev, stream)
    if n == 0:
        return dev_out, sel_idx, sel_pos
    with torch.cuda.device(dev):
        rc = C.lib().tread_deviation_topk(
            k1.data_ptr(), v1.data_ptr(), f_st, f_sh, K1.data_ptr(), V1.data_ptr(), c_st, c_sh, K1.shape[1],
            cand_pos.data_ptr(), n, H, D, budget, C.dtype_code(k1.dtype), dev_out.data_ptr(),
            sel_idx.data_ptr() if budget else None, sel_pos.data_ptr() if budget else None, ws.data_ptr(),
            _stream_arg(stream, dev))
    C.check(rc, "tread_deviation_topk")
    return dev_out, sel_idx, sel_pos


def deviation_head_norms(k1, v1, K1, V1, cand_pos, norms_out=None, ws=None, stream=None):
    """Per-head layer-1 deviation norms of this rank's KV-head slice: fp32 [2, H, n] (K heads,
    then V heads), each norm computed exactly as inside `deviation_topk`."""
    k1, f_st, f_sh = _rows_view(k1, "k1")
    v1, f_st2, f_sh2 = _rows_view(v1, "v1")
    K1, c_st, c_sh = _rows_view(K1, "K1")
    V1, c_st2, c_sh2 = _rows_view(V1, "V1")
    if (f_st, f_sh) != (f_st2, f_sh2) or (c_st, c_sh) != (c_st2, c_sh2):
        raise ValueError("k1/v1 (and K1/V1) must share strides")
    C.same_device(k1, v1=v1, K1=K1, V1=V1, cand_pos=cand_pos, ws=ws)
    H, n, D = k1.shape
    if v1.shape != k1.shape or K1.shape[0] != H or K1.shape[2] != D or V1.shape != K1.shape:
        raise ValueError("shape mismatch between fresh rows and cache")
    if not (k1.dtype == v1.dtype == K1.dtype == V1.dtype):
        raise TypeError("k1, v1, K1, V1 must share a dtype")
    if cand_pos.dtype != torch.int64 or not cand_pos.is_cuda or cand_pos.numel() != n or not cand_pos.is_contiguous():
        raise ValueError("cand_pos must be a contiguous int64 CUDA tensor of length n")
    dev = k1.device
    if norms_out is None:
        norms_out = torch.empty(2, H, n, dtype=torch.float32, device=dev)
    elif (norms_out.shape != (2, H, n) or norms_out.dtype != torch.float32 or not norms_out.is_contiguous()
          or norms_out.device != k1.device):
        raise ValueError("norms_out must be a contiguous fp32 [2, H, n] tensor on k1's device")
    if ws is None:
        ws = workspace(dev, stream)
    if n == 0:
        return norms_out
    with torch.cuda.device(dev):
        rc = C.lib().tread_deviation_head_norms(
            k1.data_ptr(), v1.data_ptr(), f_st, f_sh, K1.data_ptr(), V1.data_ptr(), c_st, c_sh, K1.shape[1],
            cand_pos.data_ptr(), n, H, D, C.dtype_code(k1.dtype), norms_out.data_ptr(), ws.data_ptr(),
            _stream_arg(stream, dev))
    C.check(rc, "tread_deviation_head_norms")
    return norms_out


def select_head_norms(norms, cand_pos, budget, dev_out=None, sel_idx=None, sel_pos=None, ws=None, stream=None):
    """Deviation and top-`budget` selection from every head's norms, fp32 [2, H, n] in global head
    order (an all-gather of `deviation_head_norms` over the KV-head ranks). Same results as
    `deviation_topk` on a single GPU holding all heads."""
    C.require_cuda(norms, "norms")
    C.same_device(norms, cand_pos=cand_pos, dev_out=dev_out, sel_idx=sel_idx, sel_pos=sel_pos, ws=ws)
    if norms.dim() != 3 or norms.shape[0] != 2 or norms.dtype != torch.float32 or not norms.is_contiguous():
        raise ValueError("norms must be a contiguous fp32 [2, H, n] tensor")
    _, H, n = norms.shape
    if cand_pos.dtype != torch.int64 or not cand_pos.is_cuda or cand_pos.numel() != n or not cand_pos.is_contiguous():
        raise ValueError("cand_pos must be a contiguous int64 CUDA tensor of length n")
    budget = int(budget)
    if not 0 <= budget <= n:
        raise ValueError(f"budget {budget} outside [0, {n}]")
    dev = norms.device
    if dev_out is None:
        dev_out = torch.empty(n, dtype=torch.float32, device=dev)
    if sel_idx is None:
        sel_idx = torch.empty(budget, dtype=torch.int64, device=dev)
    if sel_pos is None:
        sel_pos = torch.empty(budget, dtype=torch.int64, device=dev)
    if ws is None:
        ws = workspace(dev, stream)
    if n == 0:
        return dev_out, sel_idx, sel_pos
    with torch.cuda.device(dev):
        rc = C.lib().tread_select_head_norms(
            norms.data_ptr(), n, H, budget, cand_pos.data_ptr(), dev_out.data_ptr(),
            sel_idx.data_ptr() if budget else None, sel_pos.data_ptr() if budget else None, ws.data_ptr(),
            _stream_arg(stream, dev))
    C.check(rc, "tread_select_head_norms")
    return dev_out, sel_idx, sel_pos


# ---- recompute rows: RoPE + K/V splice, attention -------------------------------------------

def _layer_cache(K, name):
    """A layer cache view [Hkv, T, D] (or [1, Hkv, T, D]) with contiguous [T, D] per head."""
    C.require_cuda(K, name)
    if K.dim() == 4:
        K = K[0]
    if K.dim() != 3 or K.stride(2) != 1 or K.stride(1) != K.shape[2]:
        raise ValueError(f"{name} must be [Hkv, T, D] with contiguous [T, D] planes")
    return K


def rope_rows(qkv, pos, Hq, Hkv, D, q_out, K, V, inv_freq, attn_scaling=1.0, err=None, stream=None,
              kv_by_row=False):
    """Rotate the rows' q heads into q_out [R, Hq, D] (skipped if q_out is None) and splice their
    rotated k / plain v into the layer cache K/V at `pos` (tread/blend.py:82-90,106); with
    kv_by_row, row r's k/v go to cache row r instead (dense [Hkv, R, D] outputs).
    qkv: [R, >= (Hq+2Hkv)*D] with unit column stride; with q_out None and Hq = 0 the rows hold
    only [k heads | v heads]."""
    C.require_cuda(qkv, "qkv")
    K = _layer_cache(K, "K")
    V = _layer_cache(V, "V")
    C.same_device(qkv, pos=pos, q_out=q_out, K=K, V=V, err=err)
    R = qkv.shape[0]
    if qkv.dim() != 2 or qkv.stride(1) != 1:
        raise ValueError("qkv must be 2-D with unit column stride")
    if pos.dtype != torch.int64 or pos.numel() != R or not pos.is_contiguous():
        raise ValueError("pos must be a contiguous int64 tensor of length R")
    if q_out is not None and (q_out.shape != (R, Hq, D) or not q_out.is_contiguous() or q_out.dtype != qkv.dtype):
        raise ValueError("q_out must be a contiguous [R, Hq, D] tensor of qkv's dtype")
    if not (qkv.dtype == K.dtype == V.dtype) or K.stride(0) != V.stride(0) or K.shape != V.shape:
        raise ValueError("dtype/stride mismatch between qkv and the cache")
    if K.shape[0] != Hkv or K.shape[2] != D:
        raise ValueError("cache head count / head_dim do not match")
    inv = inv_freq.tolist() if isinstance(inv_freq, torch.Tensor) else list(inv_freq)
    with torch.cuda.device(qkv.device):
        rc = C.lib().tread_rope_rows(qkv.data_ptr(), qkv.stride(0), pos.data_ptr(), R, Hq, Hkv, D,
                                     None if q_out is None else q_out.data_ptr(), K.data_ptr(), V.data_ptr(),
                                     K.stride(0), K.shape[1], int(bool(kv_by_row)), C.f32_array(inv),
                                     float(attn_scaling), C.dtype_code(qkv.dtype),
                                     None if err is None else err.data_ptr(), _stream_arg(stream, qkv.device))
    C.check(rc, "tread_rope_rows")
    return q_out


_attn_ws = {}


def attn_workspace(device):
    """The zero-filled split-tile workspace of tread_attn_rows on `device` (allocated once, then kept:
    captured CUDA graphs hold its address). Calls sharing it must be stream-ordered."""
    idx = torch.device(device).index
    ws = _attn_ws.get(idx)
    if ws is None:
        with torch.cuda.device(device):
            n = C.lib().tread_attn_rows_workspace_bytes()
        ws = torch.zeros(n, dtype=torch.uint8, device=device)
        _attn_ws[idx] = ws
    return ws


def reset_attn_workspace(device):
    """Zero the workspace's counters again (needed only after a kernel gave up on a wait)."""
    ws = _attn_ws.get(torch.device(device).index)
    if ws is not None:
        ws.zero_()


_SCHEDULES = {None: 0, "stream_k": 2, "tail_split": 4}


def attn_rows(q, K, V, pos, out=None, sm_scale=None, err=None, stream=None, cuda_cores=False, workspace=True,
              schedule=None):
    """Each row of q [R, Hq, D] attends to keys at positions <= pos[row] of the layer cache K/V
    ([Hkv, T, D]) with GQA (tread/blend.py:76,110). Returns out [R, Hq, D]. bf16/fp16 with D=128
    run on tensor cores unless `cuda_cores`. With `workspace` (default) the tensor-core kernel runs
    one CTA per SM over the device's shared workspace: whole row tiles, longest first, with the
    tiles left after the last full round split into key ranges; `schedule` ("tail_split" or
    "stream_k") selects one explicitly. Without it every CTA runs one whole row tile."""
    C.require_cuda(q, "q")
    K = _layer_cache(K, "K")
    V = _layer_cache(V, "V")
    C.same_device(q, K=K, V=V, pos=pos, out=out, err=err)
    R, Hq, D = q.shape
    Hkv = K.shape[0]
    if not q.is_contiguous() or K.shape != V.shape or K.stride(0) != V.stride(0) or K.shape[2] != D:
        raise ValueError("q must be contiguous [R, Hq, D]; K/V [Hkv, T, D] with equal strides")
    if pos.dtype != torch.int64 or pos.numel() != R or not pos.is_contiguous():
        raise ValueError("pos must be a contiguous int64 tensor of length R")
    if out is None:
        out = torch.empty_like(q)
    if sm_scale is None:
        sm_scale = D ** -0.5
    ws = attn_workspace(q.device) if workspace and not cuda_cores else None
    if schedule not in _SCHEDULES:
        raise ValueError(f"schedule must be one of {list(_SCHEDULES)}")
    flags = 1 if cuda_cores else _SCHEDULES[schedule]
    with torch.cuda.device(q.device):
        rc = C.lib().tread_attn_rows(q.data_ptr(), K.data_ptr(), V.data_ptr(), K.stride(0), K.shape[1], pos.data_ptr(),
                                     R, Hq, Hkv, D, float(sm_scale), out.data_ptr(), C.dtype_code(q.dtype), flags,
                                     None if err is None else err.data_ptr(), None if ws is None else ws.data_ptr(),
                                     0 if ws is None else ws.numel(), _stream_arg(stream, q.device))
    C.check(rc, "tread_attn_rows")
    return out


# ---- few-row projections on the tensor cores ----------------------------------------------------

ROWS_GEMM_MAX_ROWS = 128
_gemm_ws = {}


def rows_gemm_workspace(device):
    """The K-split workspace of tread_rows_gemm on `device` (allocated once, then kept: captured CUDA
    graphs hold its address). Calls sharing it must be stream-ordered."""
    idx = torch.device(device).index
    ws = _gemm_ws.get(idx)
    if ws is None:
        with torch.cuda.device(device):
            n = C.lib().tread_rows_gemm_workspace_bytes()
        ws = torch.zeros(n, dtype=torch.uint8, device=device)
        _gemm_ws[idx] = ws
    return ws


def rows_gemm_fits(x, w):
    """True when x [M, K] @ w[N, K]^T can run on tread_rows_gemm: both on one CUDA device, 1..128
    rows, bf16 / fp16, unit column strides, 16-byte aligned rows and K a multiple of 8."""
    return (x.dim() == 2 and w.dim() == 2 and 0 < x.shape[0] <= ROWS_GEMM_MAX_ROWS and x.is_cuda
            and w.device == x.device and x.dtype in (torch.bfloat16, torch.float16) and w.dtype == x.dtype and x.shape[1] == w.shape[1]
            and x.stride(1) == 1 and w.stride(1) == 1 and x.shape[1] % 8 == 0 and x.stride(0) % 8 == 0
            and w.stride(0) % 8 == 0 and x.data_ptr() % 16 == 0 and w.data_ptr() % 16 == 0)


_sm_counts = {}


def rows_gemm_streams_alone(w):
    """True when w [N, K] has at least one pair of 128-feature tiles per SM, so tread_rows_gemm
    streams it in one wave without a K split. Measured on B200 (CUDA-graph replay, 7B shapes),
    those weights (gate/up: 37888 x 3584; lm_head: 151936 x 3584) run at 0.90-1.00 of the HBM copy
    peak, 2-5 % ahead of cuBLAS. The narrower ones need a K split and a second launch, and lose
    about 4 us to cuBLAS on a 26-33 MB weight."""
    idx = w.device.index
    n = _sm_counts.get(idx)
    if n is None:
        n = _sm_counts[idx] = torch.cuda.get_device_properties(w.device).multi_processor_count
    return w.shape[0] >= 256 * n


def rows_gemm(x, w, bias=None, out=None, accumulate=False, err=None, stream=None, split=True):
    """out = (accumulate ? out : 0) + x @ w^T + bias for few rows (x [M <= 128, K], w [N, K], as a
    Linear layer stores its weight), fp32 accumulation rounded once, on the tensor cores with the
    weights streamed from HBM (the query forward's projections, tread/engine.py:131-132). With
    `split` (default) weights with fewer 256-feature pairs than SMs are split along K over more CTAs
    through the device's shared workspace; the splits are added in a fixed order, so results are
    deterministic."""
    C.require_cuda(x, "x")
    C.same_device(x, w=w, bias=bias, out=out, err=err)
    if not rows_gemm_fits(x, w):
        raise ValueError("rows_gemm: x [M <= 128, K] and w [N, K] must be bf16/fp16 with unit column strides, "
                         "16-byte aligned rows and K % 8 == 0")
    M, K = x.shape
    N = w.shape[0]
    if bias is not None and (bias.shape != (N,) or bias.dtype != x.dtype or not bias.is_contiguous()
                             or bias.device != x.device):
        raise ValueError("rows_gemm: bias must be a contiguous [N] tensor of x's dtype on x's device")
    if out is None:
        if accumulate:
            raise ValueError("rows_gemm: accumulate needs out")
        out = torch.empty(M, N, dtype=x.dtype, device=x.device)
    elif out.shape != (M, N) or out.dtype != x.dtype or out.stride(1) != 1 or out.device != x.device:
        raise ValueError("rows_gemm: out must be [M, N] of x's dtype with unit column stride, on x's device")
    ws = rows_gemm_workspace(x.device) if split else None
    with torch.cuda.device(x.device):
        rc = C.lib().tread_rows_gemm(x.data_ptr(), x.stride(0), w.data_ptr(), w.stride(0),
                                     None if bias is None else bias.data_ptr(), out.data_ptr(), out.stride(0), M, N,
                                     K, 1 if accumulate else 0, C.dtype_code(x.dtype),
                                     None if err is None else err.data_ptr(), None if ws is None else ws.data_ptr(),
                                     0 if ws is None else ws.numel(), _stream_arg(stream, x.device))
    C.check(rc, "tread_rows_gemm")
    return out


# ---- fused row-wise layer pieces ----------------------------------------------------------------

def rmsnorm(x, weight, eps, out=None, stream=None):
    """HF Qwen2RMSNorm over the rows of x [R, H] (unit column stride) in one pass."""
    C.require_cuda(x, "x")
    C.same_device(x, weight=weight, out=out)
    if x.dim() != 2 or x.stride(1) != 1 or weight.shape != (x.shape[1],) or weight.dtype != x.dtype:
        raise ValueError("rmsnorm: x must be [R, H] with unit column stride and weight [H] of x's dtype")
    if out is None:
        out = torch.empty_like(x, memory_format=torch.contiguous_format)
    with torch.cuda.device(x.device):
        rc = C.lib().tread_rmsnorm(x.data_ptr(), x.stride(0), weight.data_ptr(), out.data_ptr(), out.stride(0),
                                   x.shape[0], x.shape[1], float(eps), C.dtype_code(x.dtype),
                                   _stream_arg(stream, x.device))
    C.check(rc, "tread_rmsnorm")
    return out


def silu_mul(gate_up, out=None, stream=None):
    """silu(g) * u of HF Qwen2MLP, gate_up = [g | u] of shape [R, 2I] (unit column stride)."""
    C.require_cuda(gate_up, "gate_up")
    C.same_device(gate_up, out=out)
    if gate_up.dim() != 2 or gate_up.stride(1) != 1 or gate_up.shape[1] % 2:
        raise ValueError("silu_mul: gate_up must be [R, 2I] with unit column stride")
    R, I = gate_up.shape[0], gate_up.shape[1] // 2
    if out is None:
        out = torch.empty(R, I, dtype=gate_up.dtype, device=gate_up.device)
    with torch.cuda.device(gate_up.device):
        rc = C.lib().tread_silu_mul(gate_up.data_ptr(), gate_up.stride(0), out.data_ptr(), out.stride(0), R, I,
                                    C.dtype_code(gate_up.dtype), _stream_arg(stream, gate_up.device))
    C.check(rc, "tread_silu_mul")
    return out
