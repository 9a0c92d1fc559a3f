"""Chunk KV prefill, RoPE re-rotation and selective recompute (blending) on B200 kernels.

Same functions, arguments and results as tread/blend.py (KV tensors are [1, kv_heads, T,
head_dim] per layer, keys post-RoPE as HF's DynamicCache holds them), implemented on the
tread_b200 C ABI:
  rotate_keys    -> tread_rope_gather_append (one launch, fp32 rotation, no temporaries)
  deviation/top-k-> tread_deviation_topk (fixed-order fp32 dev, deterministic selection)
  recompute layer-> tread_rope_rows (RoPE + in-place K/V splice) + tread_attn_rows (GQA
                    attention under the key_pos <= row_pos mask) around cuBLAS projections
"""
import torch
from transformers import DynamicCache

from tread_b200 import kernels
from tread_b200.qwen2 import Qwen2Rows


def rows_of(model) -> Qwen2Rows:
    """The layer math bound to `model` (built once, cached on the model object). A rows object
    (e.g. a KV-head tensor-parallel shard, tread_b200.tp) stands for its model and is returned
    as is."""
    if isinstance(model, Qwen2Rows):
        return model
    r = getattr(model, "_tread_b200_rows", None)
    if r is None:
        r = Qwen2Rows(model)
        model._tread_b200_rows = r
    return r


def _inv_freq(model):
    net = rows_of(model)
    return net.inv_freq, net.attn_scaling


def prefill_kv(model, ids):
    """Per-layer (K, V) lists of a forward over `ids` at positions 0..n-1 (tread/blend.py:12-19)."""
    net = rows_of(model)
    n = len(ids)
    K, V = net.new_cache(n)
    pos = torch.arange(n, device=ids.device)
    net.run(net.embed_ids(ids), pos, list(K.unbind(0)), list(V.unbind(0)))
    return list(K.unbind(0)), list(V.unbind(0))


def rotate_keys(model, K, delta):
    """Shift post-RoPE keys by `delta` positions: R(p + delta) = R(delta) @ R(p)
    (tread/blend.py:22-39). K may have any leading dims; returns K itself for delta == 0."""
    if delta == 0:
        return K
    inv, scale = _inv_freq(model)
    Kc = K.contiguous()
    out = torch.empty_like(Kc)
    kernels.rope_gather_append([(Kc, Kc, int(delta), 0)], out, torch.empty_like(Kc), inv, scale)
    return out


def chunk_kv(model, prefix_ids, doc_ids, mode):
    """KV for one document computed independently of other documents (tread/blend.py:42-54)."""
    if mode == "shared":
        K, V = prefill_kv(model, torch.cat([prefix_ids, doc_ids]))
        P = len(prefix_ids)
        return [k[:, :, P:] for k in K], [v[:, :, P:] for v in V], P
    K, V = prefill_kv(model, doc_ids)
    return K, V, 0


def assemble(model, prefix_ids, docs_ids, mode):
    """Exact prefix KV + independently computed, re-rotated doc KV (tread/blend.py:57-68)."""
    Kp, Vp = prefill_kv(model, prefix_ids)
    Ks, Vs = [[k] for k in Kp], [[v] for v in Vp]
    offset = len(prefix_ids)
    for d in docs_ids:
        Kd, Vd, base = chunk_kv(model, prefix_ids, d, mode)
        for l in range(len(Ks)):
            Ks[l].append(rotate_keys(model, Kd[l].contiguous(), offset - base))
            Vs[l].append(Vd[l])
        offset += len(d)
    return [torch.cat(x, dim=2) for x in Ks], [torch.cat(x, dim=2) for x in Vs]


def _deviation_pass(net, ctx_ids, K, V, all_c, inplace, extra, budget):
    """Layer 0 over every candidate (+ `extra` rows), fresh layer-1 k/v of the candidates, then
    the fused deviation + top-`budget` kernel against K[1], V[1] (tread/blend.py:117-130,160,165).
    Returns (dev, sel_idx, S, candidates' layer-0 hidden, K0, V0, extra rows' layer-0 hidden)."""
    n = len(all_c)
    K0, V0 = (K[0], V[0]) if inplace else (K[0].clone(), V[0].clone())
    h = net.embed_ids(ctx_ids[all_c])
    pos = all_c
    if extra is not None:
        h = torch.cat([h, extra[0]])
        pos = torch.cat([all_c, extra[1]])
    h = net.layer(0, h, pos, K0, V0)
    hc = h[:n]
    kv1 = net.kv(1, hc)  # k/v columns only
    k1 = torch.empty(net.Hkv, n, net.D, dtype=hc.dtype, device=hc.device)
    v1 = torch.empty_like(k1)
    kernels.rope_rows(kv1, all_c, 0, net.Hkv, net.D, None, k1, v1, net.inv_freq, net.attn_scaling, net.err,
                      kv_by_row=True)
    dev, sel_idx, S = net.deviation_select(k1, v1, K[1], V[1], all_c, budget)
    return dev, sel_idx, S, hc, K0, V0, (h[n:] if extra is not None else None)


def layer1_deviation(model, ctx_ids, K, V, all_c, inplace=False):
    """Per-token drift of reused layer-1 KV from a fresh recompute (tread/blend.py:117-130).

    Layer 0 is recomputed for every candidate (its fresh K/V spliced into K[0], V[0]); the fresh
    layer-1 k/v of the candidates are compared with K[1], V[1] at their positions.
    Returns (dev [len(all_c)], layer-0 hidden for all_c, fresh layer-0 K, fresh layer-0 V).
    """
    dev, _, _, hc, K0, V0, _ = _deviation_pass(rows_of(model), ctx_ids, K, V, all_c, inplace, None, 0)
    return dev, hc, K0, V0


def select(model, ctx_ids, K, V, candidates, ratio, policy, gen=None, inplace=False, extra=None):
    """Budget + policy of tread/blend.py:143-169 (K[0], V[0] are replaced by the layer-0-spliced
    caches for "deviation"). Returns (S sorted, hidden rows for S or None when the caller embeds
    them, start layer, all_c, layer-0 hidden of the `extra` rows or None)."""
    net = rows_of(model)
    all_c = torch.cat(candidates)
    budget = int(round(ratio * len(all_c)))
    if budget == 0:
        return all_c[:0], None, 0, all_c, None
    if policy == "boundary":
        # Water-fill: the first w tokens of every doc; short docs run out first.
        rank = torch.cat([torch.arange(len(c), device=c.device) for c in candidates])
        S = all_c[rank.argsort(stable=True)[:budget]]
        return S.sort().values, None, 0, all_c, None
    if policy == "random":
        S = all_c[torch.randperm(len(all_c), generator=gen, device="cpu").to(all_c.device)[:budget]]
        return S.sort().values, None, 0, all_c, None
    if policy == "deviation":
        _, sel_idx, S, hc, K[0], V[0], hx = _deviation_pass(net, ctx_ids, K, V, all_c, inplace, extra, budget)
        return S, hc[sel_idx], 1, all_c, hx
    raise ValueError(policy)


def blend(model, ctx_ids, K, V, candidates, ratio, policy, gen=None, inplace=False, runner=None):
    """Selectively recompute a `ratio` fraction of `candidates` (tread/blend.py:133-179).

    Returns new (K, V) lists, the selected positions S (sorted) and the effective recompute ratio
    in token-layers (deviation also pays for recomputing layer 0 over every candidate).
    """
    K, V = list(K), list(V)
    if not candidates:
        return K, V, torch.empty(0, dtype=torch.long, device=K[0].device), 0.0
    net = rows_of(model)
    S, h, start, all_c, _ = select(model, ctx_ids, K, V, candidates, ratio, policy, gen, inplace)
    if len(S) == 0:
        return K, V, S, 0.0
    if h is None:
        h = net.embed_ids(ctx_ids[S])
    if not inplace:
        for l in range(start, net.L):
            K[l], V[l] = K[l].clone(), V[l].clone()
    if runner is not None and runner.worth_it(K[0].shape[2]):
        h, K[start:], V[start:] = runner.run(h, S, K[start:], V[start:], start)
    else:
        net.run(h, S, K, V, start)
    L, n = net.L, len(all_c)
    eff = (len(S) * (L - start) + start * n) / (n * L)
    return K, V, S, eff


def to_cache(K, V):
    """HF DynamicCache over per-layer views (tread/blend.py:182-186). The layers hold the given
    tensors themselves (no copy of the assembled cache); decoding appends to them as usual.
    With per-layer cache objects (transformers >= 4.56) the layers are built directly, which
    skips update()'s lazy initialisation and concatenation with an empty tensor per layer."""
    c = DynamicCache()
    try:
        from transformers.cache_utils import DynamicLayer
    except ImportError:
        DynamicLayer = None
    if DynamicLayer is not None and isinstance(getattr(c, "layers", None), list):
        for k, v in zip(K, V):
            layer = DynamicLayer()
            layer.dtype, layer.device = k.dtype, k.device
            layer.keys, layer.values = k, v
            layer.is_initialized = True
            c.layers.append(layer)
        return c
    for l, (k, v) in enumerate(zip(K, V)):  # caches without per-layer objects: the copying update
        c.update(k, v, l)
    return c
