"""TEST INFRASTRUCTURE ONLY: a CPU restatement of tread's request path, for the CPU baseline.

bench.py's `ttft.cpu_baseline` times this on the GPU box's host cores (the reference itself is
Python and does not travel to that box); tests/test_engine_port.py pins it against fixtures the
unmodified reference produced (stats, selected positions and first-token logits). The product
never imports it.

It follows the reference step by step on HF transformers' Qwen2 modules, in plain PyTorch on
the CPU, with the reference's arithmetic (rotation through the model's rotary embedding in the
model's dtype, deviation and top-k in the model's dtype, SDPA with a boolean mask):
  - blocks keyed by sha256 over the parts, each followed by NUL (tread/store.py:21-30), the doc
    key chained from the prefix key (tread/engine.py:44-57, 65);
  - a missed doc is prefilled after the prefix at positions P.. (tread/engine.py:59-96; done here
    doc by doc, which the reference's packed block-diagonal pass equals);
  - assembly: prefix K/V, then each doc's K rotated by (offset - base) and its V as is,
    concatenated (tread/engine.py:108-120, tread/blend.py:22-39);
  - recompute (tread/blend.py:133-179): budget = int(round(ratio * n)); "deviation" recomputes
    layer 0 for every candidate, ranks sum_h ||k1 - K1|| + sum_h ||v1 - V1|| and keeps the top
    `budget`; "boundary" water-fills each doc's first tokens; then the kept rows run through the
    remaining layers with their fresh K/V spliced into the cache (blend.py:93-114);
  - the query segment runs over the cache and gives the last position's logits
    (tread/engine.py:131-132).
The block store here is a plain dict (no budget): the baseline times warm requests.
"""
import hashlib
import time

import torch
import torch.nn.functional as F
from transformers import DynamicCache
from transformers.models.qwen2.modeling_qwen2 import apply_rotary_pos_emb, repeat_kv, rotate_half


def block_key(*parts):
    h = hashlib.sha256()
    for p in parts:
        h.update(p.to(torch.int64).numpy().tobytes() if isinstance(p, torch.Tensor) else str(p).encode())
        h.update(b"\x00")
    return h.hexdigest()


def _stack(cache):
    """[L, 1, Hkv, T, D] K and V of an HF DynamicCache."""
    return (torch.stack([lay.keys for lay in cache.layers]), torch.stack([lay.values for lay in cache.layers]))


def _as_cache(K, V):
    c = DynamicCache()
    for l in range(K.shape[0]):
        c.update(K[l], V[l], l)
    return c


class CpuPort:
    def __init__(self, model):
        self.model = model
        cfg = model.config
        self.sig = (cfg._name_or_path, str(model.dtype), getattr(cfg, "rope_theta", None),
                    getattr(cfg, "rope_scaling", None))
        self.blocks = {}  # key -> (K, V, base)
        self.G = cfg.num_attention_heads // cfg.num_key_value_heads
        self.D = getattr(cfg, "head_dim", None) or cfg.hidden_size // cfg.num_attention_heads

    # -- blocks ---------------------------------------------------------------------------------
    def _forward_kv(self, ids, past=None, start=0):
        out = self.model.model(ids[None], past_key_values=past if past is not None else DynamicCache(),
                               position_ids=torch.arange(start, start + len(ids))[None],
                               cache_position=torch.arange(start, start + len(ids)), use_cache=True)
        return _stack(out.past_key_values)

    def keys(self, prefix_ids, docs, namespace=""):
        pkey = block_key(*self.sig, namespace, "prefix", prefix_ids)
        return pkey, [block_key(*self.sig, pkey, d) for d in docs]

    def _lookup(self, prefix_ids, docs, namespace, st):
        pkey, dkeys = self.keys(prefix_ids, docs, namespace)
        if pkey in self.blocks:
            st["hits"] += 1
            st["tokens_reused"] += len(prefix_ids)
        else:
            st["misses"] += 1
            st["tokens_prefilled"] += len(prefix_ids)
            K, V = self._forward_kv(prefix_ids)
            self.blocks[pkey] = (K, V, 0)
        Kp, Vp, _ = self.blocks[pkey]
        P = Kp.shape[-2]
        out = []
        for d, k in zip(docs, dkeys):
            if k in self.blocks:
                st["hits"] += 1
                st["tokens_reused"] += len(d)
            else:
                st["misses"] += 1
                st["tokens_prefilled"] += len(d)
                K, V = self._forward_kv(d, _as_cache(Kp.clone(), Vp.clone()), start=P)
                self.blocks[k] = (K[..., P:, :].contiguous(), V[..., P:, :].contiguous(), P)
            out.append(self.blocks[k])
        return (Kp, Vp), out

    def seed_blocks(self, prefix_ids, docs, gen, namespace=""):
        """Timing only: store random-valued blocks of the right shapes under the request's keys, so
        that warm requests can be timed without a cold pass (their work does not depend on the
        values)."""
        cfg = self.model.config
        pkey, dkeys = self.keys(prefix_ids, docs, namespace)
        shape = lambda n: (cfg.num_hidden_layers, 1, cfg.num_key_value_heads, n, self.D)
        rnd = lambda n: torch.randn(shape(n), generator=gen).to(self.model.dtype)
        P = len(prefix_ids)
        self.blocks[pkey] = (rnd(P), rnd(P), 0)
        for d, k in zip(docs, dkeys):
            self.blocks[k] = (rnd(len(d)), rnd(len(d)), P)

    # -- rotation and recompute -----------------------------------------------------------------
    def _shift(self, K, delta):
        if delta == 0:
            return K
        rot = self.model.model.rotary_emb
        cos, sin = rot(K, torch.full((1, K.shape[-2]), delta, dtype=torch.long))
        s = getattr(rot, "attention_scaling", 1.0)
        cos, sin = cos[0] / s, sin[0] / s
        return K * cos + rotate_half(K) * sin

    def _rows_layer(self, l, h, S, K, V, rope, mask):
        """Layer l over rows h at positions S, their fresh K/V written into K, V (in place)."""
        layer = self.model.model.layers[l]
        a = layer.self_attn
        n, D = h.shape[1], self.D
        x = layer.input_layernorm(h)
        q = a.q_proj(x).view(1, n, -1, D).transpose(1, 2)
        k = a.k_proj(x).view(1, n, -1, D).transpose(1, 2)
        v = a.v_proj(x).view(1, n, -1, D).transpose(1, 2)
        q, k = apply_rotary_pos_emb(q, k, *rope)
        K[:, :, S], V[:, :, S] = k, v
        o = F.scaled_dot_product_attention(q, repeat_kv(K, self.G), repeat_kv(V, self.G), attn_mask=mask)
        h = h + a.o_proj(o.transpose(1, 2).reshape(1, n, -1))
        return h + layer.mlp(layer.post_attention_layernorm(h))

    def _recompute(self, ctx_ids, Kl, Vl, cands, ratio, policy):
        all_c = torch.cat(cands)
        n, T = len(all_c), Kl[0].shape[2]
        budget = int(round(ratio * n))
        if budget == 0:
            return all_c[:0], 0.0
        layers = self.model.model.layers
        rot = self.model.model.rotary_emb
        start = 0
        if policy == "boundary":
            rank = torch.cat([torch.arange(len(c)) for c in cands])
            S = all_c[rank.argsort(stable=True)[:budget]]
        elif policy == "deviation":
            h0 = self.model.model.embed_tokens(ctx_ids[all_c])[None]
            rope = rot(h0, all_c[None])
            mask = (torch.arange(T)[None, :] <= all_c[:, None])[None, None]
            h = self._rows_layer(0, h0, all_c, Kl[0], Vl[0], rope, mask)
            a1 = layers[1].self_attn
            x1 = layers[1].input_layernorm(h)
            k1 = a1.k_proj(x1).view(1, n, -1, self.D).transpose(1, 2)
            v1 = a1.v_proj(x1).view(1, n, -1, self.D).transpose(1, 2)
            q_dummy = torch.zeros_like(k1)
            _, k1 = apply_rotary_pos_emb(q_dummy, k1, *rope)
            dev = ((k1 - Kl[1][:, :, all_c]).norm(dim=-1).sum(dim=1)
                   + (v1 - Vl[1][:, :, all_c]).norm(dim=-1).sum(dim=1))[0]
            top = dev.topk(budget).indices
            S, h, start = all_c[top], h[:, top], 1
        else:
            raise ValueError(policy)
        S, order = S.sort()
        h = self.model.model.embed_tokens(ctx_ids[S])[None] if start == 0 else h[:, order]
        rope = rot(h, S[None])
        mask = (torch.arange(T)[None, :] <= S[:, None])[None, None]
        for l in range(start, len(layers)):
            h = self._rows_layer(l, h, S, Kl[l], Vl[l], rope, mask)
        L = len(layers)
        return S, (len(S) * (L - start) + start * n) / (n * L)

    # -- request --------------------------------------------------------------------------------
    @torch.inference_mode()
    def prefill(self, prefix_ids, docs, query_ids, ratio=0.0, policy="deviation", namespace=""):
        """Returns (last-position logits, stats dict, selected positions S)."""
        st = dict(hits=0, misses=0, tokens_reused=0, tokens_prefilled=0, recompute_eff=0.0)
        t0 = time.perf_counter()
        (Kp, Vp), blocks = self._lookup(prefix_ids, docs, namespace, st)
        Ks, Vs, cands, off = [Kp], [Vp], [], Kp.shape[-2]
        for d, (K, V, base) in zip(docs, blocks):
            Ks.append(self._shift(K, off - base))
            Vs.append(V)
            cands.append(torch.arange(off, off + len(d)))
            off += len(d)
        K, V = torch.cat(Ks, dim=-2), torch.cat(Vs, dim=-2)
        Kl, Vl = list(K.unbind(0)), list(V.unbind(0))
        t1 = time.perf_counter()
        S = torch.empty(0, dtype=torch.long)
        if ratio > 0 and cands:
            S, st["recompute_eff"] = self._recompute(torch.cat([prefix_ids] + list(docs)), Kl, Vl, cands, ratio,
                                                     policy)
        t2 = time.perf_counter()
        out = self.model(query_ids[None], past_key_values=_as_cache(torch.stack(Kl), torch.stack(Vl)), use_cache=True,
                         logits_to_keep=1)
        logits = out.logits[0, -1]
        t3 = time.perf_counter()
        st["t"] = dict(assemble=t1 - t0, blend=t2 - t1, query=t3 - t2, ttft=t3 - t0)
        return logits, st, S


def random_bf16_model(arch, seed=0):
    """A Qwen2 model of architecture `arch` built directly in bf16 on the CPU (no fp32 copy), for
    timing 7B-class architectures on host cores. Timing only: drawing 7.6e9 normal values on the
    host takes minutes, so every Linear weight is filled from one seeded block of 2^24
    N(0, initializer_range) values, repeated; biases 0, norm weights 1, rotary frequencies as HF
    computes them."""
    from transformers import Qwen2ForCausalLM
    from transformers.models.qwen2.modeling_qwen2 import Qwen2RotaryEmbedding

    from tread_b200.configs import qwen2_config

    cfg = qwen2_config(arch)
    prev = torch.get_default_dtype()
    torch.set_default_dtype(torch.bfloat16)
    try:
        with torch.device("meta"):
            model = Qwen2ForCausalLM(cfg)
        model = model.to_empty(device="cpu")
    finally:
        torch.set_default_dtype(prev)
    g = torch.Generator().manual_seed(seed)
    src = (torch.randn(1 << 24, generator=g) * cfg.initializer_range).to(torch.bfloat16)
    with torch.no_grad():
        for name, p in model.named_parameters():
            if p.dim() >= 2:
                flat = p.view(-1)
                for i in range(0, flat.numel(), src.numel()):
                    n = min(src.numel(), flat.numel() - i)
                    flat[i:i + n].copy_(src[:n])
            elif name.endswith("bias"):
                p.zero_()
            else:
                p.fill_(1.0)
    model.model.rotary_emb = Qwen2RotaryEmbedding(config=cfg)
    return model.eval()
