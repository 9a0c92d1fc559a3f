"""KV-head tensor parallelism of the chunk-reuse path, for Qwen2 models split over the GPUs of one node.

The reference is single-GPU (tread/engine.py, tread/blend.py). Here rank r of W owns the KV
heads [r*Hkv/W, (r+1)*Hkv/W) and the G = Hq/Hkv query heads that read each of them, so the whole
KV side of the path -- blocks in the store, rotate/gather/append, the layer-1 deviation, the
recompute attention -- runs on the rank's own heads with no exchange. Per recomputed layer:

    x    = RMSNorm(h)                           replicated rows
    qkv  = x @ Wqkv_r^T + b_r                   column slice: this rank's q, k, v heads
    RoPE + splice into this rank's cache slice; attention over its heads
    h'   = h + sum_r o_r @ Wo[:, cols_r]^T      row slice + NCCL all-reduce (rank 0 adds h)
    h''  = h' + sum_r silu(g_r) u_r @ Wd[:, cols_r]^T   (gate/up column slice, down row slice)

so the only collectives are the two all-reduces of [rows, hidden] per layer, plus one all-gather
of the per-head layer-1 norms ([2, Hkv/W, n] fp32 per rank) before the selection: every rank
sums all heads' norms in global head order and runs the same top-k, so every rank selects the
same tokens as a single GPU holding all heads would from the same norms.

Each rank runs the same Engine on the same requests with its own BlockStore holding its head
slice of every block ([L, 1, Hkv/W, n, D]); block keys, hits and evictions therefore agree
across ranks (give every rank the same budget fraction). Embedding, final norm and lm_head are
replicated, so every rank ends with the same first-token logits.
"""
import torch
import torch.distributed as dist

from tread_b200 import kernels
from tread_b200.qwen2 import Qwen2Rows


def kv_head_range(Hkv, rank, world):
    """KV heads [h0, h1) owned by `rank`."""
    if Hkv % world:
        raise ValueError(f"{Hkv} KV heads do not split over {world} ranks")
    n = Hkv // world
    return rank * n, (rank + 1) * n


def shard_layer(w, Hq, Hkv, D, rank, world):
    """This rank's slice of one decoder layer.

    w: full weights {ln1, ln1_eps, wq, bq, wk, bk, wv, bv, wo, ln2, ln2_eps, wg, wu, wd} in the
    HF layout (out_features x in_features). Returns the layer dict Qwen2Rows.layer reads, with the
    q/k/v rows of this rank's heads packed as [q heads | k heads | v heads], Wo's matching input
    columns, and the rank's contiguous slice of the MLP's intermediate dimension."""
    h0, h1 = kv_head_range(Hkv, rank, world)
    G = Hq // Hkv
    q0, q1, k0, k1 = h0 * G * D, h1 * G * D, h0 * D, h1 * D
    inter = w["wg"].shape[0]
    if inter % world:
        raise ValueError(f"MLP width {inter} does not split over {world} ranks")
    i0, i1 = inter * rank // world, inter * (rank + 1) // world
    return dict(
        ln1=w["ln1"], ln1_eps=w["ln1_eps"],
        wqkv=torch.cat([w["wq"][q0:q1], w["wk"][k0:k1], w["wv"][k0:k1]]).contiguous(),
        bqkv=torch.cat([w["bq"][q0:q1], w["bk"][k0:k1], w["bv"][k0:k1]]).contiguous(),
        wo=w["wo"][:, q0:q1].contiguous(),
        ln2=w["ln2"], ln2_eps=w["ln2_eps"],
        wgu=torch.cat([w["wg"][i0:i1], w["wu"][i0:i1]]).contiguous(),
        wd=w["wd"][:, i0:i1].contiguous(),
        inter=i1 - i0,
    )


def _hf_layer(layer):
    a, m = layer.self_attn, layer.mlp
    return dict(ln1=layer.input_layernorm.weight, ln1_eps=layer.input_layernorm.variance_epsilon,
                wq=a.q_proj.weight, bq=a.q_proj.bias, wk=a.k_proj.weight, bk=a.k_proj.bias,
                wv=a.v_proj.weight, bv=a.v_proj.bias, wo=a.o_proj.weight,
                ln2=layer.post_attention_layernorm.weight,
                ln2_eps=layer.post_attention_layernorm.variance_epsilon,
                wg=m.gate_proj.weight, wu=m.up_proj.weight, wd=m.down_proj.weight)


def _normal(shape, seed, device, dtype, std):
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return (torch.randn(shape, generator=g, device=device, dtype=torch.float32) * std).to(dtype)


def _random_layers(cfg, seed, device, dtype):
    """Full per-layer weights drawn like HF's Qwen2 init (Linear weights N(0, initializer_range),
    biases 0, RMSNorm weights 1), one layer at a time from per-tensor seeds, so every rank and
    every world size sees the same model."""
    hid = cfg.hidden_size
    D = getattr(cfg, "head_dim", None) or cfg.hidden_size // cfg.num_attention_heads
    nq, nkv, inter = cfg.num_attention_heads * D, cfg.num_key_value_heads * D, cfg.intermediate_size
    std, eps = cfg.initializer_range, cfg.rms_norm_eps
    ones = torch.ones(hid, dtype=dtype, device=device)
    for l in range(cfg.num_hidden_layers):
        s = seed * 1_000_003 + l * 16
        yield dict(ln1=ones, ln1_eps=eps, ln2=ones, ln2_eps=eps,
                   wq=_normal((nq, hid), s + 1, device, dtype, std), bq=torch.zeros(nq, dtype=dtype, device=device),
                   wk=_normal((nkv, hid), s + 2, device, dtype, std), bk=torch.zeros(nkv, dtype=dtype, device=device),
                   wv=_normal((nkv, hid), s + 3, device, dtype, std), bv=torch.zeros(nkv, dtype=dtype, device=device),
                   wo=_normal((hid, nq), s + 4, device, dtype, std),
                   wg=_normal((inter, hid), s + 5, device, dtype, std),
                   wu=_normal((inter, hid), s + 6, device, dtype, std),
                   wd=_normal((hid, inter), s + 7, device, dtype, std))


def gather_head_norms(norms, group=None):
    """All ranks' per-head norms [2, Hkv/W, n] -> every head's [2, Hkv, n] in global head order."""
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    if world == 1:
        return norms
    parts = [torch.empty_like(norms) for _ in range(world)]
    dist.all_gather(parts, norms.contiguous(), group=group)
    return torch.cat(parts, dim=1)


class TPQwen2Rows(Qwen2Rows):
    """Qwen2Rows over this rank's KV-head slice: Hq and Hkv are the rank's own head counts, every
    cache and block it touches is [.., Hkv/W, T, D], and `layer` / `deviation_select` add the
    collectives. Build with `from_model` (slices an HF model's weights) or `random` (seeded
    random-init weights of a config, generated layer by layer on the device)."""

    def __init__(self, cfg, layers, embed, norm_w, norm_eps, lm_head, group=None, dtype=None, device=None,
                 rotary=None):
        """rotary: the model's rotary-embedding module (its inv_freq buffer as the model holds it:
        a model cast to bf16 carries bf16-rounded frequencies, and its own RoPE uses those);
        default: a fresh fp32 one from `cfg`, as a model loaded in its dtype has."""
        from transformers.models.qwen2.modeling_qwen2 import Qwen2RotaryEmbedding

        self.model = None
        self.config = cfg
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.L = cfg.num_hidden_layers
        self.hidden = cfg.hidden_size
        self.D = getattr(cfg, "head_dim", None) or cfg.hidden_size // cfg.num_attention_heads
        self.Hq_total, self.Hkv_total = cfg.num_attention_heads, cfg.num_key_value_heads
        h0, h1 = kv_head_range(self.Hkv_total, self.rank, self.world)
        self.kv_heads = (h0, h1)
        self.Hkv = h1 - h0
        self.Hq = self.Hkv * (self.Hq_total // self.Hkv_total)
        self.eps = cfg.rms_norm_eps
        self.dtype = dtype or embed.dtype
        self.device = device or embed.device
        rot = rotary if rotary is not None else Qwen2RotaryEmbedding(config=cfg)
        if getattr(rot, "rope_type", "default") not in ("default", "linear", "llama3"):
            raise NotImplementedError(f"rope_type {rot.rope_type} is not supported")
        self.inv_freq = rot.inv_freq.float().cpu().tolist()
        self.attn_scaling = float(getattr(rot, "attention_scaling", 1.0))
        self.embed, self.norm_w, self.norm_eps, self.lm_head = embed, norm_w, norm_eps, lm_head
        self.layers = [shard_layer(w, self.Hq_total, self.Hkv_total, self.D, self.rank, self.world) for w in layers]
        self.err = torch.zeros(4, dtype=torch.int32, device=self.device)
        if self.device.type == "cuda":
            kernels.rows_gemm_workspace(self.device)  # before any graph capture holds its address

    @classmethod
    def from_model(cls, model, group=None):
        """This rank's slice of an HF Qwen2ForCausalLM (weights copied; the model may be freed)."""
        with torch.no_grad():
            return cls(model.config, (_hf_layer(layer) for layer in model.model.layers),
                       model.model.embed_tokens.weight, model.model.norm.weight, model.model.norm.variance_epsilon,
                       model.lm_head.weight, group, model.dtype, model.device, model.model.rotary_emb)

    @classmethod
    def random(cls, cfg, group=None, seed=0, dtype=torch.bfloat16, device="cuda"):
        """Seeded random-init weights of `cfg`; identical on every rank and for every world size."""
        device = torch.device(device)
        with torch.no_grad():
            base = seed * 1_000_003 + cfg.num_hidden_layers * 16
            embed = _normal((cfg.vocab_size, cfg.hidden_size), base + 1, device, dtype, cfg.initializer_range)
            lm_head = embed if cfg.tie_word_embeddings else _normal(
                (cfg.vocab_size, cfg.hidden_size), base + 2, device, dtype, cfg.initializer_range)
            norm_w = torch.ones(cfg.hidden_size, dtype=dtype, device=device)
            return cls(cfg, _random_layers(cfg, seed, device, dtype), embed, norm_w, cfg.rms_norm_eps, lm_head,
                       group, dtype, device)

    # -- collective timing (off unless a caller sets `collective_events` to a list) ---------------
    collective_events = None

    def _timed(self, name, fn):
        """Run the collective `fn`; with collective timing on, bracket it with CUDA events on the
        current stream (its device time on this rank, waiting for the peers included)."""
        if self.collective_events is None:
            return fn()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        out = fn()
        b.record()
        self.collective_events.append((name, a, b))
        return out

    def collective_ms(self):
        """Milliseconds per collective kind since collective timing was switched on (synchronises)."""
        torch.cuda.synchronize(self.device)
        tot = {}
        for name, a, b in self.collective_events or ():
            tot[name] = tot.get(name, 0.0) + a.elapsed_time(b)
        return tot

    def _row_parallel(self, a, w, h, name):
        """h + sum over ranks of a_r @ w_r^T (rank 0 folds the residual into its product)."""
        out = (self.linear(a, w, out=h.clone(), accumulate=True, err=self.err) if self.rank == 0
               else self.linear(a, w, err=self.err))
        if self.world > 1:
            self._timed(name, lambda: dist.all_reduce(out, group=self.group))
        return out

    def layer_tail(self, l, h, o):
        """Row-parallel o_proj and down_proj with their all-reduces; returns the new residual rows
        (a new tensor, identical on every rank)."""
        p = self.layers[l]
        h = self._row_parallel(o, p["wo"], h, "o_proj_allreduce")
        x = self.rmsnorm(h, p["ln2"], p["ln2_eps"])
        a = kernels.silu_mul(self.linear(x, p["wgu"], err=self.err))
        return self._row_parallel(a, p["wd"], h, "down_proj_allreduce")

    def deviation_select(self, k1, v1, K1, V1, cand_pos, budget):
        """Per-head norms of this rank's heads, all-gathered, then the fixed-order head sum and
        the top-`budget` selection on every rank (same result everywhere)."""
        norms = kernels.deviation_head_norms(k1, v1, K1, V1, cand_pos)
        allnorms = self._timed("head_norms_allgather", lambda: gather_head_norms(norms, self.group))
        return kernels.select_head_norms(allnorms, cand_pos, budget)

    def check_errors(self):
        """Raise on every rank if a kernel on any rank flagged an error (row kernels' error word
        or the selector's out-of-range flag), with one all-reduce."""
        sel = kernels.selector_flags(self.device)
        e = torch.cat([self.err, sel]).max()
        if self.world > 1:
            dist.all_reduce(e, op=dist.ReduceOp.MAX, group=self.group)
        if int(e.item()):
            self.err.zero_()
            sel.zero_()
            if int(e.item()) & 4:
                kernels.reset_attn_workspace(self.device)
            raise RuntimeError(f"tread_b200 kernel reported an error on some rank (flags {int(e):#x})")
