"""Qwen2 decoder math over token rows at arbitrary positions, on tread_b200 kernels.

The reference drives HF's Qwen2 modules directly (tread/blend.py:82-114, tread/engine.py:86-88,
131-132). This module owns the same layer arithmetic (weights taken from the HF module) so
that every path the hot path needs is one primitive: a set of token rows, each at its own
absolute position, runs through layers [l0, l1) against per-layer KV caches, with

    x = RMSNorm(h) (tread_rmsnorm);  qkv = x @ Wqkv^T + b  (one GEMM)
    RoPE(q, k at pos) ; K[pos], V[pos] = k, v              (tread_rope_rows)
    o = attention(q, K, V, key_pos <= pos)                 (tread_attn_rows)
    h = h + o @ Wo^T ; h = h + down(silu(gate) * up)       (GEMMs; tread_silu_mul)

GEMMs of up to 128 rows (the query segment alone) against the widest weights (gate/up, lm_head)
stream those weights through tread_rows_gemm on the tensor cores; the rest run as cuBLAS GEMMs.

Rows are: recomputed tokens (blend), the query segment, a prefix or a doc being prefilled.
A row only ever sees keys at positions <= its own, which is the causal mask of a prefill, the
subset mask of tread/blend.py:76, and the query's causal attention over the assembled cache.
"""
import torch
import torch.nn.functional as F

from tread_b200 import kernels


class Qwen2Rows:
    def __init__(self, model):
        cfg = model.config
        self.model = model
        self.config = cfg
        self.L = cfg.num_hidden_layers
        self.hidden = cfg.hidden_size
        self.Hq = cfg.num_attention_heads
        self.Hkv = cfg.num_key_value_heads
        self.D = getattr(cfg, "head_dim", None) or cfg.hidden_size // cfg.num_attention_heads
        self.eps = cfg.rms_norm_eps
        self.dtype = model.dtype
        self.device = model.device
        rot = model.model.rotary_emb
        self.inv_freq = rot.inv_freq.float().cpu().tolist()
        self.attn_scaling = float(getattr(rot, "attention_scaling", 1.0))
        if getattr(rot, "rope_type", "default") not in ("default", "linear", "llama3"):
            # position-dependent frequency schemes (dynamic NTK) would need a per-request inv_freq
            raise NotImplementedError(f"rope_type {rot.rope_type} is not supported")
        self.embed = model.model.embed_tokens.weight
        self.norm_w = model.model.norm.weight
        self.norm_eps = model.model.norm.variance_epsilon
        self.lm_head = model.lm_head.weight
        self.layers = []
        with torch.no_grad():
            for layer in model.model.layers:
                a, m = layer.self_attn, layer.mlp
                wqkv = torch.cat([a.q_proj.weight, a.k_proj.weight, a.v_proj.weight], 0).contiguous()
                bqkv = torch.cat([a.q_proj.bias, a.k_proj.bias, a.v_proj.bias], 0).contiguous()
                wgu = torch.cat([m.gate_proj.weight, m.up_proj.weight], 0).contiguous()
                # The HF modules keep working on views of the packed tensors, so the packing costs
                # no extra HBM (values are unchanged).
                nq, nk = a.q_proj.weight.shape[0], a.k_proj.weight.shape[0]
                a.q_proj.weight.data, a.k_proj.weight.data, a.v_proj.weight.data = (
                    wqkv[:nq], wqkv[nq:nq + nk], wqkv[nq + nk:])
                a.q_proj.bias.data, a.k_proj.bias.data, a.v_proj.bias.data = (
                    bqkv[:nq], bqkv[nq:nq + nk], bqkv[nq + nk:])
                inter = m.gate_proj.weight.shape[0]
                m.gate_proj.weight.data, m.up_proj.weight.data = wgu[:inter], wgu[inter:]
                self.layers.append(dict(
                    ln1=layer.input_layernorm.weight,
                    ln1_eps=layer.input_layernorm.variance_epsilon,
                    wqkv=wqkv, bqkv=bqkv, wo=a.o_proj.weight,
                    ln2=layer.post_attention_layernorm.weight,
                    ln2_eps=layer.post_attention_layernorm.variance_epsilon,
                    wgu=wgu, wd=m.down_proj.weight, inter=inter,
                ))
        self.err = torch.zeros(4, dtype=torch.int32, device=self.device)
        if self.device.type == "cuda":
            kernels.rows_gemm_workspace(self.device)  # before any graph capture holds its address

    # -- elementwise pieces (HF Qwen2RMSNorm / SwiGLU semantics, fused kernels) ------------------
    @staticmethod
    def rmsnorm(x, w, eps):
        return kernels.rmsnorm(x, w, eps)

    def embed_ids(self, ids):
        return F.embedding(ids, self.embed)

    @staticmethod
    def linear(x, w, bias=None, out=None, accumulate=False, err=None):
        """x @ w^T (+ bias), or out + x @ w^T in place when `accumulate`, rounded once (HF Linear /
        torch.addmm). Up to 128 rows against a weight wide enough to fill every SM without a K
        split (the gate/up projection, the lm_head): tread_rows_gemm, weights streamed on the
        tensor cores; everything else: cuBLAS. `err`: the device error word in which a bounded
        wait of the tensor-core kernel that gave up sets bit 2."""
        if kernels.rows_gemm_fits(x, w) and kernels.rows_gemm_streams_alone(w):
            return kernels.rows_gemm(x, w, bias=bias, out=out, accumulate=accumulate, err=err)
        if accumulate:
            if bias is not None:
                raise ValueError("linear: accumulate takes no bias")
            return out.addmm_(x, w.t())
        y = x @ w.t() if bias is None else torch.addmm(bias, x, w.t())
        if out is not None:
            out.copy_(y)
            return out
        return y

    # -- one layer over rows ----------------------------------------------------------------------
    def qkv(self, l, h):
        p = self.layers[l]
        return self.linear(self.rmsnorm(h, p["ln1"], p["ln1_eps"]), p["wqkv"], bias=p["bqkv"], err=self.err)

    def kv(self, l, h):
        """Only the k and v columns of layer l's projection, [R, 2 * Hkv * D]: the deviation
        selector's fresh layer-1 rows (tread/blend.py:127-128) need no queries, so their GEMM
        skips the Hq * D query columns."""
        p = self.layers[l]
        nq = self.Hq * self.D
        return self.linear(self.rmsnorm(h, p["ln1"], p["ln1_eps"]), p["wqkv"][nq:], bias=p["bqkv"][nq:],
                           err=self.err)

    def layer(self, l, h, pos, K, V, qkv=None):
        """h: [R, hidden] rows at positions pos (int64 [R]); K, V: layer-l caches [1, Hkv, T, D]
        (or [Hkv, T, D]); the rows' k/v are written into them. Returns the new residual rows
        (for this class: h itself, updated in place)."""
        return self.layer_segments(l, h, [(0, h.shape[0], pos, K, V)], qkv)

    def layer_segments(self, l, h, segs, qkv=None):
        """One layer over rows that belong to independent caches: segs = [(r0, r1, pos, K, V)],
        rows r0..r1-1 of h sit at positions pos and read/write cache K, V. The projections and the
        MLP run once over all rows; RoPE + splice and attention run per segment."""
        R = h.shape[0]
        if qkv is None:
            qkv = self.qkv(l, h)
        q = torch.empty(R, self.Hq, self.D, dtype=h.dtype, device=h.device)
        o = torch.empty_like(q)
        for r0, r1, pos, K, V in segs:
            kernels.rope_rows(qkv[r0:r1], pos, self.Hq, self.Hkv, self.D, q[r0:r1], K, V, self.inv_freq,
                              self.attn_scaling, self.err)
            kernels.attn_rows(q[r0:r1], K, V, pos, out=o[r0:r1], err=self.err)
        return self.layer_tail(l, h, o.view(R, -1))

    def layer_tail(self, l, h, o):
        """h + o_proj(o), then h + down(silu(gate) * up) of its RMSNorm (residuals in place)."""
        p = self.layers[l]
        self.linear(o, p["wo"], out=h, accumulate=True, err=self.err)
        x = self.rmsnorm(h, p["ln2"], p["ln2_eps"])
        a = kernels.silu_mul(self.linear(x, p["wgu"], err=self.err))
        return self.linear(a, p["wd"], out=h, accumulate=True, err=self.err)

    def run(self, h, pos, Ks, Vs, l0=0, l1=None):
        """Rows h through layers [l0, l1); returns the final hidden rows (h itself is not modified)."""
        h = h.clone()
        for l in range(l0, self.L if l1 is None else l1):
            h = self.layer(l, h, pos, Ks[l], Vs[l])
        return h

    def logits(self, h_last):
        """Final RMSNorm + lm_head of the given rows (HF Qwen2Model.norm, Qwen2ForCausalLM.lm_head)."""
        x = self.rmsnorm(h_last, self.norm_w, self.norm_eps)
        return self.linear(x, self.lm_head, err=self.err)

    def deviation_select(self, k1, v1, K1, V1, cand_pos, budget):
        """Layer-1 deviation of the candidates and the top-`budget` selection (dev, sel_idx, S);
        the KV-head tensor-parallel rows override this with the split selector."""
        return kernels.deviation_topk(k1, v1, K1, V1, cand_pos, budget)

    def new_cache(self, T):
        """Zeroed per-request KV cache [L, 1, Hkv, T, D] for K and for V."""
        shape = (self.L, 1, self.Hkv, T, self.D)
        return (torch.zeros(shape, dtype=self.dtype, device=self.device),
                torch.zeros(shape, dtype=self.dtype, device=self.device))

    def check_errors(self):
        """Raise if a kernel flagged an out-of-range row position: the row kernels' error word and
        the selector's sticky flag, read with one device sync."""
        sel = kernels.selector_flags(self.device)
        e = int(torch.cat([self.err, sel]).max().item())
        if e:
            self.err.zero_()
            sel.zero_()
            if e & 4:  # an attention kernel gave up on a wait: its split-tile counters may be stale
                kernels.reset_attn_workspace(self.device)
            raise RuntimeError(f"tread_b200 kernel reported an error (flags {e:#x}: 1, 2 out-of-range position, "
                               f"4 wait timeout)")
