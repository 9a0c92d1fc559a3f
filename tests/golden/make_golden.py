"""Generate the golden fixtures in tests/golden/ by running the UNMODIFIED tread reference.

Run where the reference sources are checked out, naming their root (the directory that holds
the `tread` package) with --reference or the TREAD_REFERENCE_ROOT environment variable:

    python tests/golden/make_golden.py --reference <root> [fixture ...]

The reference is imported through oracle/ref_shim.py (transformers 5.x attribute renames
only). Models are seeded random-init Qwen2 architectures (tread_b200/configs.py): the HF
checkpoints the reference tests use are not available offline. Token ids are seeded uniform
draws standing in for the reference's HotpotQA workload.

Fixtures:
  rope.npz      rotate_keys (tread/blend.py:22-39) in fp32 for D=64/128 and shifts up to 16384,
                plus HF rotary_emb cos/sin for each shift.
  deviation.npz layer1_deviation inputs/outputs and the deviation top-k selection
                (tread/blend.py:117-130,145,158-169) on the tiny architecture.
  attention.npz _layer_subset's masked GQA attention (tread/blend.py:106-110) on random q/K/V.
  store.npz     StoreStats and tier contents after each op of a seeded get/put trace against
                tread.store.BlockStore (tread/store.py:56-125).
  engine_tiny.npz, engine_cfg1.npz
                Engine.prefill (tread/engine.py:98-136) cold then reordered requests, ratios 0 /
                0.2 deviation / 1.0 boundary: stats, selected positions, first-token logits, and
                prefill_full logits (the KL reference).
  engine_bf16_tiny.npz, engine_bf16_7b3l.npz
                the same requests on bf16 models (the tiny architecture, and the configs[2]
                Qwen2.5-7B architecture cut to 3 layers with the full 256 + 16 x 496 + 64 request),
                ratios 0 / 0.2 / 0.5 deviation / 1.0 boundary, with the reference's own bf16
                deviation values; the tiny fixture also holds the reference's layer-1 k1, v1 and
                gathered K1, V1 of the 0.2 request (bf16 bits) for the selection-convention gate.
  server.npz    the reference's HTTP app on its own engine (tiny fp32 model, character-level stub
                tokenizer): each response's text, finish reason, usage and reuse stats, and
                /metrics after the sequence.
  store_engine_bf16.npz
                a sequence of requests on the bf16 tiny model through a store whose GPU tier holds
                about two doc blocks and whose pinned tier holds three: all eight StoreStats
                counters, both tiers' key order and the first-token logits after every request.
"""
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import ref_shim  # noqa: E402
from tread_b200.configs import random_model, random_tokens  # noqa: E402

ROPE_DELTAS = [0, 1, -1, 37, -37, 511, 4096, -4096, 16383, 16384, -16384]


def bf16_bits(t):
    return t.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)


def make_rope(tread):
    from tread.blend import rotate_keys

    out = {}
    for D, arch_kw in ((64, dict(arch="tiny")), (128, dict(arch="tiny"))):
        if D == 128:
            from transformers import Qwen2Config, Qwen2ForCausalLM

            cfg = Qwen2Config(vocab_size=64, hidden_size=512, intermediate_size=64, num_hidden_layers=1,
                              num_attention_heads=4, num_key_value_heads=2, rope_theta=1e6,
                              max_position_embeddings=32768)
            torch.manual_seed(0)
            model = Qwen2ForCausalLM(cfg).eval()
        else:
            model = random_model(**arch_kw, layers=1)
        g = torch.Generator().manual_seed(100 + D)
        K = torch.randn(2, 1, 2, 21, D, generator=g)
        Kb = K.to(torch.bfloat16)
        out[f"d{D}_k_bf16"] = bf16_bits(Kb)
        Kf = Kb.float()
        out[f"d{D}_inv_freq"] = model.model.rotary_emb.inv_freq.float().numpy()
        for d in ROPE_DELTAS:
            with torch.no_grad():
                r = rotate_keys(model, Kf, d)
                cos, sin = model.model.rotary_emb(Kf, torch.full((1, 1), d, dtype=torch.long))
            out[f"d{D}_rot_{d}"] = r.numpy().astype(np.float32)
            out[f"d{D}_cos_{d}"] = cos[0, 0].numpy()
            out[f"d{D}_sin_{d}"] = sin[0, 0].numpy()
    out["deltas"] = np.array(ROPE_DELTAS, np.int64)
    np.savez_compressed(os.path.join(HERE, "rope.npz"), **out)


def tiny_request(vocab, seed=0, n_prefix=16, doc_lens=(40, 33, 47), n_query=8):
    g = torch.Generator().manual_seed(seed)
    prefix = random_tokens(n_prefix, vocab, g)
    docs = [random_tokens(n, vocab, g) for n in doc_lens]
    query = random_tokens(n_query, vocab, g)
    return prefix, docs, query


def make_deviation(tread):
    import tread.blend as tb
    from tread.engine import Engine
    from tread.store import BlockStore

    model = random_model("tiny")
    prefix, docs, query = tiny_request(model.config.vocab_size)
    cap = {}
    orig = tb.layer1_deviation

    def spy(model_, ctx_ids, K, V, all_c, inplace=False):
        K1 = K[1][:, :, all_c].clone()
        V1 = V[1][:, :, all_c].clone()
        dev, h, K0, V0 = orig(model_, ctx_ids, K, V, all_c, inplace=inplace)
        # recompute k1/v1 exactly as layer1_deviation does, for the kernel-level fixture
        layers = model_.model.layers
        _, k1, v1 = tb._qkv(layers[1], model_, layers[1].input_layernorm(h), all_c,
                            tb._subset_ctx(model_, all_c, K[0].shape[2], h)[0])
        cap.update(dev=dev.clone(), all_c=all_c.clone(), k1=k1.clone(), v1=v1.clone(), K1=K1, V1=V1)
        return dev, h, K0, V0

    tb.layer1_deviation = spy
    orig_blend = tb.blend

    def blend_spy(*a, **kw):
        K, V, S, eff = orig_blend(*a, **kw)
        cap.update(S=S.clone(), eff=eff)
        return K, V, S, eff

    import tread.engine as te
    te.blend = blend_spy
    try:
        eng = Engine(model, BlockStore(1 << 30))
        with torch.inference_mode():
            eng.prefill(prefix, docs, query)
            order = [docs[2], docs[0], docs[1]]
            eng.prefill(prefix, order, query, ratio=0.2, policy="deviation")
    finally:
        tb.layer1_deviation = orig
        te.blend = orig_blend
    n = len(cap["all_c"])
    budget = int(round(0.2 * n))
    np.savez_compressed(
        os.path.join(HERE, "deviation.npz"),
        k1=cap["k1"][0].numpy(), v1=cap["v1"][0].numpy(), K1=cap["K1"][0].numpy(), V1=cap["V1"][0].numpy(),
        dev=cap["dev"].numpy(), all_c=cap["all_c"].numpy(), S=cap["S"].numpy(), budget=np.int64(budget),
        topk=cap["dev"].topk(budget).indices.numpy(), eff=np.float64(cap["eff"]))


def make_attention(tread):
    import torch.nn.functional as F
    from transformers.models.qwen2.modeling_qwen2 import repeat_kv

    out = {}
    for name, (Hq, Hkv, D, T, nq) in {"a": (4, 2, 64, 160, 24), "b": (7, 1, 128, 150, 17)}.items():
        g = torch.Generator().manual_seed(7 + D)
        q = torch.randn(1, Hq, nq, D, generator=g)
        K = torch.randn(1, Hkv, T, D, generator=g)
        V = torch.randn(1, Hkv, T, D, generator=g)
        S = torch.sort(torch.randperm(T, generator=g)[:nq]).values
        # the mask and call of tread/blend.py:76,110
        mask = (torch.arange(T)[None, :] <= S[:, None])[None, None]
        o = F.scaled_dot_product_attention(q, repeat_kv(K, Hq // Hkv), repeat_kv(V, Hq // Hkv), attn_mask=mask)
        out.update({f"{name}_q": q[0].numpy(), f"{name}_K": K[0].numpy(), f"{name}_V": V[0].numpy(),
                    f"{name}_S": S.numpy(), f"{name}_o": o[0].numpy()})
    np.savez_compressed(os.path.join(HERE, "attention.npz"), **out)


def make_store(tread):
    from tread.store import BlockStore

    # The trace runs on CPU tensors: pin_memory (tread/store.py:111) needs a CUDA driver and does
    # not influence any decision, so it is an identity here.
    torch.Tensor.pin_memory = lambda self, *a, **k: self
    rng = np.random.default_rng(5)
    unit = 1024
    store = BlockStore(6 * unit, cpu_budget_bytes=5 * unit)
    ops, stats, gpu_keys, cpu_keys, results = [], [], [], [], []
    keys = [f"k{i}" for i in range(12)]
    for step in range(400):
        key = keys[int(rng.integers(len(keys)))]
        if rng.random() < 0.45:
            size = int(rng.integers(1, 5))  # K+V bytes = 2 * size * 128 floats * 4 B = size * unit
            K = torch.zeros(size, 128)
            V = torch.zeros(size, 128)
            if rng.random() < 0.03:
                K = torch.zeros(7, 128)  # larger than the GPU budget -> put returns None
                V = torch.zeros(7, 128)
                size = 7
            b = store.put(key, K, V, int(rng.integers(0, 64)))
            ops.append(("put", key, size))
            results.append(-1 if b is None else b.nbytes)
        else:
            b = store.get(key)
            ops.append(("get", key, 0))
            results.append(-1 if b is None else b.hits)
        s = store.stats
        stats.append([s.hits, s.misses, s.evictions, s.bytes_used, s.cpu_hits, s.offloads, s.cpu_evictions,
                      s.cpu_bytes_used])
        gpu_keys.append(",".join(store.blocks.keys()))
        cpu_keys.append(",".join(store.cpu_blocks.keys()))
    np.savez_compressed(
        os.path.join(HERE, "store.npz"), op=np.array([o[0] for o in ops]), key=np.array([o[1] for o in ops]),
        size=np.array([o[2] for o in ops], np.int64), unit=np.int64(unit), budget=np.int64(6 * unit),
        cpu_budget=np.int64(5 * unit), result=np.array(results, np.int64), stats=np.array(stats, np.int64),
        gpu_keys=np.array(gpu_keys), cpu_keys=np.array(cpu_keys))


RATIOS = (("r0", 0.0, "deviation"), ("r02", 0.2, "deviation"), ("b10", 1.0, "boundary"))
RATIOS_BF16 = (("r0", 0.0, "deviation"), ("r02", 0.2, "deviation"), ("r05", 0.5, "deviation"),
               ("b10", 1.0, "boundary"))


def logits_out(logits):
    """fp32 logits as they are; a bf16 model's logits as their exact bf16 bits."""
    if logits.dtype == torch.bfloat16:
        return bf16_bits(logits)
    return logits.float().numpy()


def run_engine(model, prefix, docs, query, reorder, ratios=RATIOS, layer1_tag=None):
    import tread.blend as tb
    import tread.engine as te
    from tread.engine import Engine, prefill_full
    from tread.store import BlockStore

    cap = {}
    orig_blend = te.blend
    orig_dev = tb.layer1_deviation

    def blend_spy(*a, **kw):
        K, V, S, eff = orig_blend(*a, **kw)
        cap["S"] = S.clone()
        return K, V, S, eff

    def dev_spy(model_, ctx_ids, K, V, all_c, inplace=False):
        K1 = K[1][:, :, all_c].clone()
        V1 = V[1][:, :, all_c].clone()
        dev, h, K0, V0 = orig_dev(model_, ctx_ids, K, V, all_c, inplace=inplace)
        cap["dev"] = dev.clone()
        if cap.get("want_layer1"):
            # k1/v1 exactly as layer1_deviation forms them (tread/blend.py:127-128)
            layers = model_.model.layers
            _, k1, v1 = tb._qkv(layers[1], model_, layers[1].input_layernorm(h), all_c,
                                tb._subset_ctx(model_, all_c, K[0].shape[2], h)[0])
            cap.update(k1=k1[0].clone(), v1=v1[0].clone(), K1=K1[0], V1=V1[0], all_c=all_c.clone())
        return dev, h, K0, V0

    te.blend = blend_spy
    tb.layer1_deviation = dev_spy
    out = {}
    try:
        with torch.inference_mode():
            eng = Engine(model, BlockStore(1 << 34))
            _, _, st1 = eng.prefill(prefix, docs, query)
            order = [docs[i] for i in reorder]
            out["stats_cold"] = np.array([st1.hits, st1.misses, st1.tokens_reused, st1.tokens_prefilled], np.int64)
            for tag, ratio, policy in ratios:
                cap.pop("S", None)
                cap.pop("dev", None)
                cap["want_layer1"] = tag == layer1_tag
                logits, _, st = eng.prefill(prefix, order, query, ratio=ratio, policy=policy)
                out[f"logits_{tag}"] = logits_out(logits)
                if "dev" in cap:
                    out[f"dev_{tag}"] = cap["dev"].float().numpy()
                if tag == layer1_tag:
                    for k in ("k1", "v1", "K1", "V1"):
                        out[f"l1_{k}"] = bf16_bits(cap[k])
                    out["l1_all_c"] = cap["all_c"].numpy()
                out[f"stats_{tag}"] = np.array([st.hits, st.misses, st.tokens_reused, st.tokens_prefilled],
                                               np.int64)
                out[f"eff_{tag}"] = np.float64(st.recompute_eff)
                if "S" in cap:
                    out[f"S_{tag}"] = cap["S"].numpy()
            ref, _, _ = prefill_full(model, prefix, order, query)
            out["logits_full"] = logits_out(ref)
            s = eng.store.stats
            out["store_stats"] = np.array([s.hits, s.misses, s.evictions, s.bytes_used, s.cpu_hits, s.offloads,
                                           s.cpu_evictions, s.cpu_bytes_used], np.int64)
    finally:
        te.blend = orig_blend
        tb.layer1_deviation = orig_dev
    out.update(prefix=prefix.numpy(), query=query.numpy(), reorder=np.array(reorder, np.int64))
    for i, d in enumerate(docs):
        out[f"doc{i}"] = d.numpy()
    return out


def make_engine_tiny(tread):
    model = random_model("tiny")
    prefix, docs, query = tiny_request(model.config.vocab_size)
    out = run_engine(model, prefix, docs, query, [2, 0, 1])
    np.savez_compressed(os.path.join(HERE, "engine_tiny.npz"), **out)


def make_engine_cfg1(tread):
    """random-init Qwen2.5-0.5B architecture, fp32; prefix 32, docs A-D of
    250, query 16 (seeded uniform ids); request 1 A,B,C,D cold; request 2 D,B,A,C."""
    model = random_model("qwen2.5-0.5b")
    g = torch.Generator().manual_seed(0)
    V = model.config.vocab_size
    prefix = random_tokens(32, V, g)
    docs = [random_tokens(250, V, g) for _ in range(4)]
    query = random_tokens(16, V, g)
    out = run_engine(model, prefix, docs, query, [3, 1, 0, 2])
    np.savez_compressed(os.path.join(HERE, "engine_cfg1.npz"), **out)


def make_engine_bf16_tiny(tread):
    """The tiny architecture in bf16: the engine_tiny request at ratios 0 / 0.2 / 0.5 / 1.0, the
    reference's bf16 deviation values, and its layer-1 tensors of the 0.2 request."""
    model = random_model("tiny", dtype=torch.bfloat16)
    prefix, docs, query = tiny_request(model.config.vocab_size)
    out = run_engine(model, prefix, docs, query, [2, 0, 1], ratios=RATIOS_BF16, layer1_tag="r02")
    np.savez_compressed(os.path.join(HERE, "engine_bf16_tiny.npz"), **out)


def make_engine_bf16_7b3l(tread):
    """BASELINE configs[2] in bf16: the Qwen2.5-7B architecture (hidden 3584, 28/4 heads, head_dim
    128, MLP 18944, vocab 152064) cut to 3 layers so the reference runs on host cores; the full
    request shape, 256 prefix + 16 docs x 496 + 64 query, cold then one reordering."""
    model = random_model("qwen2.5-7b", dtype=torch.bfloat16, layers=3)
    g = torch.Generator().manual_seed(2)
    V = model.config.vocab_size
    prefix = random_tokens(256, V, g)
    docs = [random_tokens(496, V, g) for _ in range(16)]
    query = random_tokens(64, V, g)
    reorder = torch.randperm(16, generator=g).tolist()
    out = run_engine(model, prefix, docs, query, reorder, ratios=RATIOS_BF16)
    np.savez_compressed(os.path.join(HERE, "engine_bf16_7b3l.npz"), **out)


# Requests of the store-pressure sequence: (doc indices in request order, ratio); policy deviation.
STORE_SEQ = (([0, 1, 2], 0.0), ([2, 0, 1], 0.2), ([3, 4], 0.0), ([0, 5, 3], 0.2), ([1, 2, 4, 5], 0.0),
             ([5, 4, 3, 2, 1, 0], 0.2), ([0, 1], 0.0), ([4, 0], 0.5))
STORE_DOC_LENS = (40, 33, 47, 29, 52, 36)


def make_store_engine_bf16(tread):
    """Engine requests through a small two-tier store (tread/store.py:56-125 decisions under
    eviction, offload and CPU-tier hits), bf16 tiny model. Block bytes = 2 * L * Hkv * n * D * 2."""
    from tread.engine import Engine
    from tread.store import BlockStore

    torch.Tensor.pin_memory = lambda self, *a, **k: self  # no CUDA driver here; changes no decision
    model = random_model("tiny", dtype=torch.bfloat16)
    cfg = model.config
    per_tok = 2 * cfg.num_hidden_layers * cfg.num_key_value_heads * (cfg.hidden_size // cfg.num_attention_heads) * 2
    gpu_budget, cpu_budget = per_tok * 100, per_tok * 130
    g = torch.Generator().manual_seed(11)
    prefix = random_tokens(16, cfg.vocab_size, g)
    docs = [random_tokens(n, cfg.vocab_size, g) for n in STORE_DOC_LENS]
    query = random_tokens(8, cfg.vocab_size, g)
    eng = Engine(model, BlockStore(gpu_budget, cpu_budget_bytes=cpu_budget))
    req_stats, store_stats, gpu_keys, cpu_keys, logits, effs = [], [], [], [], [], []
    with torch.inference_mode():
        for idx, ratio in STORE_SEQ:
            lg, _, st = eng.prefill(prefix, [docs[i] for i in idx], query, ratio=ratio)
            req_stats.append([st.hits, st.misses, st.tokens_reused, st.tokens_prefilled])
            effs.append(st.recompute_eff)
            s = eng.store.stats
            store_stats.append([s.hits, s.misses, s.evictions, s.bytes_used, s.cpu_hits, s.offloads,
                                s.cpu_evictions, s.cpu_bytes_used])
            gpu_keys.append(",".join(eng.store.blocks.keys()))
            cpu_keys.append(",".join(eng.store.cpu_blocks.keys()))
            logits.append(bf16_bits(lg))
    out = dict(seq_docs=np.concatenate([np.array(i, np.int64) for i, _ in STORE_SEQ]),
               seq_lens=np.array([len(i) for i, _ in STORE_SEQ], np.int64),
               seq_ratio=np.array([r for _, r in STORE_SEQ], np.float64),
               prefix=prefix.numpy(), query=query.numpy(), gpu_budget=np.int64(gpu_budget),
               cpu_budget=np.int64(cpu_budget), req_stats=np.array(req_stats, np.int64),
               store_stats=np.array(store_stats, np.int64), eff=np.array(effs, np.float64),
               gpu_keys=np.array(gpu_keys), cpu_keys=np.array(cpu_keys), logits=np.stack(logits))
    for i, d in enumerate(docs):
        out[f"doc{i}"] = d.numpy()
    np.savez_compressed(os.path.join(HERE, "store_engine_bf16.npz"), **out)


def make_server(tread):
    """The reference's HTTP app (tread/server.py:131-237) on its own engine, tiny fp32 model, the
    character-level stub tokenizer, a store small enough to evict and offload: the response of
    each request in stub_tokenizer.SERVER_REQUESTS (timing fields dropped) and /metrics after
    the last one. Also records the smallest gap between the two largest logits met by any greedy
    step, so a test can tell that argmax decisions are not knife-edge."""
    import json

    import tread.server as ts
    from fastapi.testclient import TestClient
    from tread.engine import Engine
    from tread.store import BlockStore

    sys.path.insert(0, HERE)
    from stub_tokenizer import SERVER_REQUESTS, StubTokenizer

    torch.Tensor.pin_memory = lambda self, *a, **k: self  # no CUDA driver here; changes no decision
    model = random_model("tiny")
    cfg = model.config
    per_tok = 2 * cfg.num_hidden_layers * cfg.num_key_value_heads * (cfg.hidden_size // cfg.num_attention_heads) * 4
    gpu_budget, cpu_budget = per_tok * 90, per_tok * 70
    gaps = []
    fwd = type(model).forward

    def spy(self, *a, **kw):
        out = fwd(self, *a, **kw)
        top = out.logits[0, -1].float().topk(2).values
        gaps.append(float(top[0] - top[1]))
        return out

    type(model).forward = spy
    try:
        eng = Engine(model, BlockStore(gpu_budget, cpu_budget_bytes=cpu_budget))
        app = ts.build_app(model, StubTokenizer(cfg.vocab_size), eng, eos_ids={cfg.vocab_size - 1})
        client = TestClient(app)
        responses = []
        for prefix, docs, suffix, tenant, max_tokens, ratio, policy in SERVER_REQUESTS:
            r = client.post("/v1/completions", json=dict(prefix=prefix, documents=docs, suffix=suffix, tenant=tenant,
                                                         max_tokens=max_tokens, recompute_ratio=ratio, policy=policy))
            assert r.status_code == 200, r.text
            body = r.json()
            for k in ("ttft_ms", "total_ms"):
                body["tread"].pop(k)
            responses.append(body)
        metrics = client.get("/metrics").json()
        for k in ("ttft_ms_sum", "ttft_ms_mean"):
            metrics.pop(k)
    finally:
        type(model).forward = fwd
    np.savez_compressed(os.path.join(HERE, "server.npz"), responses=np.array(json.dumps(responses)),
                        metrics=np.array(json.dumps(metrics)), gpu_budget=np.int64(gpu_budget),
                        cpu_budget=np.int64(cpu_budget), min_top2_gap=np.float64(min(gaps)))


ALL = ["rope", "deviation", "attention", "store", "engine_tiny", "engine_cfg1", "engine_bf16_tiny",
       "engine_bf16_7b3l", "store_engine_bf16", "server"]


def main():
    import argparse

    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--reference", help="root of the reference checkout (else TREAD_REFERENCE_ROOT)")
    ap.add_argument("fixtures", nargs="*", default=[], help="fixtures to generate (default: all): " + ", ".join(ALL))
    a = ap.parse_args()
    if a.reference:
        ref_shim.set_root(a.reference)
    tread = ref_shim.install()
    torch.set_num_threads(min(8, os.cpu_count() or 1))
    for w in a.fixtures or ALL:
        print("generating", w, flush=True)
        globals()[f"make_{w}"](tread)


if __name__ == "__main__":
    main()
