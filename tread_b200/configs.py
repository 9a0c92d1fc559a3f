"""Qwen2-architecture configurations used by the benchmark and the parity tests.

The reference runs real HF checkpoints (`tests/test_engine.py:14`,
`bench/bench_ttft.py:58`); none are available offline, so every model here is a
random-init `transformers.Qwen2ForCausalLM` of the named architecture, built from a fixed
seed so that two processes (or two machines with the same torch build) get identical
weights.
"""
import torch

ARCHS = {
    # name: (layers, hidden, q heads, kv heads, mlp, vocab)
    "qwen2.5-0.5b": (24, 896, 14, 2, 4864, 151936),
    "qwen2.5-7b": (28, 3584, 28, 4, 18944, 152064),
    "qwen2.5-32b": (64, 5120, 40, 8, 27648, 152064),
    # small architecture with the 0.5B's head geometry, for quick GPU/CPU tests
    "tiny": (4, 256, 4, 2, 512, 4096),
}


def qwen2_config(arch, vocab=None, layers=None):
    from transformers import Qwen2Config

    L, hid, hq, hkv, mlp, voc = ARCHS[arch]
    cfg = Qwen2Config(
        vocab_size=vocab or voc,
        hidden_size=hid,
        intermediate_size=mlp,
        num_hidden_layers=layers or L,
        num_attention_heads=hq,
        num_key_value_heads=hkv,
        max_position_embeddings=32768,
        rope_theta=1e6,
        rms_norm_eps=1e-6,
        tie_word_embeddings=False,
        use_sliding_window=False,
    )
    cfg._name_or_path = f"random-init/{arch}"
    cfg._attn_implementation = "sdpa"
    return cfg


def random_model(arch, dtype=torch.float32, device="cpu", seed=0, vocab=None, layers=None, init_on_device=False):
    """Seeded random-init Qwen2ForCausalLM of architecture `arch`.

    By default weights are drawn on the CPU (fp32, then cast and moved), so every process gets the
    same weights. `init_on_device=True` draws them directly on `device` in `dtype` (seconds instead
    of minutes for 7B+ architectures; reproducible on the same GPU model and torch build)."""
    from transformers import Qwen2ForCausalLM

    cfg = qwen2_config(arch, vocab=vocab, layers=layers)
    torch.manual_seed(seed)
    if init_on_device:
        with torch.device(device):
            model = Qwen2ForCausalLM._from_config(cfg, dtype=dtype)
        return model.eval()
    with torch.device("cpu"):
        model = Qwen2ForCausalLM(cfg)
    return model.to(dtype=dtype, device=device).eval()


def random_tokens(n, vocab, gen):
    """Token ids uniform in [0, vocab) from a torch CPU generator."""
    return torch.randint(0, vocab, (n,), generator=gen, dtype=torch.long)
