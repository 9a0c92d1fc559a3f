"""Test infrastructure: import the unmodified tread reference under transformers 5.x.

Used only by `tests/golden/make_golden.py` (fixture generation) and by CPU tests that
cross-check the oracle against the live reference when it is present. Nothing in the
product imports this module.

tread was written against transformers 4.46.3 (`requirements.txt:3-4`); the installed
transformers is 5.5. Three attribute renames separate them, and this shim bridges them
without touching the reference sources:

1. `DynamicCache.key_cache` / `.value_cache` (read by `tread/blend.py:19`,
   `tread/engine.py:89`) -> per-layer `.layers[i].keys` / `.values`;
2. `Qwen2Attention.num_heads` / `.num_key_value_heads` (read by `tread/blend.py:84-86,107`)
   -> derived from the config;
3. `Qwen2ForCausalLM.forward(num_logits_to_keep=...)` (`tread/engine.py:132,148,161`)
   -> `logits_to_keep=`.
"""
import os
import sys

# The reference checkout's root (the directory that holds the `tread` package): taken from the
# TREAD_REFERENCE_ROOT environment variable, or set with `set_root()` before `install()`.
REFERENCE_ROOT = os.environ.get("TREAD_REFERENCE_ROOT", "")


def set_root(path):
    global REFERENCE_ROOT
    REFERENCE_ROOT = path


def available() -> bool:
    return bool(REFERENCE_ROOT) and os.path.isdir(os.path.join(REFERENCE_ROOT, "tread"))


_patched = False


def install():
    """Patch transformers once and put the reference on sys.path. Returns the `tread` package."""
    global _patched
    if not available():
        raise RuntimeError(f"tread reference not found under {REFERENCE_ROOT!r}: set TREAD_REFERENCE_ROOT")
    if not _patched:
        from transformers import DynamicCache
        from transformers.models.qwen2 import modeling_qwen2 as mq

        DynamicCache.key_cache = property(lambda self: [layer.keys for layer in self.layers])
        DynamicCache.value_cache = property(lambda self: [layer.values for layer in self.layers])
        mq.Qwen2Attention.num_heads = property(lambda self: self.config.num_attention_heads)
        mq.Qwen2Attention.num_key_value_heads = property(lambda self: self.config.num_key_value_heads)
        fwd = mq.Qwen2ForCausalLM.forward

        def forward(self, *a, num_logits_to_keep=None, **kw):
            if num_logits_to_keep is not None:
                kw["logits_to_keep"] = num_logits_to_keep
            return fwd(self, *a, **kw)

        mq.Qwen2ForCausalLM.forward = forward
        if REFERENCE_ROOT not in sys.path:
            sys.path.insert(0, REFERENCE_ROOT)
        _patched = True
    import tread  # noqa: F401  (the reference package)
    import tread.blend
    import tread.engine
    import tread.graphs
    import tread.store
    return tread
