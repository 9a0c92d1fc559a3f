"""Block store bookkeeping against the reference (host-only; tier transfers need no GPU here
because the trace uses CPU tensors)."""
import hashlib

import numpy as np
import torch

from conftest import golden
from tread_b200.store import BlockStore, block_key


def test_store_trace_matches_reference_decisions():
    """Every hit/miss/eviction/offload counter and both tiers' LRU order after each op of a seeded
    get/put trace equal tread.store.BlockStore's (tests/golden/store.npz)."""
    g = golden("store.npz")
    store = BlockStore(int(g["budget"]), cpu_budget_bytes=int(g["cpu_budget"]))
    for i, (op, key, size) in enumerate(zip(g["op"], g["key"], g["size"])):
        if op == "put":
            K = torch.zeros(int(size), 128)
            V = torch.zeros(int(size), 128)
            b = store.put(str(key), K, V, 0)
            assert (-1 if b is None else b.nbytes) == g["result"][i]
        else:
            b = store.get(str(key))
            assert (-1 if b is None else b.hits) == g["result"][i]
        s = store.stats
        got = [s.hits, s.misses, s.evictions, s.bytes_used, s.cpu_hits, s.offloads, s.cpu_evictions,
               s.cpu_bytes_used]
        np.testing.assert_array_equal(got, g["stats"][i], err_msg=f"op {i}: {op} {key}")
        assert ",".join(store.blocks.keys()) == g["gpu_keys"][i]
        assert ",".join(store.cpu_blocks.keys()) == g["cpu_keys"][i]
        assert store.stats.bytes_used <= store.budget and store.stats.cpu_bytes_used <= store.cpu_budget


def test_block_key_is_the_reference_hash():
    """sha256 over str(part) / int64 token bytes, each followed by NUL (tread/store.py:21-30)."""
    ids = torch.tensor([3, 1, 4, 1, 5], dtype=torch.int32)
    h = hashlib.sha256()
    for part in (b"model", b"torch.bfloat16", b"1000000.0"):
        h.update(part + b"\x00")
    h.update(np.array([3, 1, 4, 1, 5], np.int64).tobytes() + b"\x00")
    assert block_key("model", "torch.bfloat16", 1e6, ids) == h.hexdigest()
    assert block_key("a", ids) != block_key("b", ids)
    assert block_key("a", ids) != block_key("a", ids[:4])


def test_oversize_put_returns_none_without_side_effects():
    store = BlockStore(1000, cpu_budget_bytes=10_000)
    assert store.put("x", torch.zeros(1, 200), torch.zeros(1, 200), 0) is None  # 1600 B > budget
    assert len(store) == 0 and store.stats.misses == 0 and store.stats.evictions == 0


def test_cpu_tier_drop_when_block_exceeds_cpu_budget():
    store = BlockStore(800, cpu_budget_bytes=300)
    store.put("a", torch.zeros(1, 50), torch.zeros(1, 50), 0)  # 400 B
    store.put("b", torch.zeros(1, 50), torch.zeros(1, 50), 0)  # 800 B used: fits exactly
    store.put("c", torch.zeros(1, 50), torch.zeros(1, 50), 0)  # evicts a: 400 > cpu budget -> dropped
    assert store.stats.evictions == 1 and store.stats.offloads == 0 and "a" not in store.cpu_blocks
    assert store.get("a") is None and store.stats.misses == 1
