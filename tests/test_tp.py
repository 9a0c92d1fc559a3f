"""Host logic of KV-head tensor parallelism (tread_b200.tp), on CPU: the weight slicing
reproduces the full layer's arithmetic, and the all-gather of per-head deviation norms over
`gloo` ranks puts every head in global order so the fixed-order sum equals the single-process
oracle deviation bit for bit."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
import torch.nn.functional as F

from oracle import oracle as orc
from tread_b200 import tp
from tread_b200.configs import random_model


def _rms(x, w, eps):
    return w * (x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps))


def _tp_layer_emulated(shards, h, Hq, Hkv, D, world):
    """The TP layer's arithmetic in fp32 torch (no RoPE, causal attention over the rows): per rank
    the column slices, attention over its heads, the row-parallel partial products; summed."""
    R = h.shape[0]
    out = h.clone()
    for p in shards:
        x = _rms(h, p["ln1"], p["ln1_eps"])
        qkv = x @ p["wqkv"].t() + p["bqkv"]
        hq, hk = Hq // world, Hkv // world
        q = qkv[:, :hq * D].view(R, hq, D).transpose(0, 1)
        k = qkv[:, hq * D:(hq + hk) * D].view(R, hk, D).transpose(0, 1)
        v = qkv[:, (hq + hk) * D:].view(R, hk, D).transpose(0, 1)
        G = hq // hk
        o = F.scaled_dot_product_attention(q, k.repeat_interleave(G, 0), v.repeat_interleave(G, 0), is_causal=True)
        out = out + o.transpose(0, 1).reshape(R, -1) @ p["wo"].t()
    h2 = out
    out = h2.clone()
    for p in shards:
        x = _rms(h2, p["ln2"], p["ln2_eps"])
        gu = x @ p["wgu"].t()
        a = F.silu(gu[:, :p["inter"]]) * gu[:, p["inter"]:]
        out = out + a @ p["wd"].t()
    return out


@pytest.mark.parametrize("world", [1, 2])
def test_shards_reproduce_full_layer(world):
    model = random_model("tiny", torch.float32)
    cfg = model.config
    Hq, Hkv = cfg.num_attention_heads, cfg.num_key_value_heads
    D = cfg.hidden_size // Hq
    w = tp._hf_layer(model.model.layers[0])
    with torch.no_grad():
        for b in ("bq", "bk", "bv"):
            w[b].normal_(0, 0.1)  # exercise the bias slicing
        shards = [tp.shard_layer(w, Hq, Hkv, D, r, world) for r in range(world)]
        full = [tp.shard_layer(w, Hq, Hkv, D, 0, 1)]
        h = torch.randn(37, cfg.hidden_size)
        got = _tp_layer_emulated(shards, h, Hq, Hkv, D, world)
        ref = _tp_layer_emulated(full, h, Hq, Hkv, D, 1)
    torch.testing.assert_close(got, ref, rtol=1e-5, atol=1e-5)
    # every weight element lands in exactly one shard
    assert sum(s["wqkv"].numel() for s in shards) == full[0]["wqkv"].numel()
    assert sum(s["wd"].numel() for s in shards) == full[0]["wd"].numel()


def test_kv_head_range():
    assert [tp.kv_head_range(8, r, 4) for r in range(4)] == [(0, 2), (2, 4), (4, 6), (6, 8)]
    with pytest.raises(ValueError):
        tp.kv_head_range(4, 0, 8)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gather_worker(rank, world, port, H, n, D, T, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        rng = np.random.default_rng(3)
        k1 = rng.standard_normal((H, n, D)).astype(np.float32)
        v1 = rng.standard_normal((H, n, D)).astype(np.float32)
        K1 = rng.standard_normal((H, T, D)).astype(np.float32)
        V1 = rng.standard_normal((H, T, D)).astype(np.float32)
        pos = np.sort(rng.choice(T, n, replace=False)).astype(np.int64)
        h0, h1 = tp.kv_head_range(H, rank, world)
        local = orc.head_norms(k1[h0:h1], v1[h0:h1], K1[h0:h1], V1[h0:h1], pos)
        got = tp.gather_head_norms(torch.from_numpy(local)).numpy()
        dev = orc.dev_from_head_norms(got)
        ok = (np.array_equal(got, orc.head_norms(k1, v1, K1, V1, pos)) and
              np.array_equal(dev, orc.deviation(k1, v1, K1, V1, pos)))
        q.put((rank, ok, orc.select_topk(dev, orc.budget_for(0.2, n)).tolist()))
        dist.destroy_process_group()
    except Exception as e:  # report to the parent instead of hanging it
        q.put((rank, False, repr(e)))


@pytest.mark.parametrize("world", [2, 4])
def test_gather_head_norms_gloo(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gather_worker, args=(r, world, port, 8, 257, 64, 300, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    assert all(ok for _, ok, _ in res), res
    sels = [s for _, _, s in res]
    assert all(s == sels[0] for s in sels)  # every rank selects the same tokens


def test_engine_rejects_graphs_with_tensor_parallel_rows(monkeypatch):
    """A request graph would capture the all-reduces of a KV-head split: Engine refuses it."""
    from tread_b200.engine import Engine
    from tread_b200.store import BlockStore

    model = random_model("tiny", torch.float32)
    net = tp.TPQwen2Rows.from_model(model)
    net.world = 2  # as on a rank of a 2-way split
    with pytest.raises(ValueError):
        Engine(net, BlockStore(1 << 20), graphs=True)
    Engine(net, BlockStore(1 << 20), graphs=False)
