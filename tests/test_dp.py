"""Hash-sharded data-parallel block exchange (tread_b200.dp.HashShardedBlocks) on CPU `gloo`
ranks with synthetic blocks: every rank receives, bit for bit, the blocks its requests need
(prefix and docs, docs computed behind their prefix by their owner); each key lives only in its
owner's store; a key hits iff an earlier round used it; small budgets that force spills to the
host tier and fetches back change none of that."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from tread_b200.dp import HashShardedBlocks, owner_of
from tread_b200.store import BlockStore, block_key

L, H, D = 2, 1, 4


def make_prefix(ids):
    t = torch.from_numpy(np.asarray(ids, np.float32))
    K = (t.view(1, 1, 1, -1, 1) + torch.arange(L).view(L, 1, 1, 1, 1) * 0.5
         + torch.arange(D).view(1, 1, 1, 1, D) * 0.25).expand(L, 1, H, len(ids), D).contiguous()
    return K, -K


def make_doc(ids, pb):
    K, V = make_prefix(ids)
    return K + pb.K.sum() * 1e-3, V - pb.V.sum() * 1e-3  # depends on the prefix it sits behind


def empty_block(n):
    return torch.empty(L, 1, H, n, D), torch.empty(L, 1, H, n, D)


def _requests(world, rounds, seed=0):
    """Per round, per rank: None or (prefix ids, [doc ids]); docs drawn from a small pool with
    repeats, two prefixes."""
    rng = np.random.default_rng(seed)
    pool = [rng.integers(0, 1000, rng.integers(3, 9)) for _ in range(12)]
    prefixes = [rng.integers(0, 1000, 5), rng.integers(0, 1000, 7)]
    out = []
    for _ in range(rounds):
        rnd = []
        for _r in range(world):
            if rng.random() < 0.15:
                rnd.append(None)
                continue
            docs = [pool[i] for i in rng.choice(len(pool), rng.integers(1, 5), replace=False)]
            rnd.append((prefixes[rng.integers(0, 2)], docs))
        out.append(rnd)
    return out


def _worker(rank, world, port, budget, cpu_budget, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        store = BlockStore(budget, cpu_budget)
        sh = HashShardedBlocks(store, make_prefix, lambda ids, pb: [make_doc(x, pb) for x in ids], empty_block)
        seen = set()
        ok, why = True, ""
        for rnd in _requests(world, 10):
            req = rnd[rank]
            if req is None:
                sh.resolve(None)
            else:
                pids, docs = req
                pkey = block_key("sig", "prefix", torch.from_numpy(pids))
                dkeys = [block_key("sig", pkey, torch.from_numpy(d)) for d in docs]
                pb, blocks, flags = sh.resolve((pkey, pids, list(zip(dkeys, docs))))
                eK, eV = make_prefix(pids)
                ok &= torch.equal(pb.K, eK) and torch.equal(pb.V, eV) and pb.base == 0
                for d, b in zip(docs, blocks):
                    dK, dV = make_doc(d, pb)
                    ok &= torch.equal(b.K, dK) and torch.equal(b.V, dV) and b.base == len(pids)
                if budget >= 1 << 30:  # nothing is ever dropped: hit iff an earlier round used it
                    ok &= flags == [k in seen for k in [pkey] + dkeys]
                if not ok and not why:
                    why = f"mismatch in a round on rank {rank}"
            for rr in rnd:  # every rank knows the whole round's requests (same seed)
                if rr is None:
                    continue
                pk = block_key("sig", "prefix", torch.from_numpy(rr[0]))
                seen.add(pk)
                seen.update(block_key("sig", pk, torch.from_numpy(d)) for d in rr[1])
        keys = set(store.blocks) | set(store.cpu_blocks)
        ok &= all(owner_of(k, world) == rank for k in keys)
        q.put((rank, bool(ok), why, sorted(keys), store.stats.offloads, store.stats.cpu_hits))
        dist.destroy_process_group()
    except Exception as e:  # report to the parent instead of hanging it
        import traceback

        q.put((rank, False, traceback.format_exc(), [], 0, 0))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world,budget,cpu_budget", [(2, 1 << 30, 0), (3, 1 << 30, 0), (2, 600, 1 << 20)])
def test_sharded_exchange_gloo(world, budget, cpu_budget):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, budget, cpu_budget, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=180) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, ok, why, keys, offloads, cpu_hits in res:
        assert ok, why
    if budget >= 1 << 30:
        # the shards partition every key used
        all_keys = [k for r in res for k in r[3]]
        assert len(all_keys) == len(set(all_keys))
    else:
        assert sum(r[4] for r in res) > 0 and sum(r[5] for r in res) > 0  # spills and fetches happened


def test_owner_spreads_keys():
    keys = [block_key("k", i) for i in range(4000)]
    counts = np.bincount([owner_of(k, 8) for k in keys], minlength=8)
    assert counts.min() > 400
