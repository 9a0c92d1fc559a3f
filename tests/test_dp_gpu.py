"""Hash-sharded data-parallel replicas on 2 GPUs (NCCL): each replica serves its own requests
through tread_b200.dp.ShardedEngine, receiving the blocks other replicas own by peer copy.
Bars: first-token logits equal (KL < 1e-6) those of a single-GPU Engine serving the same
request on the same weights; each replica's shard holds only keys it owns; the store counters
add up across replicas. Skipped with fewer than 2 GPUs."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

WORLD = 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, port, q):
    try:
        import torch.distributed as dist

        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=WORLD, device_id=dev,
                                timeout=datetime.timedelta(seconds=120))
        from tread_b200.configs import random_model
        from tread_b200.dp import ShardedEngine, owner_of
        from tread_b200.engine import Engine
        from tread_b200.store import BlockStore

        model = random_model("tiny", torch.float32, device=dev, vocab=4096)
        g = torch.Generator().manual_seed(3)
        prefix = torch.randint(0, 4096, (24,), generator=g)
        pool = [torch.randint(0, 4096, (int(n),), generator=g) for n in torch.randint(40, 200, (10,), generator=g)]
        rounds = []
        for _ in range(6):
            rnd = []
            for _r in range(WORLD):
                idx = torch.randperm(10, generator=g)[:int(torch.randint(2, 6, (1,), generator=g))].tolist()
                rnd.append(([pool[i] for i in idx], torch.randint(0, 4096, (8,), generator=g)))
            rounds.append(rnd)
        # small GPU shard budget so blocks spill to the pinned tier and come back
        eng = ShardedEngine(model, BlockStore(1 << 20, 1 << 30))
        ref = Engine(model, BlockStore(1 << 34))
        kls, hits = [], 0
        for i, rnd in enumerate(rounds):
            docs, query = rnd[rank]
            ratio = (0.0, 0.2, 1.0)[i % 3]
            logits, _, st = eng.serve(prefix, docs, query, ratio=ratio)
            want, _, _ = ref.prefill(prefix, docs, query, ratio=ratio)
            p = torch.log_softmax(want.double(), -1)
            lq = torch.log_softmax(logits.double(), -1)
            kls.append(float((p.exp() * (p - lq)).sum()))
            hits += st.hits
        keys = list(eng.store.blocks) + list(eng.store.cpu_blocks)
        owned = all(owner_of(k, WORLD) == rank for k in keys)
        s = eng.store.stats
        q.put((rank, "ok", kls, owned, hits, s.offloads, s.cpu_hits, eng.shards.sent_bytes, eng.shards.recv_bytes))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        import traceback

        q.put((rank, "error", traceback.format_exc(), None, 0, 0, 0, 0, 0))


def test_dp2_sharded_replicas_match_single_gpu():
    if torch.cuda.device_count() < WORLD:
        pytest.skip(f"needs {WORLD} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    out = [q.get(timeout=600) for _ in procs]
    for p in procs:
        p.join(timeout=120)
    for r in out:
        assert r[1] == "ok", r[2]
    for rank, _, kls, owned, hits, offloads, cpu_hits, sent, recv in out:
        assert max(kls) < 1e-6, kls
        assert owned
    assert sum(r[4] for r in out) > 0  # later rounds hit blocks that earlier rounds made
    assert sum(r[7] for r in out) == sum(r[8] for r in out) > 0  # peer copies happened, bytes balance
    assert sum(r[5] for r in out) > 0 and sum(r[6] for r in out) > 0  # spills and fetches happened
