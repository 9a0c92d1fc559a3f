"""KV-head tensor parallelism on 2 GPUs (NCCL): the TP engine (tread_b200.tp.TPQwen2Rows under
the same Engine) against the single-GPU engine on the same weights and requests.

Bars: store counters identical; selected positions identical across ranks and, for the fp32
model, identical to the single-GPU selection; first-token logits bit-identical across ranks and
within KL 1e-4 (fp32) / 1e-3 (bf16) of the single-GPU engine. Skipped with fewer than 2 GPUs."""
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


def _kl(p_logits, q_logits):
    p = torch.log_softmax(torch.from_numpy(p_logits).double(), -1)
    q = torch.log_softmax(torch.from_numpy(q_logits).double(), -1)
    return float((p.exp() * (p - q)).sum())


def _requests(vocab, seed, doc_len, ndocs):
    g = torch.Generator().manual_seed(seed)
    ids = lambda n: torch.randint(0, vocab, (n,), generator=g)
    prefix, docs, query = ids(32), [ids(doc_len) for _ in range(ndocs)], ids(16)
    order = [docs[i] for i in torch.randperm(ndocs, generator=g).tolist()]
    return prefix, docs, query, order


def _run(engine, reqs, cases):
    """Cold request, then the reordered request per (ratio, policy); numpy results only (the
    queue to the parent would otherwise share tensors by fd, which die with this process)."""
    import tread_b200.engine as te

    prefix, docs, query, order = reqs
    out = []
    _, _, st = engine.prefill(prefix, docs, query)
    out.append(("cold", [st.hits, st.misses, st.tokens_reused, st.tokens_prefilled], None, None))
    for ratio, policy in cases:
        cap = {}
        orig = te.select

        def spy(*a, **kw):
            r = orig(*a, **kw)
            cap["S"] = r[0].cpu().numpy().copy()
            return r

        te.select = spy
        try:
            logits, _, st = engine.prefill(prefix, order, query, ratio=ratio, policy=policy)
        finally:
            te.select = orig
        out.append(((ratio, policy), [st.hits, st.misses, st.tokens_reused, st.tokens_prefilled], cap.get("S"),
                    logits.float().cpu().numpy()))
    return out


def _worker(rank, port, arch, dtype, layers, q):
    try:
        import torch.distributed as dist

        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=WORLD, device_id=dev,
                                timeout=datetime.timedelta(seconds=120))
        from tread_b200.configs import random_model
        from tread_b200.engine import Engine
        from tread_b200.store import BlockStore
        from tread_b200.tp import TPQwen2Rows

        model = random_model(arch, dtype, device=dev, layers=layers, vocab=4096)
        reqs = _requests(4096, 5, 300, 4)
        cases = [(0.0, "deviation"), (0.2, "deviation"), (1.0, "boundary")]
        single = _run(Engine(model, BlockStore(1 << 34)), reqs, cases)
        net = TPQwen2Rows.from_model(model)
        del model
        res = _run(Engine(net, BlockStore(1 << 34)), reqs, cases)
        gathered = []  # every rank's logits, for the bit-identity check
        for (_, _, _, lg) in res[1:]:
            t = torch.from_numpy(lg).to(dev)
            parts = [torch.empty_like(t) for _ in range(WORLD)]
            dist.all_gather(parts, t)
            gathered.append([p.cpu().numpy() for p in parts])
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok", single, res, gathered))
    except Exception as e:  # report to the parent instead of hanging it
        import traceback

        q.put((rank, "error", traceback.format_exc(), repr(e), None))


def _spawn(arch, dtype, layers):
    if torch.cuda.device_count() < WORLD:
        pytest.skip(f"needs {WORLD} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, arch, dtype, layers, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    out = [q.get(timeout=600) for _ in procs]
    for p in procs:
        p.join(timeout=120)
    for r in out:
        assert r[1] == "ok", r[2]
    return sorted(out, key=lambda r: r[0])


@pytest.mark.parametrize("arch,dtype,layers,kl_tol,exact_sel", [
    ("tiny", torch.float32, None, 1e-4, True),
    ("qwen2.5-7b", torch.bfloat16, 3, 1e-3, False),
])
def test_tp2_engine_matches_single_gpu(arch, dtype, layers, kl_tol, exact_sel):
    out = _spawn(arch, dtype, layers)
    for rank, _, single, res, gathered in out:
        for (case_s, st_s, S_s, lg_s), (case_t, st_t, S_t, lg_t) in zip(single, res):
            assert case_s == case_t and st_s == st_t, (case_s, st_s, st_t)
            if lg_s is not None:
                assert _kl(lg_s, lg_t) < kl_tol, (case_s, _kl(lg_s, lg_t))
            if S_s is not None:
                if exact_sel:
                    np.testing.assert_array_equal(S_s, S_t)
                else:
                    assert len(np.intersect1d(S_s, S_t)) >= 0.95 * len(S_s), case_s
        for parts in gathered:
            assert all(np.array_equal(parts[0], p) for p in parts), "ranks disagree on the logits"
    for a, b in zip(out[0][3], out[1][3]):  # both ranks selected the same tokens
        if a[2] is not None:
            np.testing.assert_array_equal(a[2], b[2])
