"""Reuse engine: build a request's KV cache from content-addressed chunk blocks, on B200.

Same contract as tread/engine.py: a request is [prefix][doc_1]...[doc_N][query] given as
separate segments; the prefix is reused as an exact prefix, each doc block is computed once
after the prefix (base position P), cached under a key chained from the prefix key, and
re-rotated to wherever it lands in later requests; optional selective recompute repairs the
missing cross-doc attention. Hit/miss accounting and store decisions match the reference.

B200 changes inside `prefill`:
  - assembly is ONE launch of tread_rope_gather_append over all hit blocks straight into the
    request cache [L, 1, Hkv, T + q, D] (reference: one rotate per block + torch.cat); blocks
    fetched from the pinned-host tier are assembled by a second launch that waits only on their
    transfer events, so those copies overlap the first launch;
  - the query segment's rows ride along in the recompute pass (same layer launches, one weight
    read per layer), and with ratio 0 they are the only rows: every row attends to the keys at
    positions <= its own, which reproduces blend-then-query exactly;
  - stage timers keep the reference's names: `blend` covers the layer pass (recompute rows and
    query rows) and the first-token logits, `query` the cache handle;
  - with graphs=True everything after assembly (selection, layers, logits) replays as one CUDA
    graph per request shape, and the request cache is that graph's static buffer, assembled in
    place: the returned cache is valid until the next request of the same shape (as the
    reference's graphed runner returns views of its static buffers, tread/graphs.py:8-13).
"""
import time
from dataclasses import dataclass, field

import torch

from tread_b200 import kernels
from tread_b200.blend import rows_of, select, to_cache
from tread_b200.graphs import RequestGraph, SubsetRunner
from tread_b200.store import BlockStore, block_key


@dataclass
class RequestStats:
    hits: int = 0
    misses: int = 0
    tokens_reused: int = 0
    tokens_prefilled: int = 0
    recompute_eff: float = 0.0
    t: dict = field(default_factory=dict)  # stage -> seconds


class _Tmp:
    """Uncached block (store budget too small for it): same fields as store.Block."""

    def __init__(self, K, V, base):
        self.K, self.V, self.base, self.n_tokens = K, V, base, K.shape[-2]
        self.ready = None

    def wait(self, stream=None):
        pass


def fetch_overlap(store, engine):
    """Share of the logged fetch time (host tier -> HBM copies on the store's transfer stream) that
    the compute stream did not wait for, i.e. that ran under other work of the requests: 1 minus
    the device time of the engine's waits on still-running fetches (recorded while `store.timing`
    is on) over the fetches' own device time. Synchronises the device."""
    torch.cuda.synchronize()
    fetch_ms = sum(a.elapsed_time(b) for k, a, b, _ in store.transfers if k == "fetch")
    if fetch_ms <= 0:
        return None
    waited = sum(max(0.0, a.elapsed_time(b)) for a, b in engine.fetch_waits)
    return max(0.0, 1.0 - waited / fetch_ms)


def _split_ids(segments, device):
    """Host (CPU int64) and device views of a request's token-id segments with at most one
    device->host and one host->device copy: block keys hash host ids, kernels read device ids.
    The reference hashes each segment with its own blocking device->host copy (tread/store.py:26)."""
    lens = [len(s) for s in segments]
    if all(not s.is_cuda for s in segments):
        host = [s.to(torch.int64) for s in segments]
        flat = torch.cat(host)
        if torch.cuda.is_available():
            flat = flat.pin_memory()
        dev_flat = flat.to(device, non_blocking=True)
    else:
        dev_flat = torch.cat([s.to(device=device, dtype=torch.int64) for s in segments])
        host = list(dev_flat.cpu().split(lens))
    return host, list(dev_flat.split(lens))


class Engine:
    def __init__(self, model, store: BlockStore, graphs=False):
        self.model = model
        self.store = store
        self.net = rows_of(model)
        if graphs and getattr(self.net, "world", 1) > 1:
            # a request graph would capture the tensor-parallel all-reduces: not supported
            raise ValueError("graphs=True is not supported with tensor-parallel rows")
        self.runner = SubsetRunner(model) if graphs else None
        self.fetch_waits = []  # (start, end) events of compute-stream waits on fetches, while the store times
        cfg = model.config
        self.sig = (cfg._name_or_path, str(model.dtype), getattr(cfg, "rope_theta", None),
                    getattr(cfg, "rope_scaling", None))

    def _sync(self):
        if torch.cuda.is_available():
            torch.cuda.synchronize()

    # -- blocks ----------------------------------------------------------------------------------
    def _prefill_rows(self, ids, base_cache=None, P=0):
        """K/V [L, 1, Hkv, P + n, D] of `ids` run at positions P.. after an existing prefix cache."""
        net = self.net
        n = len(ids)
        K, V = net.new_cache(P + n)
        if base_cache is not None and P:
            kernels.rope_gather_append([(base_cache[0], base_cache[1], 0, 0)], K, V, net.inv_freq, net.attn_scaling)
        pos = torch.arange(P, P + n, device=ids.device)
        net.run(net.embed_ids(ids), pos, list(K.unbind(0)), list(V.unbind(0)))
        return K, V

    def _prefill_docs(self, docs, pb, max_rows=16384):
        """K/V blocks [L, 1, Hkv, n_i, D] of several docs, each computed at positions P.. behind
        the prefix block `pb`, seeing the prefix and itself only: the block-diagonal packed
        prefill of tread/engine.py:59-96. Docs go through the layers together, up to `max_rows`
        rows per pass: the projections and the MLP run once over all their rows, and RoPE + splice
        and attention run per doc against its own [prefix | doc] cache."""
        net = self.net
        P = pb.n_tokens
        pb.wait()
        out, i = [], 0
        while i < len(docs):
            group = [docs[i]]
            rows = len(docs[i])
            i += 1
            while i < len(docs) and rows + len(docs[i]) <= max_rows:
                group.append(docs[i])
                rows += len(docs[i])
                i += 1
            segs, r0 = [], 0
            for d in group:
                K, V = net.new_cache(P + len(d))
                if P:
                    kernels.rope_gather_append([(pb.K, pb.V, 0, 0)], K, V, net.inv_freq, net.attn_scaling)
                segs.append((r0, r0 + len(d), torch.arange(P, P + len(d), device=d.device), K, V))
                r0 += len(d)
            h = net.embed_ids(torch.cat(group))
            for l in range(net.L):
                h = net.layer_segments(l, h, [(a, b, pos, K[l], V[l]) for a, b, pos, K, V in segs])
            out.extend((K[..., P:, :].contiguous(), V[..., P:, :].contiguous()) for _, _, _, K, V in segs)
        return out

    @torch.inference_mode()
    def prefix_block(self, prefix_ids, st, namespace="", host_ids=None):
        # Doc keys derive from this key, so a namespace isolates a tenant's whole block tree.
        key = block_key(*self.sig, namespace, "prefix", prefix_ids if host_ids is None else host_ids)
        b = self.store.get(key, wait=False)
        if b is None:
            st.misses += 1
            st.tokens_prefilled += len(prefix_ids)
            K, V = self._prefill_rows(prefix_ids.to(self.net.device))
            b = self.store.put(key, K, V, 0) or _Tmp(K, V, 0)
        else:
            st.hits += 1
            st.tokens_reused += len(prefix_ids)
        return key, b

    @torch.inference_mode()
    def doc_blocks(self, prefix_key, pb, docs, st, host_docs=None):
        """Look up every doc's block; prefill the misses after the cached prefix (tread/engine.py:59-96).

        Each missed doc runs at positions P.. over [prefix KV | its own KV], so it sees the prefix
        and itself, never another doc: the reference's block-diagonal packed prefill, with all
        missed docs in one pass (`_prefill_docs`).
        """
        keys = [block_key(*self.sig, prefix_key, d) for d in (docs if host_docs is None else host_docs)]
        blocks = [self.store.get(k, wait=False) for k in keys]
        miss = [i for i, b in enumerate(blocks) if b is None]
        st.hits += len(docs) - len(miss)
        st.tokens_reused += sum(len(d) for d, b in zip(docs, blocks) if b is not None)
        if not miss:
            return blocks
        st.misses += len(miss)
        P = pb.n_tokens
        made = self._prefill_docs([docs[i].to(self.net.device) for i in miss], pb)
        for i, (K, V) in zip(miss, made):
            st.tokens_prefilled += len(docs[i])
            blocks[i] = self.store.put(keys[i], K, V, P) or _Tmp(K, V, P)
        return blocks

    # -- request -----------------------------------------------------------------------------------
    @torch.inference_mode()
    def prefill(self, prefix_ids, docs, query_ids, ratio=0.0, policy="deviation", namespace=""):
        """Build the context cache from blocks, optionally blend, run the query.

        Returns (logits of the last query position, DynamicCache for decoding, RequestStats).
        """
        net = self.net
        st = RequestStats()
        self._sync()
        t0 = time.perf_counter()

        host, devs = _split_ids([prefix_ids] + list(docs) + [query_ids], net.device)
        prefix_ids, docs, query_ids = devs[0], devs[1:-1], devs[-1]
        pkey, pb = self.prefix_block(prefix_ids, st, namespace, host_ids=host[0])
        blocks = self.doc_blocks(pkey, pb, docs, st, host_docs=host[1:-1])
        return self._run_request(st, t0, prefix_ids, docs, query_ids, pb, blocks, ratio, policy)

    def _run_request(self, st, t0, prefix_ids, docs, query_ids, pb, blocks, ratio, policy):
        """Assembly of the prefix block `pb` and the doc `blocks` (device ids), then selection,
        the recompute + query rows and the first-token logits; fills the stage timers of `st`
        (t0: the request's start) and returns (logits, DynamicCache, st)."""
        net = self.net
        P = pb.n_tokens
        nq = len(query_ids)
        T = P + sum(len(d) for d in docs)
        graph = None
        if self.runner is not None and (policy != "random" or ratio == 0):
            # the request's cache is the graph's static buffer: assembled in place, nothing copied
            lens = tuple(len(d) for d in docs)
            graph = self.runner.request_graph(
                (P, lens, nq, ratio, policy),
                lambda: RequestGraph(self._compute, self.net, P, lens, nq, ratio, policy))
            K, V = graph.K, graph.V
        else:
            K, V = self._request_cache(T + nq)
        segs, pending, cands = [(pb, 0, 0)], [], []
        offset = P
        for d, b in zip(docs, blocks):
            segs.append((b, offset - b.base, offset))
            offset += len(d)
        if docs:  # every doc's candidate positions as views of one arange (one launch)
            cands = list(torch.arange(P, offset, device=docs[0].device).split([len(d) for d in docs]))
        ready = [s for s in segs if s[0].ready is None or s[0].ready.query()]
        pending = [s for s in segs if not (s[0].ready is None or s[0].ready.query())]
        timing = getattr(self.store, "timing", False) and torch.cuda.is_available()
        for group in (ready, pending):
            if group:
                if timing and group is pending:
                    # the device time the compute stream spends waiting for still-running fetches
                    a = torch.cuda.Event(enable_timing=True)
                    a.record()
                for b, _, _ in group:
                    b.wait()
                if timing and group is pending:
                    z = torch.cuda.Event(enable_timing=True)
                    z.record()
                    self.fetch_waits.append((a, z))
                kernels.rope_gather_append([(b.K, b.V, dl, o) for b, dl, o in group], K, V, net.inv_freq,
                                           net.attn_scaling)
        self._sync()
        t1 = time.perf_counter()

        ctx = torch.cat([prefix_ids] + list(docs))
        if graph is not None:
            graph.ctx.copy_(ctx)
            graph.q.copy_(query_ids)
            graph.graph.replay()
            logits, st.recompute_eff = graph.logits.clone(), graph.eff
        else:
            logits, st.recompute_eff = self._compute(K, V, ctx, query_ids, cands, T, nq, ratio, policy)
        self._sync()
        t2 = time.perf_counter()
        net.check_errors()

        cache = to_cache(list(K.unbind(0)), list(V.unbind(0)))
        self._sync()
        t3 = time.perf_counter()
        st.t = dict(assemble=t1 - t0, blend=t2 - t1, query=t3 - t2, ttft=t3 - t0)
        return logits, cache, st

    def _compute(self, K, V, ctx, query_ids, cands, T, nq, ratio, policy):
        """Everything after assembly, with no host synchronisation (so it can be graph-captured):
        token selection, the recompute + query rows through the layers, first-token logits.
        Returns (logits [vocab], effective recompute ratio)."""
        net = self.net
        Kl, Vl = list(K.unbind(0)), list(V.unbind(0))
        hq = net.embed_ids(query_ids)
        qpos = torch.arange(T, T + nq, device=query_ids.device)
        start, rows_h, rows_pos, eff = 0, hq, qpos, 0.0
        if ratio > 0 and cands:
            S, hS, start, all_c, hx = select(self.model, ctx, Kl, Vl, cands, ratio, policy, inplace=True,
                                             extra=(hq, qpos))
            if len(S):
                if hS is None:
                    hS = net.embed_ids(ctx[S])
                if hx is not None:
                    hq = hx  # query rows already went through layer 0 with the candidates
                rows_h, rows_pos = torch.cat([hS, hq]), torch.cat([S, qpos])
                n, L = len(all_c), net.L
                eff = (len(S) * (L - start) + start * n) / (n * L)
            else:
                start = 0
        h = net.run(rows_h, rows_pos, Kl, Vl, start)
        return net.logits(h[-1:])[0], eff

    def _request_cache(self, T):
        shape = (self.net.L, 1, self.net.Hkv, T, self.net.D)
        return (torch.empty(shape, dtype=self.net.dtype, device=self.net.device),
                torch.empty(shape, dtype=self.net.dtype, device=self.net.device))

    @torch.inference_mode()
    def prefill_prefix_only(self, prefix_ids, docs, query_ids):
        """Baseline: exact-prefix caching only (tread/engine.py:138-152). The prefix comes from the
        store; every doc is prefilled again."""
        st = RequestStats()
        self._sync()
        t0 = time.perf_counter()
        _, pb = self.prefix_block(prefix_ids, st)
        pb.wait()
        rest = torch.cat(list(docs) + [query_ids]).to(self.net.device)
        st.tokens_prefilled += len(rest) - len(query_ids)
        P = pb.n_tokens
        K, V = self.net.new_cache(P + len(rest))
        kernels.rope_gather_append([(pb.K, pb.V, 0, 0)], K, V, self.net.inv_freq, self.net.attn_scaling)
        Kl, Vl = list(K.unbind(0)), list(V.unbind(0))
        h = self.net.run(self.net.embed_ids(rest), torch.arange(P, P + len(rest), device=rest.device), Kl, Vl)
        logits = self.net.logits(h[-1:])[0]
        self._sync()
        st.t = dict(ttft=time.perf_counter() - t0)
        return logits, to_cache(Kl, Vl), st


@torch.inference_mode()
def prefill_full(model, prefix_ids, docs, query_ids):
    """Baseline: no caching at all (tread/engine.py:155-166), on the same layer math."""
    net = rows_of(model)
    if torch.cuda.is_available():
        torch.cuda.synchronize()
    t0 = time.perf_counter()
    ids = torch.cat([prefix_ids] + list(docs) + [query_ids]).to(net.device)
    K, V = net.new_cache(len(ids))
    Kl, Vl = list(K.unbind(0)), list(V.unbind(0))
    h = net.run(net.embed_ids(ids), torch.arange(len(ids), device=ids.device), Kl, Vl)
    logits = net.logits(h[-1:])[0]
    if torch.cuda.is_available():
        torch.cuda.synchronize()
    st = RequestStats(tokens_prefilled=len(ids) - len(query_ids), t=dict(ttft=time.perf_counter() - t0))
    return logits, to_cache(Kl, Vl), st
