"""Data-parallel replicas with KV blocks sharded by content hash across the GPUs of one node.

The reference is single-GPU: one Engine, one BlockStore (tread/engine.py:31-136,
tread/store.py:56-125). Here every GPU runs a full model replica, and the block store is split
across the replicas: block key k (the reference's sha256, tread/store.py:21-30) lives only in
the store of its owner, rank int(k[:16], 16) mod W. That keeps one copy of each block in the
node's HBM, and each replica's GPU/pinned-host budget covers only its shard.

Replicas serve in lockstep rounds, one request each (or none). A round (`HashShardedBlocks.resolve`):
  1. all-gather the request descriptors: prefix key + ids, and each doc's key + ids;
  2. every owner looks its keys up once (GPU tier, or pinned-host tier with an async fetch back)
     and all-gathers which keys it found;
  3. prefix blocks: owners prefill the missing ones, then send each one to every rank that
     needs it. That is the ranks whose request uses it and the owners of missing docs that
     must be prefilled after it. This is one grouped NCCL send/recv batch over NVLink,
     received straight into HBM buffers of the needer;
  4. doc blocks: owners prefill missing docs after their prefix (a doc block is computed at
     positions P.. behind its prefix, base P, as tread/engine.py:86-96 does), then one more
     grouped send/recv batch delivers them to the ranks whose requests use them;
  5. each replica assembles its request from its own and the received blocks with the same
     rotate/gather/append launch and runs blend + query as the single-GPU engine does.

A received block is a transient peer copy: it lives in the needer's HBM for the request only and
is not entered in its store. The exchange is point-to-point only: no TMA, no multicast loads.
"""
import time
from collections import defaultdict

import numpy as np
import torch
import torch.distributed as dist

from tread_b200.engine import Engine, RequestStats, _split_ids, _Tmp
from tread_b200.store import block_key


def owner_of(key: str, world: int) -> int:
    """Rank whose store holds block `key` (a sha256 hex digest)."""
    return int(key[:16], 16) % world


class HashShardedBlocks:
    """The per-round block exchange of hash-sharded replicas.

    store: this rank's BlockStore (its shard). make_prefix(ids) -> (K, V) computes a prefix block;
    make_docs([ids, ...], prefix_block) -> [(K, V), ...] computes doc blocks behind their prefix
    (all of a round's missing docs under one prefix in one call); empty_block(n) -> (K, V)
    allocates receive buffers for an n-token block. ids are int64 numpy arrays."""

    def __init__(self, store, make_prefix, make_docs, empty_block, group=None):
        self.store = store
        self.make_prefix, self.make_docs, self.empty_block = make_prefix, make_docs, empty_block
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.sent_bytes = 0  # peer-copy bytes this rank sent / received (cumulative)
        self.recv_bytes = 0

    def _all_gather(self, obj):
        if self.world == 1:
            return [obj]
        out = [None] * self.world
        dist.all_gather_object(out, obj, group=self.group)
        return out

    def _owner(self, key):
        return owner_of(key, self.world)

    def _put(self, key, K, V, base):
        return self.store.put(key, K, V, base) or _Tmp(K, V, base)

    def _exchange(self, transfers, have, n_tok, base):
        """transfers: sorted (key, needer) pairs, the same list on every rank. Owners send the
        block's K and V, needers receive them; one grouped batch."""
        ops, recv = [], {}
        for key, r in transfers:
            o = self._owner(key)
            if o == self.rank:
                b = have[key]
                b.wait()  # an async pinned-host fetch into the block must land first
                for t in (b.K, b.V):
                    ops.append(dist.P2POp(dist.isend, t, dist.get_global_rank(self.group, r) if self.group else r,
                                          self.group))
                    self.sent_bytes += t.numel() * t.element_size()
            elif r == self.rank:
                K, V = self.empty_block(n_tok[key])
                recv[key] = (K, V)
                for t in (K, V):
                    ops.append(dist.P2POp(dist.irecv, t, dist.get_global_rank(self.group, o) if self.group else o,
                                          self.group))
                    self.recv_bytes += t.numel() * t.element_size()
        if ops:
            for w in dist.batch_isend_irecv(ops):
                w.wait()
        for key, (K, V) in recv.items():
            have[key] = _Tmp(K, V, base[key])

    def resolve(self, desc):
        """One round; every rank calls it. desc: None (no request this round) or
        (prefix_key, prefix_ids, [(doc_key, doc_ids), ...]). Returns None for None, else
        (prefix block, doc blocks, hit flags [prefix, docs...]) with every block on this rank."""
        descs = self._all_gather(desc)
        prefix_ids, doc_of, users = {}, {}, defaultdict(set)
        for r, d in enumerate(descs):
            if d is None:
                continue
            pkey, pids, docs = d
            prefix_ids[pkey] = pids
            users[pkey].add(r)
            for dkey, ids in docs:
                doc_of[dkey] = (pkey, ids)
                users[dkey].add(r)
        keys = sorted(set(prefix_ids) | set(doc_of))
        have, found = {}, {}
        for k in keys:
            if self._owner(k) == self.rank:
                b = self.store.get(k, wait=False)
                found[k] = b is not None
                if b is not None:
                    have[k] = b
        hit = {}
        for p in self._all_gather(found):
            hit.update(p)

        # prefix blocks: to their users and to the owners of missing docs behind them
        for pkey in sorted(prefix_ids):
            if self._owner(pkey) == self.rank and not hit[pkey]:
                K, V = self.make_prefix(prefix_ids[pkey])
                have[pkey] = self._put(pkey, K, V, 0)
        need = {pkey: set(users[pkey]) for pkey in prefix_ids}
        for dkey, (pkey, _) in doc_of.items():
            if not hit[dkey]:
                need[pkey].add(self._owner(dkey))
        self._exchange(sorted((k, r) for k, rs in need.items() for r in rs if r != self._owner(k)), have,
                       {k: len(v) for k, v in prefix_ids.items()}, {k: 0 for k in prefix_ids})

        # doc blocks: prefilled by their owners behind their prefix (one batch per prefix), then
        # to their users
        todo = defaultdict(list)
        for dkey in sorted(doc_of):
            if self._owner(dkey) == self.rank and not hit[dkey]:
                todo[doc_of[dkey][0]].append(dkey)
        for pkey in sorted(todo):
            pb = have[pkey]
            made = self.make_docs([doc_of[k][1] for k in todo[pkey]], pb)
            for dkey, (K, V) in zip(todo[pkey], made):
                have[dkey] = self._put(dkey, K, V, pb.n_tokens)
        self._exchange(sorted((k, r) for k in doc_of for r in users[k] if r != self._owner(k)), have,
                       {k: len(v[1]) for k, v in doc_of.items()},
                       {k: len(prefix_ids[v[0]]) for k, v in doc_of.items()})
        for k in list(have):  # keep only what this rank's own request reads
            if self.rank not in users[k]:
                del have[k]
        if desc is None:
            return None
        pkey, _, docs = desc
        return have[pkey], [have[k] for k, _ in docs], [hit[pkey]] + [hit[k] for k, _ in docs]


class ShardedEngine(Engine):
    """Engine of one data-parallel replica whose BlockStore is this rank's hash shard. `serve` is
    collective: every rank calls it once per round, with its own request or with no arguments."""

    def __init__(self, model, store, group=None):
        super().__init__(model, store, graphs=False)
        self.shards = HashShardedBlocks(store, self._make_prefix, self._make_docs, self._empty_block, group)

    def _ids(self, ids):
        return torch.from_numpy(np.ascontiguousarray(ids, dtype=np.int64)).to(self.net.device)

    def _make_prefix(self, ids):
        return self._prefill_rows(self._ids(ids))

    def _make_docs(self, ids_list, pb):
        return self._prefill_docs([self._ids(ids) for ids in ids_list], pb)

    def _empty_block(self, n):
        shape = (self.net.L, 1, self.net.Hkv, n, self.net.D)
        return (torch.empty(shape, dtype=self.net.dtype, device=self.net.device),
                torch.empty(shape, dtype=self.net.dtype, device=self.net.device))

    @torch.inference_mode()
    def serve(self, prefix_ids=None, docs=(), query_ids=None, ratio=0.0, policy="deviation", namespace=""):
        """Engine.prefill for this replica's request of the round (same arguments and results);
        with no request, takes part in the round's exchange and returns None."""
        if prefix_ids is None:
            self.shards.resolve(None)
            return None
        net = self.net
        st = RequestStats()
        self._sync()
        t0 = time.perf_counter()
        host, devs = _split_ids([prefix_ids] + list(docs) + [query_ids], net.device)
        pkey = block_key(*self.sig, namespace, "prefix", host[0])
        dkeys = [block_key(*self.sig, pkey, d) for d in host[1:-1]]
        desc = (pkey, host[0].numpy(), [(k, d.numpy()) for k, d in zip(dkeys, host[1:-1])])
        pb, blocks, flags = self.shards.resolve(desc)
        for seg, f in zip(host[:-1], flags):
            if f:
                st.hits += 1
                st.tokens_reused += len(seg)
            else:
                st.misses += 1
                st.tokens_prefilled += len(seg)
        return self._run_request(st, t0, devs[0], devs[1:-1], devs[-1], pb, blocks, ratio, policy)
