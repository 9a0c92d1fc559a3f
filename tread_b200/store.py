"""Content-addressed KV block store: GPU (HBM) tier + pinned-host tier, byte budgets, LRU.

Same contract and the same decisions as tread/store.py:56-125 (hit/miss/eviction/offload
accounting is bit-for-bit the reference's): a block is the K/V of one chunk for all layers,
stacked [layers, 1, kv_heads, tokens, head_dim], plus the position it was computed at (`base`).

What changes on B200 is how bytes move between tiers:
  - spill (GPU -> pinned host on eviction, tread/store.py:111) is one DMA copy through the C ABI
    (tread_kv_spill) on a dedicated transfer stream, ordered after the producer by an event, and
    does not block the host; the reference does a synchronous pageable copy plus a pin copy;
  - fetch (pinned host -> GPU on a CPU-tier hit, tread/store.py:75-76) is a DMA copy on the same
    transfer stream that records `Block.ready`; `get(key)` makes the caller's stream wait for it
    (the reference's stream semantics), while the engine passes `wait=False` and waits per block
    just before the rotation kernel that reads it, so fetches overlap rotation of resident blocks.
"""
import hashlib
from collections import OrderedDict
from dataclasses import dataclass
from typing import Optional

import torch

from tread_b200 import kernels


def block_key(*parts) -> str:
    """SHA-256 over every part (tensors as int64 little-endian bytes, everything else as str),
    each followed by a NUL byte: tread/store.py:21-30, so keys are identical to the reference's."""
    h = hashlib.sha256()
    for p in parts:
        if isinstance(p, torch.Tensor):
            h.update(p.detach().to("cpu", torch.int64).numpy().tobytes())
        else:
            h.update(str(p).encode())
        h.update(b"\x00")
    return h.hexdigest()


@dataclass
class Block:
    K: torch.Tensor
    V: torch.Tensor
    base: int
    n_tokens: int
    nbytes: int
    device: torch.device
    hits: int = 0
    ready: Optional[torch.cuda.Event] = None  # set while an async tier transfer into K/V is in flight

    def wait(self, stream=None):
        """Order `stream` (default: current) after any in-flight transfer into this block."""
        if self.ready is not None:
            if self.K.is_cuda:
                (stream or torch.cuda.current_stream(self.K.device)).wait_event(self.ready)
            else:
                self.ready.synchronize()


@dataclass
class StoreStats:
    """Counters with the reference's field names and meanings: `hits` counts lookups served by
    either tier (`cpu_hits` those served from pinned host memory); `evictions` counts every block
    pushed out of HBM, whether it moved to the host tier (`offloads`) or was discarded;
    `cpu_evictions` counts blocks discarded from the host tier; `bytes_used` / `cpu_bytes_used`
    are the bytes each tier holds now."""
    hits: int = 0
    misses: int = 0
    evictions: int = 0
    bytes_used: int = 0
    cpu_hits: int = 0
    offloads: int = 0
    cpu_evictions: int = 0
    cpu_bytes_used: int = 0


class BlockStore:
    def __init__(self, budget_bytes: int, cpu_budget_bytes: int = 0):
        self.budget = budget_bytes
        self.cpu_budget = cpu_budget_bytes
        self.blocks: "OrderedDict[str, Block]" = OrderedDict()  # GPU tier
        self.cpu_blocks: "OrderedDict[str, Block]" = OrderedDict()
        self.stats = StoreStats()
        self._xfer = {}  # device index -> transfer stream
        self._inflight = []  # (event, tensors) kept alive until the copy reading them completes
        # (kind, start event, end event, bytes) of every tier transfer while `timing` is on; no
        # host synchronisation until transfer_rates() reads them
        self.timing = False
        self.transfers = []

    def transfer_stream(self, device):
        idx = torch.device(device).index or 0
        s = self._xfer.get(idx)
        if s is None:
            s = torch.cuda.Stream(device=device)
            self._xfer[idx] = s
        return s

    def get(self, key, wait=True):
        if self._inflight:
            self._reap()
        b = self.blocks.get(key)
        if b is not None:
            self.blocks.move_to_end(key)
        else:
            b = self.cpu_blocks.pop(key, None)
            if b is None:
                self.stats.misses += 1
                return None
            self.stats.cpu_bytes_used -= b.nbytes
            self.stats.cpu_hits += 1
            self._fetch(b)
            self._insert(key, b)
        b.hits += 1
        self.stats.hits += 1
        if wait:
            b.wait()
        return b

    def put(self, key, K, V, base):
        nbytes = sum(t.numel() * t.element_size() for t in (K, V))
        if nbytes > self.budget:
            return None  # larger than the whole HBM budget: the caller uses the K/V uncached
        for tier in (self.blocks, self.cpu_blocks):
            if key in tier:
                self._remove(tier, key)
        b = Block(K=K, V=V, base=base, n_tokens=K.shape[-2], nbytes=nbytes, device=K.device)
        self._insert(key, b)
        return b

    def _insert(self, key, b):
        while self.stats.bytes_used + b.nbytes > self.budget:
            self._evict_gpu()
        self.blocks[key] = b
        self.stats.bytes_used += b.nbytes

    def _evict_gpu(self):
        key, b = self.blocks.popitem(last=False)
        self.stats.bytes_used -= b.nbytes
        self.stats.evictions += 1
        if b.nbytes > self.cpu_budget:
            return
        while self.stats.cpu_bytes_used + b.nbytes > self.cpu_budget:
            _, old = self.cpu_blocks.popitem(last=False)
            self.stats.cpu_bytes_used -= old.nbytes
            self.stats.cpu_evictions += 1
        # The host copy is a separate Block object: the HBM one may still be in use by a request
        # that fetched it earlier (tread/store.py:109-110).
        self.cpu_blocks[key] = self._spill(b)
        self.stats.cpu_bytes_used += b.nbytes
        self.stats.offloads += 1

    def _remove(self, tier, key):
        b = tier.pop(key)
        if tier is self.blocks:
            self.stats.bytes_used -= b.nbytes
        else:
            self.stats.cpu_bytes_used -= b.nbytes

    def __len__(self):
        return len(self.blocks) + len(self.cpu_blocks)

    # -- tier transfers ------------------------------------------------------------------------
    def _spill(self, b):
        if not b.K.is_cuda:  # CPU-only store (tests of the bookkeeping): plain copies
            return Block(K=b.K.clone(), V=b.V.clone(), base=b.base, n_tokens=b.n_tokens, nbytes=b.nbytes,
                         device=b.device, hits=b.hits)
        xs = self.transfer_stream(b.K.device)
        hk = torch.empty(b.K.shape, dtype=b.K.dtype, pin_memory=True)
        hv = torch.empty(b.V.shape, dtype=b.V.dtype, pin_memory=True)
        b.wait()
        xs.wait_stream(torch.cuda.current_stream(b.K.device))  # producer kernels finished
        t0 = self._mark(xs)
        kernels.kv_spill(hk, b.K, xs)
        kernels.kv_spill(hv, b.V, xs)
        self._log("spill", t0, xs, b.nbytes)
        b.K.record_stream(xs)  # keep the HBM alive until the copy has read it
        b.V.record_stream(xs)
        ev = torch.cuda.Event()
        ev.record(xs)
        return Block(K=hk, V=hv, base=b.base, n_tokens=b.n_tokens, nbytes=b.nbytes, device=b.device, hits=b.hits,
                     ready=ev)

    def _fetch(self, b):
        if b.device.type != "cuda":
            return
        xs = self.transfer_stream(b.device)
        dk = torch.empty(b.K.shape, dtype=b.K.dtype, device=b.device)
        dv = torch.empty(b.V.shape, dtype=b.V.dtype, device=b.device)
        xs.wait_stream(torch.cuda.current_stream(b.device))  # the fresh allocations are free to write
        t0 = self._mark(xs)
        kernels.kv_fetch(dk, b.K, xs)  # stream-ordered after this block's spill on the same stream
        kernels.kv_fetch(dv, b.V, xs)
        self._log("fetch", t0, xs, b.nbytes)
        dk.record_stream(xs)
        dv.record_stream(xs)
        b.ready = torch.cuda.Event()
        b.ready.record(xs)
        self._inflight.append((b.ready, (b.K, b.V)))  # the pinned source must outlive the DMA
        b.K, b.V = dk, dv

    def _mark(self, stream):
        if not self.timing:
            return None
        ev = torch.cuda.Event(enable_timing=True)
        ev.record(stream)
        return ev

    def _log(self, kind, t0, stream, nbytes):
        if t0 is not None:
            self.transfers.append((kind, t0, self._mark(stream), nbytes))

    def transfer_rates(self, reset=True):
        """Bytes, device milliseconds and GB/s of the spills and fetches logged while `timing` was
        on (synchronises the device)."""
        torch.cuda.synchronize()
        out = {}
        for kind in ("spill", "fetch"):
            xs = [(a.elapsed_time(b), n) for k, a, b, n in self.transfers if k == kind]
            ms, nb = sum(x[0] for x in xs), sum(x[1] for x in xs)
            out[kind] = {"count": len(xs), "bytes": nb, "ms": round(ms, 3),
                         "gbs": round(nb / (ms * 1e-3) / 1e9, 2) if ms > 0 else None}
        if reset:
            self.transfers = []
        return out

    def _reap(self):
        self._inflight = [(e, t) for e, t in self._inflight if not e.query()]
