"""CUDA-graph replay of the selective-recompute layer loop (tread/graphs.py:1-99 contract).

Eagerly, recomputing rows through L layers launches ~8 kernels per layer from Python; the
graph replays the whole loop (cuBLAS projections + tread_rope_rows + tread_attn_rows) as one
launch. Graphs need static shapes, so each call is padded into a bucket (nb >= rows,
Tb >= T + nb - rows) exactly as the reference does (`_bucket`): padded rows sit at positions
T, T+1, ... inside the padding region of the static cache, where the key_pos <= row_pos mask
keeps them invisible to every real row, and their outputs are discarded.
"""
from collections import OrderedDict

import torch

from tread_b200.blend import rows_of


def _bucket(n, T, n_min=64, n_step=256, t_step=1024):
    """(nb, Tb) of tread/graphs.py:22-27: powers of two up to n_step, then multiples of n_step."""
    nb = max(n_min, 1 << (n - 1).bit_length()) if n <= n_step else -(-n // n_step) * n_step
    Tb = -(-(T + nb - n) // t_step) * t_step
    return nb, Tb


class _Graph:
    def __init__(self, net, start, nb, Tb):
        L = net.L
        shape = (L - start, 1, net.Hkv, Tb, net.D)
        self.K = torch.zeros(shape, dtype=net.dtype, device=net.device)
        self.V = torch.zeros_like(self.K)
        self.h = torch.zeros((nb, net.hidden), dtype=net.dtype, device=net.device)
        self.pos = torch.arange(nb, device=net.device)
        self.nbytes = 2 * self.K.numel() * self.K.element_size()
        Ks, Vs = [None] * start + list(self.K.unbind(0)), [None] * start + list(self.V.unbind(0))

        def body():
            return net.run(self.h, self.pos, Ks, Vs, start)

        s = torch.cuda.Stream(device=net.device)
        s.wait_stream(torch.cuda.current_stream(net.device))
        with torch.cuda.stream(s):
            for _ in range(2):
                body()
        torch.cuda.current_stream(net.device).wait_stream(s)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.out = body()


class SubsetRunner:
    """Caches one graph per (start layer, bucket); keeps at most `max_graphs` (LRU). The engine
    also keeps its whole-request graphs (RequestGraph) here, under the same LRU limit."""

    def __init__(self, model, max_graphs=4, max_ctx=2048):
        self.model = model
        self.net = rows_of(model)
        self.max_graphs = max_graphs
        # Above ~2k tokens the copy of the cache into and out of the static buffers costs more
        # than the launches saved (tread/graphs.py:64-66): run eagerly there.
        self.max_ctx = max_ctx
        self.graphs: "OrderedDict[tuple, _Graph]" = OrderedDict()
        self.captures = 0

    def worth_it(self, T):
        return T <= self.max_ctx

    def request_graph(self, key, build):
        key = ("request",) + tuple(key)
        g = self.graphs.get(key)
        if g is None:
            while len(self.graphs) >= self.max_graphs:
                self.graphs.popitem(last=False)
            g = build()
            self.graphs[key] = g
            self.captures += 1
        self.graphs.move_to_end(key)
        return g

    def _graph(self, n, T, start):
        nb, Tb = _bucket(n, T)
        key = (start, nb, Tb)
        g = self.graphs.get(key)
        if g is None:
            while len(self.graphs) >= self.max_graphs:
                self.graphs.popitem(last=False)
            g = _Graph(self.net, start, nb, Tb)
            self.graphs[key] = g
            self.captures += 1
        self.graphs.move_to_end(key)
        return g, nb

    def _replay(self, h, pos, K, V, start, T):
        """K, V: per-layer [1, Hkv, T, D] caches of layers start..L-1 (updated in place)."""
        n = len(pos)
        g, nb = self._graph(n, T, start)
        g.K[..., :T, :].copy_(torch.stack(list(K)))
        g.V[..., :T, :].copy_(torch.stack(list(V)))
        g.pos[:n].copy_(pos)
        g.pos[n:].copy_(torch.arange(T, T + nb - n, device=pos.device))
        g.h[:n].copy_(h.reshape(n, -1))
        g.h[n:].zero_()
        g.graph.replay()
        for l in range(len(K)):
            K[l].copy_(g.K[l, ..., :T, :])
            V[l].copy_(g.V[l, ..., :T, :])
        return g.out[:n]

    @torch.inference_mode()
    def run(self, h, S, K, V, start):
        """Recompute layers start..L-1 for sorted positions S (tread/graphs.py:75-99). K/V: per-layer
        lists for those layers, updated in place. Returns (h, K list, V list)."""
        K, V = list(K), list(V)
        out = self._replay(h, S, K, V, start, K[0].shape[-2])
        return out.reshape(h.shape), K, V

    @torch.inference_mode()
    def run_rows(self, h, pos, Kl, Vl, start):
        """Engine path: rows h at positions pos through layers start..L-1 of the full per-layer
        cache lists Kl/Vl (updated in place). Returns the rows' final hidden states."""
        return self._replay(h, pos, Kl[start:], Vl[start:], start, Kl[0].shape[-2])


class RequestGraph:
    """Everything after assembly for one request shape (prefix length, doc lengths, query length,
    ratio, policy), captured as one CUDA graph over static buffers: the request KV cache (which
    the engine assembles into directly), the context and query token ids, and the logits."""

    def __init__(self, compute, net, P, doc_lens, nq, ratio, policy):
        T = P + sum(doc_lens)
        shape = (net.L, 1, net.Hkv, T + nq, net.D)
        self.K = torch.zeros(shape, dtype=net.dtype, device=net.device)
        self.V = torch.zeros_like(self.K)
        self.ctx = torch.zeros(T, dtype=torch.int64, device=net.device)
        self.q = torch.zeros(nq, dtype=torch.int64, device=net.device)
        # Every tensor the captured kernels read must outlive the graph: keep them on self.
        self.cands = (list(torch.arange(P, T, device=net.device).split(list(doc_lens))) if doc_lens else [])

        def body():
            return compute(self.K, self.V, self.ctx, self.q, self.cands, T, nq, ratio, policy)

        s = torch.cuda.Stream(device=net.device)
        s.wait_stream(torch.cuda.current_stream(net.device))
        with torch.cuda.stream(s):
            for _ in range(2):
                body()
        torch.cuda.current_stream(net.device).wait_stream(s)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.logits, self.eff = body()
        net.err.zero_()  # the warm-up ran on an all-zero cache
