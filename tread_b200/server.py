"""HTTP front end of the B200 engine, with tread's serving contract (tread/server.py:131-237).

    POST /v1/completions   segments in ({prefix, documents[], suffix, tenant, max_tokens,
                           recompute_ratio, policy}), greedy text out, plus the `tread` block of
                           reuse stats (block hits/misses, tokens reused/prefilled, recompute_eff,
                           ttft_ms, total_ms)
    GET  /metrics          request counters and the block store's occupancy and decisions
    GET  /health

Request and response fields, status codes (422 schema, 413 prompt too long, 429 queue full, 503
timed out waiting for the GPU, 401 bad bearer token) and greedy decoding are the reference's,
so a client of the reference server sees the same API. What differs is below the API: prefill is
`tread_b200.Engine.prefill` (host token ids in; one host-to-device copy inside the call) and the
decode steps run the HF model over the `DynamicCache` that prefill hands back, whose layers are
views of the request's assembled cache.

The engine is not thread-safe: one lock serialises GPU work; at most `max_queue` requests may be in
flight. Documents are tokenized as untrusted text (control-token text stays plain text); prefix
and suffix are operator-controlled. The tokenizer is shared, so every call to it holds a lock.
"""
import hmac
import threading
import time
from typing import Annotated

import torch
from fastapi import Depends, FastAPI, HTTPException, Request
from pydantic import BaseModel, Field, StringConstraints

MAX_SEGMENT_CHARS = 200_000
MAX_DOCUMENTS = 256
# generous characters-per-token bound used to reject huge prompts before tokenizing them
MAX_CHARS_PER_TOKEN = 32


class CompletionRequest(BaseModel):
    prefix: str = Field(min_length=1, max_length=MAX_SEGMENT_CHARS)
    documents: list[Annotated[str, StringConstraints(min_length=1, max_length=MAX_SEGMENT_CHARS)]] = Field(
        default_factory=list, max_length=MAX_DOCUMENTS)
    suffix: str = Field(min_length=1, max_length=MAX_SEGMENT_CHARS)
    tenant: str = Field("", max_length=128)
    max_tokens: int = Field(64, ge=1, le=2048)
    recompute_ratio: float = Field(0.2, ge=0.0, le=1.0)
    policy: str = Field("deviation", pattern="^(deviation|boundary|random)$")


class _Tokenizer:
    """HF tokenizer behind a lock; `untrusted` text is split without special-token parsing."""

    def __init__(self, tok):
        self.tok, self.lock = tok, threading.Lock()

    def encode(self, text, untrusted):
        with self.lock:
            return self.tok(text, add_special_tokens=False, split_special_tokens=untrusted).input_ids

    def decode(self, ids):
        with self.lock:
            return self.tok.decode(ids)


def build_app(model, tok, engine, eos_ids, max_context=16384, api_key=None, max_queue=16, queue_timeout=30.0,
              max_seconds=120.0):
    """FastAPI app serving `engine` (a tread_b200.Engine over `model`) with tokenizer `tok`."""

    def auth(request: Request):
        if api_key is not None and not hmac.compare_digest(request.headers.get("authorization", "").encode(),
                                                           f"Bearer {api_key}".encode()):
            raise HTTPException(401, "invalid or missing bearer token", headers={"WWW-Authenticate": "Bearer"})

    app = FastAPI(title="tread_b200", dependencies=[Depends(auth)])
    gpu = threading.Lock()
    slots = threading.BoundedSemaphore(max_queue)
    tk = _Tokenizer(tok)
    eos = set(int(e) for e in eos_ids)
    counters = dict(requests=0, ttft_ms_sum=0.0, tokens_reused=0, tokens_prefilled=0, generated_tokens=0)

    def tokenize(req):
        segs = [(req.prefix, False)] + [(d, True) for d in req.documents] + [(req.suffix, False)]
        if sum(len(t) for t, _ in segs) > max_context * MAX_CHARS_PER_TOKEN:
            raise HTTPException(413, f"prompt exceeds {max_context * MAX_CHARS_PER_TOKEN} characters")
        left, ids = max_context - req.max_tokens, []
        for text, untrusted in segs:
            ids.append(tk.encode(text, untrusted))
            left -= len(ids[-1])
            if left < 0:
                raise HTTPException(413, f"prompt + {req.max_tokens} new tokens exceeds limit {max_context}")
        return ids

    def generate(req, ids):
        host = [torch.tensor(x, dtype=torch.long) for x in ids]
        with torch.inference_mode():
            t0 = time.perf_counter()
            logits, cache, st = engine.prefill(host[0], host[1:-1], host[-1], ratio=req.recompute_ratio,
                                               policy=req.policy, namespace=req.tenant)
            nxt = int(logits.argmax().item())
            out, reason = [], "stop"
            dev = logits.device
            while nxt not in eos:
                if len(out) >= req.max_tokens:
                    reason = "length"
                    break
                if time.perf_counter() - t0 > max_seconds:
                    reason = "time"
                    break
                out.append(nxt)
                o = model(torch.tensor([[nxt]], device=dev), past_key_values=cache, use_cache=True, logits_to_keep=1)
                cache, nxt = o.past_key_values, int(o.logits[0, -1].argmax().item())
            total = time.perf_counter() - t0
        counters["requests"] += 1
        counters["ttft_ms_sum"] += st.t["ttft"] * 1e3
        counters["tokens_reused"] += st.tokens_reused
        counters["tokens_prefilled"] += st.tokens_prefilled
        counters["generated_tokens"] += len(out)
        return {
            "text": tk.decode(out),
            "finish_reason": reason,
            "usage": {"prompt_tokens": sum(map(len, ids)), "completion_tokens": len(out)},
            "tread": {"block_hits": st.hits, "block_misses": st.misses, "tokens_reused": st.tokens_reused,
                      "tokens_prefilled": st.tokens_prefilled, "recompute_eff": round(st.recompute_eff, 4),
                      "ttft_ms": round(st.t["ttft"] * 1e3, 2), "total_ms": round(total * 1e3, 2)},
        }

    @app.get("/health")
    def health():
        return {"status": "ok", "model": model.config._name_or_path}

    @app.post("/v1/completions")
    def complete(req: CompletionRequest):
        if not slots.acquire(blocking=False):
            raise HTTPException(429, f"server busy: {max_queue} requests already in flight",
                                headers={"Retry-After": "1"})
        try:
            ids = tokenize(req)
            if not gpu.acquire(timeout=queue_timeout):
                raise HTTPException(503, f"timed out after {queue_timeout}s waiting for the GPU",
                                    headers={"Retry-After": "5"})
            try:
                return generate(req, ids)
            finally:
                gpu.release()
        finally:
            slots.release()

    @app.get("/metrics")
    def metrics():
        s = engine.store.stats
        return {**counters, "ttft_ms_mean": counters["ttft_ms_sum"] / max(1, counters["requests"]),
                "store": {"blocks_gpu": len(engine.store.blocks), "blocks_cpu": len(engine.store.cpu_blocks),
                          "gpu_bytes": s.bytes_used, "cpu_bytes": s.cpu_bytes_used, "hits": s.hits,
                          "misses": s.misses, "cpu_hits": s.cpu_hits, "offloads": s.offloads,
                          "evictions": s.evictions, "cpu_evictions": s.cpu_evictions}}

    return app
