"""The HTTP front end (tread_b200.server.build_app) on the B200 engine against the reference's own
server run on its own engine (tests/golden/server.npz): the same requests give the same greedy
text, finish reasons, usage and reuse stats, and /metrics reports the same counters and store
occupancy (tiny fp32 model, character-level stub tokenizer, a store small enough to evict,
offload and hit its pinned tier)."""
import json

import numpy as np
import pytest
import torch
from fastapi.testclient import TestClient

from conftest import golden
from golden.stub_tokenizer import SERVER_REQUESTS, StubTokenizer
from tread_b200 import BlockStore, Engine
from tread_b200.configs import random_model
from tread_b200.server import build_app

pytestmark = pytest.mark.gpu


def _client(cuda, g, **kw):
    model = random_model("tiny").to(cuda)
    V = model.config.vocab_size
    eng = Engine(model, BlockStore(int(g["gpu_budget"]), cpu_budget_bytes=int(g["cpu_budget"])))
    return TestClient(build_app(model, StubTokenizer(V), eng, eos_ids={V - 1}, **kw))


def test_server_matches_reference_server(cuda):
    g = golden("server.npz")
    # greedy steps of the reference never had its top two logits closer than this, far above the
    # fp32 differences between the two engines, so every argmax must agree
    assert float(g["min_top2_gap"]) > 1e-3
    want = json.loads(str(g["responses"]))
    client = _client(cuda, g)
    for (prefix, docs, suffix, tenant, max_tokens, ratio, policy), ref in zip(SERVER_REQUESTS, want):
        r = client.post("/v1/completions", json=dict(prefix=prefix, documents=docs, suffix=suffix, tenant=tenant,
                                                     max_tokens=max_tokens, recompute_ratio=ratio, policy=policy))
        assert r.status_code == 200, r.text
        body = r.json()
        assert body["tread"]["ttft_ms"] > 0 and body["tread"]["total_ms"] >= body["tread"]["ttft_ms"]
        for k in ("ttft_ms", "total_ms"):
            body["tread"].pop(k)
        assert body == ref
    m = client.get("/metrics").json()
    assert m["ttft_ms_mean"] > 0
    for k in ("ttft_ms_sum", "ttft_ms_mean"):
        m.pop(k)
    assert m == json.loads(str(g["metrics"]))
    assert client.get("/health").json()["status"] == "ok"


def test_server_contract_errors(cuda):
    g = golden("server.npz")
    client = _client(cuda, g, max_context=64, api_key="k")
    ok = {"authorization": "Bearer k"}
    body = dict(prefix="p", documents=["d"], suffix="s", max_tokens=4)
    assert client.post("/v1/completions", json=body).status_code == 401
    assert client.post("/v1/completions", json={**body, "policy": "nope"}, headers=ok).status_code == 422
    assert client.post("/v1/completions", json={**body, "recompute_ratio": 1.5}, headers=ok).status_code == 422
    assert client.post("/v1/completions", json={**body, "documents": ["x" * 100]}, headers=ok).status_code == 413
    r = client.post("/v1/completions", json=body, headers=ok)
    assert r.status_code == 200 and r.json()["usage"]["prompt_tokens"] == 3
