"""The CPU restatement of the request path (oracle/engine_port.py, the TTFT CPU baseline) against
fixtures the unmodified reference produced: request stats, selected positions and first-token
logits on the tiny (fp32, bf16) and configs[0] (Qwen2.5-0.5B architecture, fp32) models."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from conftest import golden
from oracle.engine_port import CpuPort
from tread_b200.configs import random_model


def kl(a, b):
    return F.kl_div(F.log_softmax(torch.as_tensor(a).float(), -1), F.log_softmax(torch.as_tensor(b).float(), -1),
                    log_target=True, reduction="sum").item()


def logits_of(g, key):
    a = g[key]
    if a.dtype == np.uint16:  # bf16 bits
        return torch.from_numpy((a.astype(np.uint32) << 16).view(np.float32))
    return torch.from_numpy(a)


def _port_vs_golden(model, g, kl_tol, tags):
    prefix = torch.from_numpy(g["prefix"])
    docs = [torch.from_numpy(g[f"doc{i}"]) for i in range(sum(k.startswith("doc") for k in g.files))]
    query = torch.from_numpy(g["query"])
    order = [docs[i] for i in g["reorder"]]
    port = CpuPort(model)
    _, st, _ = port.prefill(prefix, docs, query)
    assert [st[k] for k in ("hits", "misses", "tokens_reused", "tokens_prefilled")] == g["stats_cold"].tolist()
    for tag, ratio, policy in tags:
        logits, st, S = port.prefill(prefix, order, query, ratio=ratio, policy=policy)
        assert [st[k] for k in ("hits", "misses", "tokens_reused", "tokens_prefilled")] == g[f"stats_{tag}"].tolist()
        assert st["recompute_eff"] == pytest.approx(float(g[f"eff_{tag}"]), abs=1e-12)
        if f"S_{tag}" in g.files:
            np.testing.assert_array_equal(S.numpy(), g[f"S_{tag}"])
        assert kl(logits_of(g, f"logits_{tag}"), logits) < kl_tol, tag


TAGS = (("r0", 0.0, "deviation"), ("r02", 0.2, "deviation"), ("b10", 1.0, "boundary"))


def test_port_tiny_fp32():
    _port_vs_golden(random_model("tiny"), golden("engine_tiny.npz"), 1e-6, TAGS)


def test_port_tiny_bf16():
    _port_vs_golden(random_model("tiny", dtype=torch.bfloat16), golden("engine_bf16_tiny.npz"), 1e-3,
                    TAGS + (("r05", 0.5, "deviation"),))


def test_port_cfg1_fp32():
    _port_vs_golden(random_model("qwen2.5-0.5b"), golden("engine_cfg1.npz"), 1e-4, TAGS)
