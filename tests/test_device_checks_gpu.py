"""The kernel wrappers refuse a tensor that is not on the call's device (a host tensor here)
before anything launches: every kernel dereferences all its tensors on that one device."""
import pytest
import torch

from tread_b200 import kernels

pytestmark = pytest.mark.gpu


def test_wrappers_refuse_host_tensors(cuda):
    g = torch.Generator(device=cuda).manual_seed(0)
    R, Hq, Hkv, D, T = 8, 4, 2, 128, 256
    q = torch.randn(R, Hq, D, device=cuda, generator=g).to(torch.bfloat16)
    K = torch.randn(Hkv, T, D, device=cuda, generator=g).to(torch.bfloat16)
    V = torch.randn_like(K)
    pos = torch.arange(T - R, T, device=cuda)
    with pytest.raises(ValueError):
        kernels.attn_rows(q, K, V, pos.cpu())
    with pytest.raises(ValueError):
        kernels.attn_rows(q, K, V, pos, out=torch.empty(R, Hq, D, dtype=torch.bfloat16))
    qkv = torch.randn(R, (Hq + 2 * Hkv) * D, device=cuda, generator=g).to(torch.bfloat16)
    inv = [1.0] * (D // 2)
    with pytest.raises(ValueError):
        kernels.rope_rows(qkv, pos.cpu(), Hq, Hkv, D, torch.empty_like(q), K, V, inv)
    x = torch.randn(R, 256, device=cuda, generator=g).to(torch.bfloat16)
    with pytest.raises(ValueError):
        kernels.rmsnorm(x, torch.ones(256, dtype=torch.bfloat16), 1e-6)
    with pytest.raises(ValueError):
        kernels.silu_mul(x, out=torch.empty(R, 128, dtype=torch.bfloat16))
    k1 = torch.randn(Hkv, R, D, device=cuda, generator=g).to(torch.bfloat16)
    with pytest.raises(ValueError):
        kernels.deviation_topk(k1, k1, K, V, pos, 2, dev_out=torch.empty(R))
    torch.cuda.synchronize()
    # the same calls with every tensor on the device run
    kernels.attn_rows(q, K, V, pos)
    kernels.rmsnorm(x, torch.ones(256, dtype=torch.bfloat16, device=cuda), 1e-6)
    torch.cuda.synchronize()
