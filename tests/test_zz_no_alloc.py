"""The allocation-free selector entry point (tread_deviation_topk_noalloc).

It serves callers that cannot hand the library device scratch: serving loops whose device
memory is owned by a pooling allocator reserved at start-up, loops that avoid cudaMalloc
because it can synchronise the device, and FFI hosts with no device allocator. Its scratch is a
static device array inside the library, so the call allocates nothing. These tests call it
through the C ABI and check that it selects exactly what tread_deviation_topk selects, on two
calls in a row (the second reuses the array the first left behind). The file sorts last so that
a run stopping at the first failure has already run every other test.
"""
import pytest
import torch

from tread_b200 import _capi as C
from tread_b200 import kernels

MAX_N = 65536  # TREAD_NOALLOC_MAX_CANDIDATES


def _call_noalloc(k1, v1, K1, V1, pos, budget, sel_idx, sel_pos):
    H, n, D = k1.shape
    return C.lib().tread_deviation_topk_noalloc(
        k1.data_ptr(), v1.data_ptr(), k1.stride(1), k1.stride(0), K1.data_ptr(), V1.data_ptr(), K1.stride(1),
        K1.stride(0), K1.shape[1], pos.data_ptr(), n, H, D, budget, C.dtype_code(k1.dtype), sel_idx.data_ptr(),
        sel_pos.data_ptr(), C.P(torch.cuda.current_stream().cuda_stream))


@pytest.mark.gpu
@pytest.mark.parametrize("dtype,H,D,n,T", [(torch.bfloat16, 4, 128, 8192, 8192), (torch.float32, 2, 64, 1000, 1300)])
def test_noalloc_matches_allocating_entry_point(dtype, H, D, n, T):
    dev = torch.device("cuda:0")
    gen = torch.Generator(device=dev).manual_seed(n)
    K1 = torch.randn(H, T, D, device=dev, generator=gen).to(dtype)
    V1 = torch.randn(H, T, D, device=dev, generator=gen).to(dtype)
    pos = torch.sort(torch.randperm(T, device=dev, generator=gen)[:n]).values
    budget = int(round(0.2 * n))
    for call in range(2):
        k1 = (K1[:, pos].float() + 0.1 * torch.randn(H, n, D, device=dev, generator=gen)).to(dtype)
        v1 = (V1[:, pos].float() + 0.1 * torch.randn(H, n, D, device=dev, generator=gen)).to(dtype)
        _, ref_idx, ref_pos = kernels.deviation_topk(k1, v1, K1, V1, pos, budget)
        sel_idx = torch.full((budget,), -1, dtype=torch.int64, device=dev)
        sel_pos = torch.full((budget,), -1, dtype=torch.int64, device=dev)
        rc = _call_noalloc(k1, v1, K1, V1, pos, budget, sel_idx, sel_pos)
        assert rc == 0, C.lib().tread_last_error().decode()
        torch.cuda.synchronize()
        assert torch.equal(sel_idx, ref_idx), f"call {call}: selected indices differ"
        assert torch.equal(sel_pos, ref_pos), f"call {call}: selected positions differ"


def test_noalloc_rejects_more_candidates_than_its_scratch_holds():
    """Host-side check: nothing is launched (no GPU needed)."""
    rc = C.lib().tread_deviation_topk_noalloc(16, 16, 128, 1024, 16, 16, 128, 4096, 32, 16, MAX_N + 1, 4, 128, 5,
                                              C.TREAD_BF16, 16, 16, None)
    assert rc == 1
    assert "static scratch maximum" in C.lib().tread_last_error().decode()
