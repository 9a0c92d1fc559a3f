"""The allocation-free selector entry point (tread_deviation_topk_noalloc).

It serves callers that cannot hand the library device scratch: serving loops whose device
memory is owned by a pooling allocator reserved at start-up, loops that avoid cudaMalloc
because it can synchronise the device, and FFI hosts with no device allocator. Its scratch is a
static device array inside the library, so the call allocates nothing. These tests call it
through the C ABI and check that it selects exactly what tread_deviation_topk selects, on two
calls in a row (the second reuses the array the first left behind), on both select paths (keys
held in registers up to 8192 candidates, re-read from L2 above that, up to the array's maximum),
and that its out-of-range flag reaches the caller. The file sorts last so that a run stopping
at the first failure has already run every other test.
"""
import pytest
import torch

from tread_b200 import _capi as C
from tread_b200 import kernels

MAX_N = 65536  # TREAD_NOALLOC_MAX_CANDIDATES


def _call_noalloc(k1, v1, K1, V1, pos, budget, sel_idx, sel_pos, err_flag=None):
    H, n, D = k1.shape
    return C.lib().tread_deviation_topk_noalloc(
        k1.data_ptr(), v1.data_ptr(), k1.stride(1), k1.stride(0), K1.data_ptr(), V1.data_ptr(), K1.stride(1),
        K1.stride(0), K1.shape[1], pos.data_ptr(), n, H, D, budget, C.dtype_code(k1.dtype), sel_idx.data_ptr(),
        sel_pos.data_ptr(), None if err_flag is None else err_flag.data_ptr(),
        C.P(torch.cuda.current_stream().cuda_stream))


@pytest.mark.gpu
@pytest.mark.parametrize("dtype,H,D,n,T", [
    (torch.bfloat16, 4, 128, 8192, 8192),     # register-held keys, the configs[1] shape
    (torch.float32, 2, 64, 1000, 1300),
    (torch.bfloat16, 4, 128, 8193, 9000),     # first size on the L2 re-read select path
    (torch.bfloat16, 2, 128, MAX_N, MAX_N),   # the static array's maximum
])
def test_noalloc_matches_allocating_entry_point(dtype, H, D, n, T):
    dev = torch.device("cuda:0")
    gen = torch.Generator(device=dev).manual_seed(n)
    K1 = torch.randn(H, T, D, device=dev, generator=gen).to(dtype)
    V1 = torch.randn(H, T, D, device=dev, generator=gen).to(dtype)
    pos = torch.sort(torch.randperm(T, device=dev, generator=gen)[:n]).values
    budget = int(round(0.2 * n))
    err = torch.full((1,), 7, dtype=torch.int32, device=dev)
    for call in range(2):
        k1 = (K1[:, pos].float() + 0.1 * torch.randn(H, n, D, device=dev, generator=gen)).to(dtype)
        v1 = (V1[:, pos].float() + 0.1 * torch.randn(H, n, D, device=dev, generator=gen)).to(dtype)
        _, ref_idx, ref_pos = kernels.deviation_topk(k1, v1, K1, V1, pos, budget)
        sel_idx = torch.full((budget,), -1, dtype=torch.int64, device=dev)
        sel_pos = torch.full((budget,), -1, dtype=torch.int64, device=dev)
        rc = _call_noalloc(k1, v1, K1, V1, pos, budget, sel_idx, sel_pos, err)
        assert rc == 0, C.lib().tread_last_error().decode()
        torch.cuda.synchronize()
        assert torch.equal(sel_idx, ref_idx), f"call {call}: selected indices differ"
        assert torch.equal(sel_pos, ref_pos), f"call {call}: selected positions differ"
        assert int(err.item()) == 0, f"call {call}: out-of-range flag set on valid positions"


@pytest.mark.gpu
def test_noalloc_reports_an_out_of_range_position():
    """One candidate position past the cache end: the kernel checks the position before any load
    (that candidate's deviation is NaN), sets the flag, and the next valid call clears it."""
    dev = torch.device("cuda:0")
    gen = torch.Generator(device=dev).manual_seed(3)
    H, D, n, T = 2, 128, 300, 512
    K1 = torch.randn(H, T, D, device=dev, generator=gen).to(torch.bfloat16)
    V1 = torch.randn(H, T, D, device=dev, generator=gen).to(torch.bfloat16)
    k1 = torch.randn(H, n, D, device=dev, generator=gen).to(torch.bfloat16)
    v1 = torch.randn(H, n, D, device=dev, generator=gen).to(torch.bfloat16)
    good = torch.sort(torch.randperm(T, device=dev, generator=gen)[:n]).values
    bad = good.clone()
    bad[-1] = T  # one past the end
    sel_idx = torch.empty(60, dtype=torch.int64, device=dev)
    sel_pos = torch.empty(60, dtype=torch.int64, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    assert _call_noalloc(k1, v1, K1, V1, bad, 60, sel_idx, sel_pos, err) == 0
    torch.cuda.synchronize()
    assert int(err.item()) == 1
    assert int(sel_idx[-1].item()) == n - 1  # NaN deviation ranks first, as in tread_deviation_topk
    assert _call_noalloc(k1, v1, K1, V1, good, 60, sel_idx, sel_pos, err) == 0
    torch.cuda.synchronize()
    assert int(err.item()) == 0


def test_noalloc_rejects_more_candidates_than_its_scratch_holds():
    """Host-side check: nothing is launched (no GPU needed)."""
    rc = C.lib().tread_deviation_topk_noalloc(16, 16, 128, 1024, 16, 16, 128, 4096, 32, 16, MAX_N + 1, 4, 128, 5,
                                              C.TREAD_BF16, 16, 16, None, None)
    assert rc == 1
    assert "static scratch maximum" in C.lib().tread_last_error().decode()
