"""Qwen2Rows.linear on the CPU (the cuBLAS-side branch; the tensor-core branch needs CUDA rows):
the same results as HF Linear / torch.addmm for plain, biased and accumulating calls, and the
routing rule's inputs."""
import pytest
import torch

from tread_b200 import kernels
from tread_b200.qwen2 import Qwen2Rows


def test_linear_matches_addmm_on_cpu():
    g = torch.Generator().manual_seed(0)
    x = torch.randn(5, 32, generator=g)
    w = torch.randn(48, 32, generator=g)
    b = torch.randn(48, generator=g)
    h = torch.randn(5, 48, generator=g)
    assert torch.equal(Qwen2Rows.linear(x, w), x @ w.t())
    assert torch.equal(Qwen2Rows.linear(x, w, bias=b), torch.addmm(b, x, w.t()))
    out = h.clone()
    got = Qwen2Rows.linear(x, w, out=out, accumulate=True)
    assert got.data_ptr() == out.data_ptr() and torch.equal(got, torch.addmm(h, x, w.t()))
    out2 = torch.empty(5, 48)
    assert torch.equal(Qwen2Rows.linear(x, w, bias=b, out=out2), torch.addmm(b, x, w.t()))
    with pytest.raises(ValueError):
        Qwen2Rows.linear(x, w, bias=b, out=h.clone(), accumulate=True)


def test_rows_gemm_takes_only_cuda_16bit_few_rows():
    x = torch.zeros(4, 64, dtype=torch.bfloat16)
    w = torch.zeros(128, 64, dtype=torch.bfloat16)
    assert not kernels.rows_gemm_fits(x, w)  # CPU tensors
    assert not kernels.rows_gemm_fits(x.float(), w.float())
