"""Few-row projection GEMM (tread_rows_gemm) against an fp32 torch reference of the same op.

The kernel accumulates in fp32 and rounds once, so it must land within one output ulp of the
fp32 product (rtol 2^-7 for bf16, 2^-10 for fp16, plus a small absolute term for sums near
zero). Shapes cover the query forward's projections of the 7B architecture, ragged N and K
(partial feature tiles and K chunks), every row count class (1..128), bias, accumulation into
the output, and the K-split path (deterministic: its partial sums are added in split order).
"""
import pytest
import torch

from tread_b200 import kernels

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _case(M, N, K, dtype, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    x = torch.randn(M, K, device=DEV, generator=g).to(dtype)
    w = (torch.randn(N, K, device=DEV, generator=g) * K ** -0.5).to(dtype)
    b = torch.randn(N, device=DEV, generator=g).to(dtype)
    o = torch.randn(M, N, device=DEV, generator=g).to(dtype)
    return x, w, b, o


def _check(got, ref, dtype):
    rtol = 2.0 ** -7 if dtype == torch.bfloat16 else 2.0 ** -10
    err = (got.float() - ref).abs()
    bound = rtol * ref.abs() + 1e-3
    assert bool((err <= bound).all()), f"max err {float(err.max()):.3g} (bound at that element exceeded)"


SHAPES = [(4608, 3584), (3584, 3584), (3584, 18944), (37888 // 8, 3584), (300, 136), (1000, 72)]


@pytest.mark.parametrize("M", [1, 7, 16, 33, 64, 100, 128])
@pytest.mark.parametrize("N,K", SHAPES)
def test_rows_gemm_matches_fp32(M, N, K):
    x, w, b, _ = _case(M, N, K, torch.bfloat16, M * 131 + N + K)
    got = kernels.rows_gemm(x, w, bias=b)
    ref = x.float() @ w.float().t() + b.float()
    _check(got, ref, torch.bfloat16)


@pytest.mark.parametrize("split", [True, False])
@pytest.mark.parametrize("M", [1, 64])
def test_rows_gemm_accumulates_into_out(M, split):
    N, K = 3584, 18944
    x, w, _, o = _case(M, N, K, torch.bfloat16, 7 + M)
    ref = o.float() + x.float() @ w.float().t()
    got = kernels.rows_gemm(x, w, out=o.clone(), accumulate=True, split=split)
    _check(got, ref, torch.bfloat16)


def test_rows_gemm_fp16_and_no_bias():
    x, w, _, _ = _case(64, 4608, 3584, torch.float16, 3)
    got = kernels.rows_gemm(x, w)
    _check(got, x.float() @ w.float().t(), torch.float16)


def test_rows_gemm_split_is_deterministic():
    """K-split calls of different shapes back to back through the shared workspace give the same
    bits every time (the splits are added in split order), and the same as the unsplit kernel
    within rounding."""
    x1, w1, b1, _ = _case(64, 3584, 3584, torch.bfloat16, 11)
    x2, w2, b2, _ = _case(5, 640, 18944, torch.bfloat16, 12)
    a1 = kernels.rows_gemm(x1, w1, bias=b1)
    a2 = kernels.rows_gemm(x2, w2, bias=b2)
    for _ in range(3):
        assert torch.equal(kernels.rows_gemm(x1, w1, bias=b1), a1)
        assert torch.equal(kernels.rows_gemm(x2, w2, bias=b2), a2)
    _check(a1, kernels.rows_gemm(x1, w1, bias=b1, split=False).float(), torch.bfloat16)


def test_rows_gemm_strided_views():
    """Row-strided inputs and output (a slice of a wider tensor), as the k/v columns of a fused
    projection weight are."""
    x, w, b, _ = _case(64, 4608, 3584, torch.bfloat16, 21)
    wk = w[3584:]  # the k/v rows of a fused q/k/v weight
    out = torch.zeros(64, 2048, dtype=torch.bfloat16, device=DEV)
    got = kernels.rows_gemm(x, wk, bias=b[3584:], out=out[:, 512:1536])
    _check(got, x.float() @ wk.float().t() + b[3584:].float(), torch.bfloat16)
    assert int(out[:, :512].count_nonzero()) == 0 and int(out[:, 1536:].count_nonzero()) == 0


def test_query_forward_streams_the_wide_weights_through_rows_gemm(monkeypatch):
    """With the query rows alone (ratio 0), the engine's layer pass sends the gate/up projection
    and the lm_head of the 7B architecture to tread_rows_gemm, and the rest to cuBLAS; the logits
    match the same request with every projection on cuBLAS."""
    import torch.nn.functional as F

    from tread_b200 import BlockStore, Engine
    from tread_b200.configs import random_model, random_tokens

    if torch.cuda.get_device_properties(0).multi_processor_count * 256 > 37888:
        pytest.skip("the 7B gate/up weight fills every SM without a K split only up to 148 SMs")
    model = random_model("qwen2.5-7b", dtype=torch.bfloat16, device=DEV, layers=2, init_on_device=True)
    V = model.config.vocab_size
    g = torch.Generator().manual_seed(7)
    prefix, query = random_tokens(64, V, g), random_tokens(16, V, g)
    docs = [random_tokens(200, V, g) for _ in range(3)]
    eng = Engine(model, BlockStore(8 << 30))
    eng.prefill(prefix, docs, query)  # cold: fills the store
    calls = []
    orig = kernels.rows_gemm

    def spy(x, w, *a, **kw):
        calls.append(tuple(w.shape))
        return orig(x, w, *a, **kw)

    monkeypatch.setattr(kernels, "rows_gemm", spy)
    logits, _, st = eng.prefill(prefix, docs[::-1], query)
    assert st.hits == 4 and st.misses == 0
    assert sorted(calls) == sorted([(2 * 18944, 3584)] * 2 + [(V, 3584)])  # gate/up of both layers, lm_head
    monkeypatch.setattr(kernels, "rows_gemm_streams_alone", lambda w: False)  # every projection on cuBLAS
    calls.clear()
    ref, _, _ = eng.prefill(prefix, docs[::-1], query)
    assert calls == []
    kl = F.kl_div(F.log_softmax(ref.float(), -1), F.log_softmax(logits.float(), -1), log_target=True,
                  reduction="sum")
    assert float(kl) < 1e-3


def test_rows_gemm_refuses_operands_off_the_device():
    """A weight, bias or output that is not on x's device is refused before anything launches."""
    x, w, b, o = _case(4, 256, 64, torch.bfloat16, 5)
    with pytest.raises(ValueError):
        kernels.rows_gemm(x, w.cpu())
    with pytest.raises(ValueError):
        kernels.rows_gemm(x, w, bias=b.cpu())
    with pytest.raises(ValueError):
        kernels.rows_gemm(x, w, out=o.cpu())
    assert not kernels.rows_gemm_fits(x, w.cpu())
