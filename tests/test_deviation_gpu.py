"""Parity of the fused deviation + top-k selector (tread_deviation_topk) with the CPU oracle
(bit-exact dev and selection) and with the reference's own selection (golden)."""
import numpy as np
import pytest
import torch

from conftest import golden
from oracle import oracle as orc
from tread_b200 import kernels

pytestmark = pytest.mark.gpu


def bits(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def host(t):
    return bits(t) if t.dtype == torch.bfloat16 else t.detach().cpu().contiguous().numpy()


def test_golden_selection_matches_reference(cuda):
    g = golden("deviation.npz")
    k1, v1, K1g, V1g, all_c = g["k1"], g["v1"], g["K1"], g["V1"], g["all_c"]
    H, n, D = k1.shape
    T = int(all_c.max()) + 11
    rng = np.random.default_rng(0)
    K1 = rng.standard_normal((H, T, D)).astype(np.float32)
    V1 = rng.standard_normal((H, T, D)).astype(np.float32)
    K1[:, all_c] = K1g
    V1[:, all_c] = V1g
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
    budget = int(g["budget"])
    dev, sel, pos = kernels.deviation_topk(t(k1), t(v1), t(K1), t(V1), t(all_c.astype(np.int64)), budget)
    ref_dev = orc.deviation(k1, v1, K1, V1, all_c)
    np.testing.assert_array_equal(dev.cpu().numpy(), ref_dev)
    np.testing.assert_allclose(dev.cpu().numpy(), g["dev"], rtol=2e-6)
    np.testing.assert_array_equal(sel.cpu().numpy(), np.sort(g["topk"]))
    np.testing.assert_array_equal(pos.cpu().numpy(), g["S"])


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
# more than 8192 candidates take the selector's second path (keys re-read from L2, 8-bit radix)
@pytest.mark.parametrize("H,D,n,T", [(4, 128, 8192, 8192), (2, 64, 1000, 1032), (4, 128, 777, 4000),
                                     (8, 128, 100, 300), (1, 256, 33, 40), (2, 128, 20000, 21000),
                                     (4, 64, 9000, 9100)])
def test_random_matches_oracle_bit_exact(cuda, dtype, H, D, n, T):
    gen = torch.Generator(device=cuda).manual_seed(H * 1000 + n)
    K1 = torch.randn(H, T, D, device=cuda, generator=gen).to(dtype)
    V1 = torch.randn(H, T, D, device=cuda, generator=gen).to(dtype)
    pos = torch.sort(torch.randperm(T, device=cuda, generator=gen)[:n]).values
    # fresh rows from a packed projection output [n, (Hq + 2H) * D]: strided [H, n, D] views
    Hq = 3 * H
    qkv = torch.randn(n, (Hq + 2 * H) * D, device=cuda, generator=gen).to(dtype)
    k1 = qkv[:, Hq * D:(Hq + H) * D].view(n, H, D).transpose(0, 1)
    v1 = qkv[:, (Hq + H) * D:].view(n, H, D).transpose(0, 1)
    # make part of the candidates exactly equal to the cache -> dev == 0 ties
    tie = torch.arange(0, n, 7, device=cuda)
    k1[:, tie] = K1[:, pos[tie]]
    v1[:, tie] = V1[:, pos[tie]]
    ref_dev = orc.deviation(host(k1), host(v1), host(K1), host(V1), pos.cpu().numpy())
    for budget in sorted({0, 1, orc.budget_for(0.2, n), n - len(tie) // 2, n}):
        dev, sel, spos = kernels.deviation_topk(k1, v1, K1, V1, pos, budget)
        np.testing.assert_array_equal(dev.cpu().numpy(), ref_dev)
        ref_sel = orc.select_topk(ref_dev, budget)
        np.testing.assert_array_equal(sel.cpu().numpy(), ref_sel)
        np.testing.assert_array_equal(spos.cpu().numpy(), pos.cpu().numpy()[ref_sel])


def test_repeated_calls_share_workspace(cuda):
    gen = torch.Generator(device=cuda).manual_seed(3)
    H, D, n, T = 4, 128, 2048, 2048
    K1 = torch.randn(H, T, D, device=cuda, generator=gen, dtype=torch.float32).to(torch.bfloat16)
    V1 = torch.randn(H, T, D, device=cuda, generator=gen, dtype=torch.float32).to(torch.bfloat16)
    k1 = torch.randn(H, n, D, device=cuda, generator=gen, dtype=torch.float32).to(torch.bfloat16)
    v1 = torch.randn(H, n, D, device=cuda, generator=gen, dtype=torch.float32).to(torch.bfloat16)
    pos = torch.arange(n, device=cuda)
    ws = torch.zeros(64, dtype=torch.int32, device=cuda)
    outs = [kernels.deviation_topk(k1, v1, K1, V1, pos, 409, ws=ws)[1].clone() for _ in range(5)]
    torch.cuda.synchronize()
    for o in outs[1:]:
        assert torch.equal(o, outs[0])
    assert ws[0].item() == 0 and ws[1].item() == 0


def test_out_of_range_position_sets_flag(cuda):
    H, D, n, T = 2, 64, 64, 64
    K1 = torch.zeros(H, T, D, device=cuda)
    k1 = torch.ones(H, n, D, device=cuda)
    pos = torch.arange(n, device=cuda)
    pos[5] = T + 3  # the kernel's bounds check skips the row, flags it and reports NaN
    ws = torch.zeros(64, dtype=torch.int32, device=cuda)
    dev, sel, _ = kernels.deviation_topk(k1, k1, K1, K1, pos, 3, ws=ws)
    torch.cuda.synchronize()
    assert ws[1].item() == 1 and torch.isnan(dev[5])
    assert sel.tolist() == [5, 0, 1] or sorted(sel.tolist()) == [0, 1, 5]


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("world", [1, 2, 4])
def test_split_selector_matches_fused(cuda, dtype, world):
    """KV-head tensor-parallel selector: per-head norms of each rank's head slice (bit-exact vs
    the oracle), concatenated in rank order, then the fixed-order head sum + top-k: dev and
    selection equal the single-GPU fused kernel's bit for bit (ranks emulated on one GPU)."""
    g = torch.Generator().manual_seed(7 + world)
    H, n, T, D = 4, 3001, 4100, 128
    k1 = torch.randn(H, n, D, generator=g).to(dtype)
    v1 = torch.randn(H, n, D, generator=g).to(dtype)
    K1 = torch.randn(H, T, D, generator=g).to(dtype)
    V1 = torch.randn(H, T, D, generator=g).to(dtype)
    pos = torch.randperm(T, generator=g)[:n].sort().values
    # plant exact ties across the cut: duplicate some candidates' rows onto others
    K1[:, pos[100:140]] = K1[:, pos[0:40]]
    V1[:, pos[100:140]] = V1[:, pos[0:40]]
    k1[:, 100:140] = k1[:, 0:40]
    v1[:, 100:140] = v1[:, 0:40]
    d = [x.to(cuda) for x in (k1, v1, K1, V1, pos)]
    budget = orc.budget_for(0.2, n)
    dev_f, sel_f, pos_f = kernels.deviation_topk(*d, budget)
    parts = []
    per = H // world
    for r in range(world):
        s = slice(r * per, (r + 1) * per)
        parts.append(kernels.deviation_head_norms(d[0][s], d[1][s], d[2][s], d[3][s], d[4]))
    norms = torch.cat(parts, dim=1)
    ref_norms = orc.head_norms(host(k1), host(v1), host(K1), host(V1), pos.numpy())
    np.testing.assert_array_equal(norms.cpu().numpy(), ref_norms)
    dev_s, sel_s, pos_s = kernels.select_head_norms(norms, d[4], budget)
    np.testing.assert_array_equal(dev_s.cpu().numpy(), dev_f.cpu().numpy())
    np.testing.assert_array_equal(dev_s.cpu().numpy(), orc.dev_from_head_norms(ref_norms))
    np.testing.assert_array_equal(sel_s.cpu().numpy(), sel_f.cpu().numpy())
    np.testing.assert_array_equal(pos_s.cpu().numpy(), pos_f.cpu().numpy())


def test_split_selector_edge_cases(cuda):
    """n = 0, budget 0 and budget n through the split selector."""
    H, D = 2, 64
    e = torch.empty(H, 0, D, device=cuda)
    K = torch.randn(H, 16, D, device=cuda)
    z = torch.empty(0, dtype=torch.int64, device=cuda)
    assert kernels.deviation_head_norms(e, e, K, K, z).shape == (2, H, 0)
    k1 = torch.randn(H, 9, D, device=cuda)
    pos = torch.arange(9, device=cuda)
    norms = kernels.deviation_head_norms(k1, k1, K, K, pos)
    dev, sel, _ = kernels.select_head_norms(norms, pos, 0)
    assert sel.numel() == 0 and dev.shape == (9,)
    _, sel, p = kernels.select_head_norms(norms, pos, 9)
    np.testing.assert_array_equal(sel.cpu().numpy(), np.arange(9))
