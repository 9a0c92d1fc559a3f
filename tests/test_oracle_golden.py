"""Pin the CPU oracle against golden vectors produced by the reference itself.

Fixtures come from tests/golden/make_golden.py, which runs the unmodified tread sources.
"""
import numpy as np
import pytest

from conftest import golden
from oracle import oracle as orc


@pytest.fixture(scope="module")
def rope():
    return golden("rope.npz")


@pytest.mark.parametrize("D", [64, 128])
def test_oracle_cos_sin_matches_hf_rotary(rope, D):
    inv = rope[f"d{D}_inv_freq"]
    np.testing.assert_array_equal(inv, orc.inv_freq(D, 1e6))
    for d in rope["deltas"]:
        c, s = orc.rope_cos_sin(int(d), inv)
        half = D // 2
        # HF returns cat(freqs, freqs): both halves carry the same cos/sin.
        ref_c, ref_s = rope[f"d{D}_cos_{d}"], rope[f"d{D}_sin_{d}"]
        np.testing.assert_array_equal(ref_c[:half], ref_c[half:])
        np.testing.assert_allclose(c, ref_c[:half], rtol=0, atol=2e-7)
        np.testing.assert_allclose(s, ref_s[:half], rtol=0, atol=2e-7)


@pytest.mark.parametrize("D", [64, 128])
def test_oracle_rotation_matches_reference_rotate_keys(rope, D):
    kb = rope[f"d{D}_k_bf16"]  # [2,1,2,21,D] bf16 bits
    inv = rope[f"d{D}_inv_freq"]
    n = kb.shape[-2]
    for d in rope["deltas"]:
        ref = rope[f"d{D}_rot_{d}"]
        ok, ov = orc.rope_gather_append([(kb, kb, int(d), 0)], n, inv, out_dtype=orc.F32)
        # fp32 rotation of the same bf16 inputs: differences are cos/sin last-bit effects only
        np.testing.assert_allclose(ok, ref, rtol=0, atol=3e-6 * float(np.abs(ref).max() + 1))
        np.testing.assert_array_equal(ov, orc.bf16_to_f32(kb))
        if d == 0:
            np.testing.assert_array_equal(ok, orc.bf16_to_f32(kb))
        # bf16 output is the RNE rounding of the fp32 result
        okb, _ = orc.rope_gather_append([(kb, kb, int(d), 0)], n, inv)
        diff = np.abs(orc.bf16_to_f32(okb) - ref)
        assert (diff <= orc.bf16_ulp(ref) * 0.5 + 1e-6 * np.abs(ref)).all()


def test_oracle_assembly_places_segments(rope):
    """torch.cat order and token offsets of tread/engine.py:108-120."""
    kb = rope["d64_k_bf16"]
    inv = rope["d64_inv_freq"]
    n = kb.shape[-2]
    segs = [(kb, kb, 0, 0), (kb, kb, 37, n), (kb, kb, -1, 2 * n)]
    ok, ov = orc.rope_gather_append(segs, 3 * n + 5, inv, out_dtype=orc.F32)
    np.testing.assert_allclose(ok[..., n:2 * n, :], rope["d64_rot_37"], atol=3e-6 * 8)
    np.testing.assert_allclose(ok[..., 2 * n:3 * n, :], rope["d64_rot_-1"], atol=3e-6 * 8)
    np.testing.assert_array_equal(ok[..., :n, :], orc.bf16_to_f32(kb))
    assert (ok[..., 3 * n:, :] == 0).all() and (ov[..., 3 * n:, :] == 0).all()


def test_oracle_deviation_matches_reference_layer1_deviation():
    """dev (tread/blend.py:129) restated in a fixed fp32 order agrees with the reference's torch
    reduction to rounding, and selects the same set as the reference's topk."""
    g = golden("deviation.npz")
    k1, v1, K1g, V1g = g["k1"], g["v1"], g["K1"], g["V1"]  # [H, n, D]; K1g/V1g gathered at all_c
    H, n, D = k1.shape
    dev = orc.deviation(k1, v1, K1g, V1g, np.arange(n))
    np.testing.assert_allclose(dev, g["dev"], rtol=2e-6, atol=0)
    budget = int(g["budget"])
    assert budget == orc.budget_for(0.2, n)
    sel = orc.select_topk(dev, budget)
    np.testing.assert_array_equal(sel, np.sort(g["topk"]))
    np.testing.assert_array_equal(g["all_c"][sel], g["S"])


def test_select_topk_tie_break_and_budget_rounding():
    dev = np.array([1.0, 3.0, 3.0, 2.0, 3.0, 0.5], np.float32)
    np.testing.assert_array_equal(orc.select_topk(dev, 2), [1, 2])
    np.testing.assert_array_equal(orc.select_topk(dev, 4), [1, 2, 3, 4])
    np.testing.assert_array_equal(orc.select_topk(dev, 6), np.arange(6))
    assert orc.budget_for(0.5, 5) == 2 and orc.budget_for(0.5, 7) == 4  # banker's rounding, as Python round
    assert orc.budget_for(0.2, 7936) == 1587 and orc.budget_for(0.2, 8192) == 1638
