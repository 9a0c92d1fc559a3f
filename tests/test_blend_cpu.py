"""Host-side pieces of blend.py that need no GPU: the DynamicCache handed back to callers holds
the request cache's own per-layer views (no copy) and decodes (appends) as HF's does."""
import torch

from tread_b200.blend import to_cache


def test_to_cache_holds_views_and_appends():
    K = torch.randn(3, 1, 2, 10, 8)
    V = torch.randn(3, 1, 2, 10, 8)
    Kl, Vl = list(K.unbind(0)), list(V.unbind(0))
    c = to_cache(Kl, Vl)
    assert len(c.layers) == 3 and c.get_seq_length() == 10
    for l in range(3):
        assert c.layers[l].keys.data_ptr() == Kl[l].data_ptr()  # no copy
        assert torch.equal(c.layers[l].values, Vl[l])
    k_new, v_new = torch.randn(1, 2, 1, 8), torch.randn(1, 2, 1, 8)
    k_all, v_all = c.update(k_new, v_new, 1)
    assert k_all.shape == (1, 2, 11, 8) and torch.equal(k_all[..., :10, :], Kl[1])
    assert torch.equal(v_all[..., 10:, :], v_new) and c.get_seq_length(1) == 11
