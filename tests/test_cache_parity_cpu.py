"""The paged KV cache keeps the reference's API (tinytron/inference/cache.py): appends of
[B, H, T, D] chunks return the previous length, ``get_kv`` returns the [B, H, L, D]
prefix, and an append past ``max_seq_len`` raises the same error.  Here the pages come
from a shared pool through a page table; the contents must match the reference's flat
buffer exactly, across page boundaries.  Skipped when the reference is not installed."""
import pytest
import torch

from ref_oracle import available, cpu_reference

pytestmark = pytest.mark.skipif(not available(), reason="reference not installed under baseline/_ref")


@pytest.mark.parametrize("page_size", [1, 4, 16, 64])
def test_layer_cache_matches_reference(page_size):
    with cpu_reference():
        from tinytron.inference.cache import LayerPagedKVCache as RefCache
    from tinytron_b200.inference.cache import LayerPagedKVCache

    B, H, D, L = 3, 2, 8, 40
    kw = dict(batch_size=B, num_heads=H, head_dim=D, max_seq_len=L, page_size=page_size, device="cpu",
              dtype=torch.float32)
    ref, ours = RefCache(**kw), LayerPagedKVCache(**kw)
    g = torch.Generator().manual_seed(page_size)
    for T in (5, 1, 1, 13, 7, 1, 12):  # 40 positions in total, crossing page boundaries
        k = torch.randn(B, H, T, D, generator=g)
        v = torch.randn(B, H, T, D, generator=g)
        assert ours.append(k, v) == ref.append(k, v)
        assert ours.current_length == ref.current_length
        (rk, rv), (ok, ov) = ref.get_kv(), ours.get_kv()
        assert ok.shape == rk.shape and torch.equal(ok, rk) and torch.equal(ov, rv)
    extra = torch.zeros(B, H, 1, D)
    with pytest.raises(ValueError, match="KV cache overflow"):
        ref.append(extra, extra)
    with pytest.raises(ValueError, match="KV cache overflow"):
        ours.append(extra, extra)


def test_reset_returns_every_page_and_length():
    from tinytron_b200.inference.cache import LayerPagedKVCache

    c = LayerPagedKVCache(2, 1, 4, 16, 4, "cpu", torch.float32)
    c.append(torch.ones(2, 1, 9, 4), torch.ones(2, 1, 9, 4))
    assert (c.page_table >= 0).sum().item() == 2 * 3 and c.seq_lens == [9, 9]
    c.reset()
    assert c.current_length == 0 and c.seq_lens == [0, 0] and int(c.len_dev.item()) == 0
    assert (c.page_table < 0).all() and len(c._free) == c.k_pages.size(0)
    c.append(torch.full((2, 1, 16, 4), 2.0), torch.full((2, 1, 16, 4), 3.0))  # the whole pool again
    k, v = c.get_kv()
    assert torch.equal(k, torch.full((2, 1, 16, 4), 2.0)) and torch.equal(v, torch.full((2, 1, 16, 4), 3.0))
