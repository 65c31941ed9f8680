"""Page bookkeeping of the paged K/V pool on the CPU (models/kvpool.py): growth by whole pages, shared page lists
returned once, pages of a failed request returned by owner, exhaustion refused before anything is taken."""
import types

import pytest
import torch

from ridgefill_data_b200.models.kvpool import KVPool, PoolExhausted


def _model():
    return types.SimpleNamespace(head_dim=128, n_kv=2, layer_types=["gdn", "attn", "gdn", "attn"],
                                 device=torch.device("cpu"), dtype=torch.bfloat16)


def test_growth_release_and_owners():
    pool = KVPool(_model(), pages=6, page_size=128)
    assert pool.layers == [1, 3] and pool.k[1].shape == (6, 2, 128, 128)
    a = [{}, {}, {}, {}]
    pool.owner = "a"
    pool.grow(1, a[1], 130, "cpu")
    assert len(a[1]["pages"]) == 2 and a[1]["pages_dev"].dtype == torch.int32
    pool.grow(1, a[1], 256, "cpu")                     # still 2 pages
    assert len(a[1]["pages"]) == 2
    shared = [dict(e) for e in a]                      # finish() copies entries: the page list is shared
    pool.release(a)
    pool.release(shared)                               # returned once
    assert pool.free_pages(1) == 6
    pool.owner = "b"
    b = [{}, {}, {}, {}]
    pool.grow(3, b[3], 600, "cpu")
    assert pool.free_pages(3) == 1
    with pytest.raises(PoolExhausted):
        pool.grow(3, {}, 300, "cpu")
    assert pool.free_pages(3) == 1                     # nothing taken by the refused request
    pool.release_owner("b")                            # the failed request's pages come back
    assert pool.free_pages(3) == 6


def test_page_size_and_head_dim_checked():
    with pytest.raises(ValueError):
        KVPool(_model(), pages=4, page_size=100)
    m = _model()
    m.head_dim = 64
    with pytest.raises(ValueError):
        KVPool(m, pages=4)
