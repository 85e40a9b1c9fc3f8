"""
Host-side behaviour of the transformers caches (no GPU): construction as a
``transformers.Cache``, cursor semantics (``rollback`` moves only the cursor,
``seed_position`` declares a cached prefix, ``get_mask_sizes``), the packed
cache's slot arithmetic and the reference's validation errors
(``memforge_ml/runtime/paged_cache.py``, ``varlen_cache.py``).
"""

import pytest
import torch

pytest.importorskip("transformers")

from memforge_b200.kv_pool import ModelKVSpec, PagedKVPool  # noqa: E402
from memforge_b200.paged_cache import PagedCache, VarlenPackedCache  # noqa: E402


def pool(layers=3, block=4):
    return PagedKVPool(ModelKVSpec(layers, 2, 16, torch.float32, "cpu"), 32, block_size=block)


def test_paged_cache_is_a_transformers_cache_with_one_layer_per_model_layer():
    from transformers.cache_utils import Cache
    c = PagedCache(pool(), [3, 1, 2])
    assert isinstance(c, Cache) and len(c.layers) == 3
    assert c.position == 0 and c.get_seq_length() == 0
    assert c.block_table == [3, 1, 2]


def test_rollback_and_seed_position_move_every_layer_cursor():
    c = PagedCache(pool(), list(range(8)))
    c.seed_position(10)
    assert [l.position for l in c.layers] == [10, 10, 10]
    assert c.layers[0].get_mask_sizes(3) == (13, 0)
    c.rollback(4)
    assert c.position == 6
    c.rollback(0)
    assert c.position == 6
    with pytest.raises(ValueError, match="non-negative"):
        c.seed_position(-1)


def test_flat_indices_follow_the_block_table_and_are_memoised_per_step():
    c = PagedCache(pool(), [5, 0, 7])
    idx = c.flat_indices(2, 9)
    assert idx.tolist() == [22, 23, 0, 1, 2, 3, 28]
    assert c.flat_indices(2, 9) is idx
    c.begin_step([5, 0, 7])
    assert c.flat_indices(2, 9) is not idx
    with pytest.raises(IndexError, match="outside a block table"):
        c.flat_indices(0, 13)


def test_decode_mirror_is_not_part_of_this_build():
    with pytest.raises(ValueError, match="mutually exclusive"):
        PagedCache(pool(), [1], view_capacity=64, lazy_read=True)
    with pytest.raises(NotImplementedError):
        PagedCache(pool(), [1], view_capacity=64)


def test_packed_cache_slots_and_validation():
    p = pool()
    tables = [torch.tensor([3, 1]), torch.tensor([5, 0, 2])]
    c = VarlenPackedCache(p, 3, tables, [0, 0, 1, 1], [0, 5, 2, 9])
    assert c.write_index.tolist() == [12, 5, 22, 9]
    assert c.get_seq_length() == 0 and len(c) == 3
    with pytest.raises(IndexError, match="no block table"):
        VarlenPackedCache(p, 3, tables, [2], [0])
    with pytest.raises(IndexError, match="needs logical block"):
        VarlenPackedCache(p, 3, tables, [0], [8])
    with pytest.raises(ValueError, match="same pool slot"):
        VarlenPackedCache(p, 3, tables, [0, 0], [1, 1])
    with pytest.raises(ValueError, match="same pool slot"):
        # two sequences whose tables share block 3
        VarlenPackedCache(p, 3, [torch.tensor([3]), torch.tensor([3])], [0, 1], [1, 1])
    with pytest.raises(NotImplementedError):
        c.layers[0].crop(1)
