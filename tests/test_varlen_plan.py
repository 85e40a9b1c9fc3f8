"""Host planning of packed varlen passes (pure CPU logic)."""

import numpy as np
import pytest

from memforge_b200.varlen_plan import group_by_sequence, plan_varlen


def tables(*lens, bs=4):
    out, nxt = [], 0
    for n in lens:
        k = (n + bs - 1) // bs
        out.append(np.arange(nxt, nxt + k))
        nxt += k
    return out


def test_group_by_sequence_order():
    assert group_by_sequence([2, 0, 2, 1, 0]) == [(2, [0, 2]), (0, [1, 4]), (1, [3])]


def test_contiguous_chunk_is_one_segment_with_identity_map():
    p = plan_varlen(5, tables(12), [0] * 5, [7, 8, 9, 10, 11], 4, 4, 2)
    assert p.num_segments == 1
    assert p.cu_seqlens.tolist() == [0, 5]
    assert p.kv_lens.tolist() == [12]
    assert p.row_map is None and p.max_q_len == 5


def test_interleaved_packing_gets_a_row_map():
    p = plan_varlen(4, tables(11, 6, 20), [1, 0, 2, 0], [5, 9, 19, 10], 4, 8, 2)
    # sequence 1 first (first seen), then 0 (rows 1 and 3), then 2
    assert p.row_map.tolist() == [0, 1, 3, 2]
    assert p.kv_lens.tolist() == [6, 11, 20]
    assert p.cu_seqlens.tolist() == [0, 1, 3, 4]


def test_non_consecutive_positions_split_into_segments():
    p = plan_varlen(4, tables(20), [0, 0, 0, 0], [3, 4, 9, 10], 4, 4, 4)
    assert p.cu_seqlens.tolist() == [0, 2, 4]
    assert p.kv_lens.tolist() == [5, 11]


def test_reference_validation_messages():
    t = tables(8)
    with pytest.raises(ValueError, match="query tokens but"):
        plan_varlen(3, t, [0, 0], [5, 6, 7], 4, 4, 2)
    with pytest.raises(ValueError, match="at least one query token"):
        plan_varlen(0, t, [], [], 4, 4, 2)
    with pytest.raises(ValueError, match="negative query position"):
        plan_varlen(2, t, [0, 0], [3, -1], 4, 4, 2)
    with pytest.raises(IndexError, match="no block table"):
        plan_varlen(2, t, [0, 3], [3, 3], 4, 4, 2)
    with pytest.raises(IndexError, match="block table has"):
        plan_varlen(1, t, [0], [40], 4, 4, 2)
    with pytest.raises(ValueError, match="not a multiple of"):
        plan_varlen(1, t, [0], [7], 4, 4, 3)


def test_packed_buffer_round_trip():
    t = tables(11, 6, 20)
    p = plan_varlen(4, t, [1, 0, 2, 0], [5, 9, 19, 10], 4, 8, 2)
    buf, offs = p.packed(t)
    host = p.host_tables(t)
    o, n = offs["tables"]
    assert np.array_equal(buf[o:o + n].reshape(host.shape), host)
    o, n = offs["row_map"]
    assert np.array_equal(buf[o:o + n], p.row_map)


def test_segment_tables_hold_each_sequences_needed_prefix():
    t = tables(11, 6, 20)
    p = plan_varlen(4, t, [1, 0, 2, 0], [5, 9, 19, 10], 4, 8, 2)
    host = p.host_tables(t)
    # segments: seq 1 (6 keys, 2 blocks), seq 0 (11 keys, 3 blocks), seq 2 (20 keys, 5 blocks)
    assert p.seg_seq.tolist() == [1, 0, 2]
    assert p.needed.tolist() == [2, 3, 5]
    assert host.shape == (3, 5)
    for i, (sq, n) in enumerate(zip(p.seg_seq, p.needed)):
        assert host[i, :n].tolist() == t[sq][:n].tolist()
        assert (host[i, n:] == 0).all()


def test_planning_reads_table_lengths_only():
    """Tables whose contents cannot be read on the host (only sizes) still plan."""
    class SizedOnly:
        def __init__(self, n):
            self.n = n

        def numel(self):
            return self.n
    p = plan_varlen(3, [SizedOnly(3), SizedOnly(5)], [1, 1, 0], [8, 9, 2], 4, 4, 2)
    assert p.kv_lens.tolist() == [10, 3] and p.needed.tolist() == [3, 1]


def test_uniform_runs_in_order_pass_as_q_per_seq():
    """Equal runs already in segment order (a speculative verify pass): the
    plan reports the common length, so the call needs no per-segment offsets."""
    t = tables(20, 30, 12)
    p = plan_varlen(9, t, [0, 0, 0, 1, 1, 1, 2, 2, 2],
                    [17, 18, 19, 27, 28, 29, 9, 10, 11], 4, 8, 2)
    assert p.row_map is None and p.cu_seqlens.tolist() == [0, 3, 6, 9]
    assert p.uniform_q == 3
    # unequal runs, or rows that need a map, keep the varlen form
    assert plan_varlen(4, tables(20), [0, 0, 0, 0], [3, 4, 9, 10], 4, 4, 4).uniform_q == 2
    assert plan_varlen(3, tables(20, 12), [0, 0, 1], [8, 9, 11], 4, 4, 2).uniform_q == 0
    assert plan_varlen(4, tables(11, 6, 20), [1, 0, 2, 0], [5, 9, 19, 10], 4, 8, 2).uniform_q == 0
