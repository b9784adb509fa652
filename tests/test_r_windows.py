"""R-union attention windows (CPU): rows of one sequence on one depth slot are
grouped into bottom-right-causal windows over runs of consecutive positions
(the reference's R grouping, ouro_blocks_batch.py:184-205); the device pre-tick
kernel applies the same rule (checked on the GPU through the KV-sharing and
draft-then-verify tests)."""
from __future__ import annotations


def _windows(*a):
    from wavefront_decoding_b200.engine import r_windows
    return r_windows(*a)


def test_distinct_slots_keep_order_and_single_rows():
    # lossless WFD: every token of a sequence on its own depth slot
    order, runs = _windows([0, 1, 0, 1], [0, 0, 2, 2], [10, 7, 9, 6])
    assert order is None and runs == [1, 1, 1, 1]


def test_shared_slot_contiguous_run():
    # KV sharing s = 1: three tokens of sequence 0 at positions 12, 10, 11 on one slot
    order, runs = _windows([0, 1, 0, 0], [0, 0, 0, 0], [12, 5, 10, 11])
    assert order == [2, 3, 0, 1]
    assert runs == [3, 0, 0, 1]


def test_gaps_split_runs():
    # s = 2: alternate depths share a slot -> positions 4 and 6 are not one window
    order, runs = _windows([0, 0, 0, 0], [0, 2, 0, 2], [4, 5, 6, 7])
    assert order == [0, 2, 1, 3]
    assert runs == [1, 1, 1, 1]


def test_dtv_verify_sources():
    # draft-then-verify: K + 1 = 4 sources of sequence 1 at one depth, one draft row of sequence 0
    order, runs = _windows([1, 1, 1, 1, 0], [4, 4, 4, 4, 2], [20, 21, 22, 23, 9])
    assert order == [4, 0, 1, 2, 3]
    assert runs == [1, 4, 0, 0, 0]


def test_empty():
    assert _windows([], [], []) == (None, [])


def test_gap_mode_groups_a_slot_whatever_the_gaps():
    # s = 2 with gapped windows: positions 4, 6 (slot 0) and 5, 7 (slot 2) are two windows of two rows
    order, runs = _windows([0, 0, 0, 0], [0, 2, 0, 2], [4, 5, 6, 7], True)
    assert order == [0, 2, 1, 3]
    assert runs == [2, 0, 2, 0]
    # irregular gaps (after a rejection) and a second sequence
    order, runs = _windows([3, 3, 1, 3], [0, 0, 0, 0], [20, 11, 9, 15], True)
    assert order == [2, 1, 3, 0]
    assert runs == [1, 3, 0, 0]
