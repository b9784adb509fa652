"""Host-side scheduler logic vs the reference's own batch schedulers.

The reference's `generate_wavefront_batch` / `ar_generate_batch` /
`generate_dtv_batch` (scheduler_batch.py:185-501) were run on a deterministic stand-in for the model
blocks (golden_inputs.FakeBlocks); tests/golden/reference_scheduler.json holds
their committed tokens, every per-sequence and batch counter and the rollback
calls.  The restated scheduler must reproduce all of it exactly, and the
invariants the reference's gates check (experiments/exp4_emu/verify_step1.py:74-82,
verify_batch.py:127-164) must hold.
"""
from __future__ import annotations

import json
import pathlib

import pytest

import golden_inputs as gi

GOLD = json.loads((pathlib.Path(__file__).parent / "golden" / "reference_scheduler.json").read_text())


def _sched():
    from wavefront_decoding_b200 import scheduler
    return scheduler


@pytest.mark.parametrize("case", gi.SCHED_CASES, ids=[c["name"] for c in gi.SCHED_CASES])
def test_wfd_matches_reference_trace(case):
    sch = _sched()
    blocks = gi.FakeBlocks(case["T_total"])
    emus = None
    if case["alpha"] is not None:
        emus = [sch.EmulatedAcceptance(case["alpha"], seed=100 + b) for b in range(case["B"])]
    bt = sch.generate_wavefront_batch(blocks, gi.sched_prompts(case), case["new"],
                                      sch.SsdPolicy(T_total=case["T_total"], T_draft=case["T_draft"]), emus)
    assert gi.trace_summary(bt, blocks.last_cache) == GOLD[case["name"]]


@pytest.mark.parametrize("case", gi.DTV_CASES, ids=[c["name"] for c in gi.DTV_CASES])
def test_dtv_matches_reference_trace(case):
    """Draft-then-verify (scheduler_batch.py:378-501): tokens, counters, union
    sizes and rollback calls of the reference's own run."""
    sch = _sched()
    blocks = gi.FakeBlocks(case["T_total"])
    emus = None
    if case["alpha"] is not None:
        emus = [sch.EmulatedAcceptance(case["alpha"], seed=200 + b) for b in range(case["B"])]
    bt = sch.generate_dtv_batch(blocks, gi.sched_prompts(case), case["new"],
                                sch.SsdPolicy(T_total=case["T_total"], T_draft=case["T_draft"]), case["K"], emus)
    assert gi.trace_summary(bt, blocks.last_cache) == GOLD[case["name"]]


def test_dtv_greedy_is_lossless():
    """Greedy DtV commits the AR tokens (every committed token is a full-depth id)."""
    sch = _sched()
    prompts = gi.sched_prompts(gi.SCHED_CASES[0])
    ar = sch.ar_generate_batch(gi.FakeBlocks(4), prompts, 20)
    for K in (1, 3, 6):
        bt = sch.generate_dtv_batch(gi.FakeBlocks(4), prompts, 20, sch.SsdPolicy(4, 2), K)
        assert [t.tokens for t in bt.per_seq] == [t.tokens for t in ar.per_seq]


def test_ar_matches_reference_trace():
    sch = _sched()
    blocks = gi.FakeBlocks(4)
    bt = sch.ar_generate_batch(blocks, gi.sched_prompts(gi.SCHED_CASES[0]), 12)
    assert gi.trace_summary(bt, blocks.last_cache) == GOLD["ar_T4"]


def test_alpha_one_commits_every_draft():
    """verify_step1.py:74-82: alpha = 1 gives zero rejects and exactly N commits."""
    sch = _sched()
    N = 30
    blocks = gi.FakeBlocks(8)
    emus = [sch.EmulatedAcceptance(1.0, seed=b) for b in range(3)]
    bt = sch.generate_wavefront_batch(blocks, gi.sched_prompts(gi.SCHED_CASES[0]), N, sch.SsdPolicy(8, 2), emus)
    for t in bt.per_seq:
        assert t.n_drafts_rejected == 0 and len(t.tokens) == N
    assert blocks.last_cache.drops == []


def test_ar_r_calls():
    """verify_batch.py:160-164: AR r_calls = (N - 1) * T_total per sequence."""
    sch = _sched()
    N, T = 9, 5
    bt = sch.ar_generate_batch(gi.FakeBlocks(T), gi.sched_prompts(gi.SCHED_CASES[1]), N)
    for t in bt.per_seq:
        assert t.n_r_calls == (N - 1) * T


def test_cross_sequence_isolation():
    """verify_batch.py:127-141: a sequence's committed stream does not depend on
    what its batch neighbours accept or reject."""
    sch = _sched()
    pol = sch.SsdPolicy(4, 1)
    prompts = gi.sched_prompts(gi.SCHED_CASES[0])
    runs = []
    for alphas in ([1.0, 0.0, 1.0], [1.0, 1.0, 0.0]):
        emus = [sch.EmulatedAcceptance(a, seed=7 + b) for b, a in enumerate(alphas)]
        runs.append(sch.generate_wavefront_batch(gi.FakeBlocks(4), prompts, 20, pol, emus))
    assert runs[0].per_seq[0].tokens == runs[1].per_seq[0].tokens


def test_greedy_wfd_equals_sequential_tokens():
    """Lossless WFD: with the real gold == draft comparison the committed tokens
    equal plain sequential loop decoding for every T_draft."""
    sch = _sched()
    prompts = gi.sched_prompts(gi.SCHED_CASES[0])
    ar = sch.ar_generate_batch(gi.FakeBlocks(4), prompts, 20)
    for d in (1, 2, 4):
        wfd = sch.generate_wavefront_batch(gi.FakeBlocks(4), prompts, 20, sch.SsdPolicy(4, d), None)
        assert [t.tokens for t in wfd.per_seq] == [t.tokens for t in ar.per_seq]
