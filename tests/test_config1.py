"""Config 1 (greedy end-to-end decoding of a random-init looped LM) pinned to
the reference.

tests/golden/reference_config1.json holds what the reference's own
`ParcaeBlocks` produced on the fixture model (tests/parcae_fixture.py; seed 0,
prompt of 128 ids from seed 0, T_total 4, SDPA backend, fp32): the AR tokens
(`ar_generate_parcae_blocks`, ar_baseline.py:132-193), the WFD tokens and
counters for T_draft 1, 2, 4 (`generate_wavefront_dynamic`, scheduler.py:89-225)
and every KV slot's final length.  Here (CPU): the fixture is rebuilt
identically, and the float64 full-recompute oracle reproduces the reference's
tokens.  The GPU engine is checked against the same file in
test_engine_gpu.py.
"""
from __future__ import annotations

import json
import pathlib

import torch

import parcae_fixture as pf

GOLD = json.loads((pathlib.Path(__file__).parent / "golden" / "reference_config1.json").read_text())


def test_fixture_and_prompt_reproduce():
    m = pf.ParcaeFixture(seed=0)
    assert pf.config1_prompt()[:8].tolist() == GOLD["prompt_head"]
    for a, b in zip(pf.weight_sums(m), GOLD["weight_sums"]):
        assert abs(a - b) <= 1e-9 * max(1.0, abs(b)), (a, b)


def test_reference_wfd_equals_ar():
    """The reference's own lossless claim on this fixture."""
    for d in (1, 2, 4):
        assert GOLD[f"wfd_d{d}"]["tokens"] == GOLD["ar"]["tokens"]
    assert GOLD["wfd_d1"]["n_drafts_rejected"] > 0        # the case exercises rollbacks


def test_oracle_matches_reference_tokens():
    from oracle import looped_lm as olm
    from wavefront_decoding_b200.looped_lm import LoopedLM
    m = pf.ParcaeFixture(seed=0)
    model = LoopedLM(pf.looped_config(m, GOLD["T_total"]), dtype=torch.float32, device="cpu")
    model.load_weights(pf.to_looped_weights(m))
    W, cfg = olm.weights_from(model)
    n = 8      # full recompute per token in float64: keep the CPU suite short
    assert olm.greedy_generate(W, cfg, pf.config1_prompt().tolist(), n) == GOLD["ar"]["tokens"][:n]


def test_kv_sharing_slot_map():
    """KV-sharing budget s: core depth r -> depth slot r % s, s depth slots allocated."""
    from wavefront_decoding_b200.looped_lm import LoopedLMConfig
    c = LoopedLMConfig(n_prelude=1, n_core=2, n_coda=1, T_total=4, kv_budget_s=2)
    assert c.n_depth_slots == 2 and c.n_slots == 6
    assert [c.slot_core(r, l) for r in range(4) for l in range(2)] == [1, 2, 3, 4, 1, 2, 3, 4]
    assert c.slot_coda(0) == 5
    for s in (0, 4, 9):        # off: one slot per depth
        c = LoopedLMConfig(n_prelude=1, n_core=2, n_coda=1, T_total=4, kv_budget_s=s)
        assert c.n_depth_slots == 4 and c.slot_core(3, 1) == 8 and c.slot_coda(0) == 9


def test_reference_kv_sharing_golden():
    """The reference's own results with kv_budget_s = 2 and 1: WFD commits AR's tokens
    on this fixture, the shared slots change the drafts (counters differ from the
    unshared run), and only the used slots exist (coda kept at its unshared index)."""
    for sb in (1, 2):
        for d in (1, 2):
            assert GOLD[f"wfd_d{d}_s{sb}"]["tokens"] == GOLD[f"ar_s{sb}"]["tokens"]
        assert (GOLD[f"wfd_d1_s{sb}"]["n_drafts_accepted"], GOLD[f"wfd_d2_s{sb}"]["n_drafts_accepted"]) != \
            (GOLD["wfd_d1"]["n_drafts_accepted"], GOLD["wfd_d2"]["n_drafts_accepted"])
    assert set(GOLD["ar_s2"]["seqlen"]) == {"0", "1", "2", "3", "4", "9"}
    assert set(GOLD["ar_s1"]["seqlen"]) == {"0", "1", "2", "9"}
