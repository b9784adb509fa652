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
