"""Seeded input recipes shared by tests/golden/make_golden.py and the tests.

All tensors come from torch CPU generators with fixed seeds, so the same
torch build regenerates them bit-for-bit; `checksum` lets a test prove it is
looking at the same data the golden file was made from.
"""
from __future__ import annotations

import numpy as np
import torch


def gen(seed: int) -> torch.Generator:
    return torch.Generator().manual_seed(seed)


def randn(shape, g, dtype=torch.float32) -> torch.Tensor:
    return torch.randn(shape, generator=g, dtype=torch.float32).to(dtype)


def checksum(*ts) -> list[float]:
    return [float(t.to(torch.float64).sum()) for t in ts] + [float(t.to(torch.float64).abs().sum()) for t in ts]


def _cu(lengths) -> torch.Tensor:
    return torch.tensor(np.concatenate([[0], np.cumsum(lengths)]), dtype=torch.int32)


VARLEN_CASES = [
    # wavefront decode: one query per segment, ragged prefixes, GQA 4:1
    dict(name="decode_gqa4_d64", seed=11, H=8, Hkv=2, Dh=64, q_lens=[1] * 6,
         k_lens=[37, 1, 200, 64, 129, 5], causal=False, dtype="f32"),
    dict(name="decode_gqa4_d128_bf16", seed=12, H=16, Hkv=4, Dh=128, q_lens=[1] * 5,
         k_lens=[300, 17, 256, 1, 95], causal=False, dtype="bf16"),
    # grouped / verify windows: bottom-right causal multi-row segments
    dict(name="window_causal_d128", seed=13, H=8, Hkv=2, Dh=128, q_lens=[8, 3, 1, 8],
         k_lens=[120, 3, 50, 8], causal=True, dtype="f32"),
    dict(name="window_causal_mha_d64_bf16", seed=14, H=4, Hkv=4, Dh=64, q_lens=[2, 5, 8],
         k_lens=[90, 40, 161], causal=True, dtype="bf16"),
    dict(name="mha_noncausal_multirow", seed=15, H=4, Hkv=4, Dh=64, q_lens=[3, 1, 4],
         k_lens=[10, 70, 33], causal=False, dtype="f32"),
]

Q1_PADDED_CASE = dict(name="q1_padded", seed=16, H=8, Hkv=2, Dh=128, q_lens=[1] * 4,
                      k_lens=[2, 77, 300, 31], causal=False, dtype="f32")

DENSE_CASES = [
    dict(name="causal_square", seed=21, B=2, Tq=33, Tk=33, H=4, Hkv=2, Dh=64, causal=True),
    dict(name="causal_bottom_right", seed=22, B=2, Tq=5, Tk=70, H=4, Hkv=2, Dh=64, causal=True),
    dict(name="single_query", seed=23, B=3, Tq=1, Tk=50, H=8, Hkv=2, Dh=128, causal=True),
    dict(name="noncausal", seed=24, B=1, Tq=6, Tk=40, H=4, Hkv=4, Dh=128, causal=False),
]

GATE1_LENGTHS = (600, 900, 1500, 2048)
KV_SCRIPT_GEOM = (3, 2, 64, 2, 64)  # n_slots, B, S, Hkv, Dh


def _dt(name: str) -> torch.dtype:
    return torch.bfloat16 if name == "bf16" else torch.float32


def varlen_inputs(case):
    g = gen(case["seed"])
    dt = _dt(case["dtype"])
    tq, tk = sum(case["q_lens"]), sum(case["k_lens"])
    q = randn((tq, case["H"], case["Dh"]), g, dt)
    k = randn((tk, case["Hkv"], case["Dh"]), g, dt)
    v = randn((tk, case["Hkv"], case["Dh"]), g, dt)
    return q, k, v, _cu(case["q_lens"]), _cu(case["k_lens"])


def dense_inputs(case):
    g = gen(case["seed"])
    q = randn((case["B"], case["Tq"], case["H"], case["Dh"]), g)
    k = randn((case["B"], case["Tk"], case["Hkv"], case["Dh"]), g)
    v = randn((case["B"], case["Tk"], case["Hkv"], case["Dh"]), g)
    return q, k, v


def cutoff_inputs():
    g = gen(31)
    qpos = [3, 17, 9, 40, 22]
    Tk = max(qpos) + 1
    q = randn((1, len(qpos), 8, 64), g)
    k = randn((1, Tk, 2, 64), g)
    v = randn((1, Tk, 2, 64), g)
    return q, k, v, qpos


def gate1_inputs():
    """exp5 gate 1 (verify_graph.py:45-56, 88-89): H = Hkv = 16, Dh = 128,
    MAX = 2048, one decode query and an 8-row causal window.  The reference
    draws on the GPU; here the same shapes come from CPU seed 0 (fp32)."""
    g = gen(0)
    H, Hkv, Dh, MAX = 16, 16, 128, 2048
    K = randn((MAX, Hkv, Dh), g)
    V = randn((MAX, Hkv, Dh), g)
    q1 = randn((1, H, Dh), g)
    q8 = randn((8, H, Dh), g)
    return K, V, q1, q8


def kv_script():
    """Operations replayed on BatchStaticKVCache (golden) and SlotKVCache (test)."""
    n_slots, B, S, Hkv, Dh = KV_SCRIPT_GEOM
    g = gen(41)
    ops = []
    L = 10
    for slot in range(n_slots):
        ops.append(("prefill", slot, randn((B, L, Hkv, Dh), g), randn((B, L, Hkv, Dh), g)))
    ops.append(("tokens", [0, 1, 2, 0], [0, 0, 1, 1], [10, 10, 10, 10], randn((4, Hkv, Dh), g),
                randn((4, Hkv, Dh), g)))
    ops.append(("tokens", [0, 1, 0], [0, 0, 1], [11, 11, 11], randn((3, Hkv, Dh), g), randn((3, Hkv, Dh), g)))
    ops.append(("pack", [0, 1, 2, 0], [0, 0, 1, 1], [11, 11, 10, 11]))
    ops.append(("drop", 0, 11))
    ops.append(("tokens", [2, 2], [0, 1], [12, 13], randn((2, Hkv, Dh), g), randn((2, Hkv, Dh), g)))
    ops.append(("drop", 1, 5))
    ops.append(("pack", [2, 0, 1], [1, 1, 0], [4, 4, 10]))
    return ops


def cfg3_accept() -> torch.Tensor:
    """Config 3: per-sequence accepted lengths U{0..8}, seed 3."""
    return torch.randint(0, 9, (32,), generator=gen(3))


# ---------------------------------------------------------------------------
# deterministic stand-in for the model blocks (scheduler golden runs)
# ---------------------------------------------------------------------------
def _mix(*xs) -> int:
    h = 1469598103934665603
    for x in xs:
        h ^= (int(x) + 0x9E3779B97F4A7C15) & 0xFFFFFFFFFFFFFFFF
        h = (h * 1099511628211) & 0xFFFFFFFFFFFFFFFF
    return h


class FakeCache:
    """Records the rollbacks a scheduler issues."""

    nbytes = 0

    def __init__(self):
        self.drops = []

    def drop_positions_at_and_after(self, b, position):
        self.drops.append((int(b), int(position)))


class FakeBlocks:
    """Union P / R / C interface of the reference's batch blocks
    (ouro_blocks_batch.py:123-248) with token choices that depend only on
    (sequence, position, token, depth): the greedy id at full depth for a token
    at position p is the 'gold' for p+1; at draft depth it agrees with the gold
    with probability ~ agree."""

    def __init__(self, T_total: int, vocab: int = 50, agree: float = 0.7, seed: int = 0):
        self.T_total = T_total
        self.vocab = vocab
        self.agree_mod = 1000
        self.agree_thr = int(agree * 1000)
        self.seed = seed

    def prefill(self, prompt_ids):
        B = prompt_ids.shape[0]
        logits = torch.zeros((B, self.vocab))
        for b in range(B):
            logits[b, _mix(self.seed, b, int(prompt_ids[b].sum())) % self.vocab] = 1.0
        self.last_cache = FakeCache()
        return self.last_cache, logits

    def prelude_union(self, seq_ids, toks, cache):
        for b, t in zip(seq_ids, toks):
            t.hidden = (int(b), int(t.token_id), int(t.position))
            t.static_state = None
            t.step = 0

    def advance_union(self, seq_ids, toks, cache):
        for t in toks:
            t.step += 1

    def coda_argmax_union(self, seq_ids, toks, cache):
        out = []
        for b, t in zip(seq_ids, toks):
            sb, tok, pos = t.hidden
            gold = _mix(self.seed, 1, sb, tok, pos) % self.vocab
            if t.step >= self.T_total or _mix(self.seed, 2, sb, tok, pos) % self.agree_mod < self.agree_thr:
                out.append(gold)
            else:
                out.append((gold + 1 + _mix(self.seed, 3, sb, pos) % (self.vocab - 1)) % self.vocab)
        return out


SCHED_CASES = [
    dict(name="wfd_T4_D1_greedy", T_total=4, T_draft=1, B=3, L=7, new=24, alpha=None),
    dict(name="wfd_T4_D2_greedy", T_total=4, T_draft=2, B=3, L=5, new=24, alpha=None),
    dict(name="wfd_T8_D2_emu05", T_total=8, T_draft=2, B=4, L=6, new=20, alpha=0.5),
    dict(name="wfd_T4_D4_emu1", T_total=4, T_draft=4, B=2, L=4, new=16, alpha=1.0),
    dict(name="wfd_T6_D3_emu08", T_total=6, T_draft=3, B=3, L=9, new=18, alpha=0.8),
]


# draft-then-verify (scheduler_batch.py:378-501): K = draft_length drafts per round
DTV_CASES = [
    dict(name="dtv_T4_D1_K3_greedy", T_total=4, T_draft=1, K=3, B=3, L=7, new=24, alpha=None),
    dict(name="dtv_T4_D2_K4_emu08", T_total=4, T_draft=2, K=4, B=3, L=5, new=20, alpha=0.8),
    dict(name="dtv_T8_D2_K8_emu05", T_total=8, T_draft=2, K=8, B=4, L=6, new=20, alpha=0.5),
]


def sched_prompts(case) -> torch.Tensor:
    return torch.randint(0, 50, (case["B"], case["L"]), generator=gen(97))


def trace_summary(bt, cache) -> dict:
    return {
        "tokens": [list(map(int, t.tokens)) for t in bt.per_seq],
        "counters": [[t.n_r_calls, t.n_p_calls, t.n_c_calls, t.n_drafts_proposed, t.n_drafts_accepted,
                      t.n_drafts_rejected, t.n_rollback_events] for t in bt.per_seq],
        "batch": [bt.n_r_calls, bt.n_p_calls, bt.n_c_calls, bt.r_union_total, bt.r_union_max],
        "drops": [list(d) for d in cache.drops],
    }
