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
