"""GPU parity of the wavefront attention kernels against the CPU oracle and the
reference's golden vectors.  Every call goes through libwfd_b200 (C ABI).

Tolerances: max-abs 2e-2 for bf16 inputs, 1e-5 for fp32
inputs, softmax statistics in fp32.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import golden_inputs as gi
from oracle import attention as oattn
from oracle.kv_cache import SlotCacheOracle

pytestmark = pytest.mark.gpu

TOL_BF16 = 2e-2
TOL_F32 = 1e-5


def tol(dt):
    return TOL_BF16 if dt == torch.bfloat16 else TOL_F32


def maxdiff(a, b) -> float:
    a = a.detach().float().cpu().numpy() if isinstance(a, torch.Tensor) else np.asarray(a)
    b = b.detach().float().cpu().numpy() if isinstance(b, torch.Tensor) else np.asarray(b)
    return float(np.abs(a.astype(np.float64) - b.astype(np.float64)).max())


def no_device_error(dev):
    from wavefront_decoding_b200 import runtime as rt
    assert rt.read_device_error(dev) == 0


# ---------------------------------------------------------------------------
# reference-surface functions vs golden + oracle
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("case", gi.VARLEN_CASES, ids=[c["name"] for c in gi.VARLEN_CASES])
def test_attn_varlen(cuda_dev, golden, case):
    from wavefront_decoding_b200 import attention as wa
    q, k, v, cu_q, cu_k = gi.varlen_inputs(case)
    ref = oattn.attn_varlen(q, k, v, cu_q, cu_k, causal=case["causal"])
    out = wa.attn_varlen(q.to(cuda_dev), k.to(cuda_dev), v.to(cuda_dev), cu_q.to(cuda_dev), cu_k.to(cuda_dev),
                         int((cu_q[1:] - cu_q[:-1]).max()), int((cu_k[1:] - cu_k[:-1]).max()),
                         causal=case["causal"])
    torch.cuda.synchronize()
    no_device_error(cuda_dev)
    assert maxdiff(out, ref) < tol(q.dtype)
    assert maxdiff(out, golden[f"varlen/{case['name']}/out"]) < tol(q.dtype)


def test_attn_varlen_q1_padded(cuda_dev, golden):
    from wavefront_decoding_b200 import attention as wa
    q, k, v, cu_q, cu_k = gi.varlen_inputs(gi.Q1_PADDED_CASE)
    out = wa.attn_varlen_q1_padded(q.to(cuda_dev), k.to(cuda_dev), v.to(cuda_dev), cu_k.to(cuda_dev),
                                   int((cu_k[1:] - cu_k[:-1]).max()))
    assert maxdiff(out, golden["q1_padded/out"]) < TOL_F32


@pytest.mark.parametrize("case", gi.DENSE_CASES, ids=[c["name"] for c in gi.DENSE_CASES])
def test_attn_dense(cuda_dev, golden, case):
    from wavefront_decoding_b200 import attention as wa
    q, k, v = gi.dense_inputs(case)
    out = wa.attn_dense(q.to(cuda_dev), k.to(cuda_dev), v.to(cuda_dev), causal=case["causal"])
    assert maxdiff(out, golden[f"dense/{case['name']}/out"]) < TOL_F32


def test_attn_cutoff_multi(cuda_dev, golden):
    from wavefront_decoding_b200 import attention as wa
    q, k, v, qpos = gi.cutoff_inputs()
    out = wa.attn_cutoff_multi(q.to(cuda_dev), k.to(cuda_dev), v.to(cuda_dev), qpos)
    assert maxdiff(out, golden["cutoff/out"]) < TOL_F32
    with pytest.raises(AssertionError):
        wa.attn_cutoff_multi(q.to(cuda_dev), k[:, :-1].to(cuda_dev), v[:, :-1].to(cuda_dev), qpos)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16], ids=["f32", "bf16"])
def test_gate1_graph_lengths_as_data(cuda_dev, golden, dtype):
    """exp5 gate 1 (verify_graph.py:45-147): one captured graph serves growing
    key lengths held in a device cu_k; a cross-length check proves the new
    length took effect."""
    from wavefront_decoding_b200 import attention as wa
    from wavefront_decoding_b200 import runtime as rt
    K, V, q1, q8 = gi.gate1_inputs()
    Kd, Vd = K.to(cuda_dev, dtype), V.to(cuda_dev, dtype)
    q1d, q8d = q1.to(cuda_dev, dtype), q8.to(cuda_dev, dtype)
    MAX = K.shape[0]
    cu1 = torch.tensor([0, 1], dtype=torch.int32, device=cuda_dev)
    cu8 = torch.tensor([0, 8], dtype=torch.int32, device=cuda_dev)
    cuk_a = torch.tensor([0, 600], dtype=torch.int32, device=cuda_dev)
    cuk_b = torch.tensor([0, 600], dtype=torch.int32, device=cuda_dev)
    rt.reserve_workspace(cuda_dev, 16, 128)
    rt.error_word(cuda_dev)
    out_a = torch.empty_like(q1d)
    out_b = torch.empty_like(q8d)

    def fa():
        wa.attn_varlen(q1d, Kd, Vd, cu1, cuk_a, 1, MAX, causal=False, out=out_a)

    def fb():
        wa.attn_varlen(q8d, Kd, Vd, cu8, cuk_b, 8, MAX, causal=True, out=out_b)

    graphs = []
    for fn in (fa, fb):
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(3):
                fn()
        torch.cuda.current_stream().wait_stream(side)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn()
        graphs.append(g)
    t = tol(dtype) if dtype == torch.float32 else 3e-2  # gate TOL (verify_graph.py:27)
    for n in gi.GATE1_LENGTHS:
        cuk_a[1] = n
        cuk_b[1] = n
        graphs[0].replay()
        graphs[1].replay()
        torch.cuda.synchronize()
        assert maxdiff(out_a, golden[f"gate1/a/{n}"]) < t
        assert maxdiff(out_b, golden[f"gate1/b/{n}"]) < t
    cuk_a[1] = 900
    graphs[0].replay()
    torch.cuda.synchronize()
    assert maxdiff(out_a, golden["gate1/a/600"]) > 1e-3  # DISTINGUISH (verify_graph.py:28)
    no_device_error(cuda_dev)
    del graphs


# ---------------------------------------------------------------------------
# slot-native wavefront op (fused append) vs the oracle
# ---------------------------------------------------------------------------
def _wave_case(seed, n_slots, B, S, H, Hkv, Dh, items, dtype):
    g = gi.gen(seed)
    K = gi.randn((n_slots, B, S, Hkv, Dh), g, dtype)
    V = gi.randn((n_slots, B, S, Hkv, Dh), g, dtype)
    n_rows = max(it[4] + it[3] for it in items) if items else 0
    q = gi.randn((n_rows, H, Dh), g, dtype)
    kn = gi.randn((n_rows, Hkv, Dh), g, dtype)
    vn = gi.randn((n_rows, Hkv, Dh), g, dtype)
    return K, V, q, kn, vn


def _run_wave(dev, K, V, q, kn, vn, items, max_q, slot_offset=0, kernel=-1):
    from wavefront_decoding_b200 import attention as wa
    Kd, Vd = K.to(dev).contiguous(), V.to(dev).contiguous()
    lens = torch.zeros(K.shape[:2], dtype=torch.int32, device=dev)
    it = torch.tensor(items, dtype=torch.int32, device=dev).reshape(-1, 5)
    out = wa.wave_attn(q.to(dev), kn.to(dev), vn.to(dev), Kd, Vd, it, max_q, lens=lens, slot_offset=slot_offset,
                       kernel=kernel)
    torch.cuda.synchronize()
    return out, Kd, Vd, lens


def _oracle_wave(K, V, q, kn, vn, items, slot_offset=0):
    n_slots, B, S, Hkv, Dh = K.shape
    o = SlotCacheOracle(n_slots, B, Hkv, Dh, S)
    o.K[:] = K.float().numpy()
    o.V[:] = V.float().numpy()
    ref = o.wave_attn(q.float().numpy(), kn.float().numpy(), vn.float().numpy(), items, slot_offset)
    return ref, o


WAVE_CASES = [
    # (name, n_slots, B, S, H, Hkv, Dh, items)
    ("tick_gqa4_d128", 4, 3, 300, 16, 4, 128,
     [[r, b, 250 - 7 * r + b, 1, r * 3 + b] for r in range(4) for b in range(3)]),
    ("tick_mha_d64", 3, 2, 200, 6, 6, 64, [[r, b, 100 + r, 1, r * 2 + b] for r in range(3) for b in range(2)]),
    ("first_token_and_full_slot", 2, 2, 64, 8, 2, 128, [[0, 0, 0, 1, 0], [1, 1, 63, 1, 1], [0, 1, 31, 1, 2]]),
    ("verify_windows_small", 2, 2, 160, 8, 2, 128, [[0, 0, 100, 4, 0], [1, 1, 150, 2, 4], [1, 0, 7, 1, 6]]),
    ("gqa8_d64_ragged", 3, 2, 400, 16, 2, 64, [[r, b, 13 + 131 * r + 17 * b, 1, 2 * r + b]
                                                for r in range(3) for b in range(2)]),
]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32], ids=["bf16", "f32"])
@pytest.mark.parametrize("case", WAVE_CASES, ids=[c[0] for c in WAVE_CASES])
def test_wave_attn_vs_oracle(cuda_dev, case, dtype):
    name, n_slots, B, S, H, Hkv, Dh, items = case
    K, V, q, kn, vn = _wave_case(sum(map(ord, name)), n_slots, B, S, H, Hkv, Dh, items, dtype)
    max_q = max(it[3] for it in items)
    out, Kd, Vd, lens = _run_wave(cuda_dev, K, V, q, kn, vn, items, max_q, kernel=0)
    no_device_error(cuda_dev)
    ref, o = _oracle_wave(K, V, q, kn, vn, items)
    assert maxdiff(out, ref) < tol(dtype)
    # the fused append wrote exactly the window rows
    assert maxdiff(Kd, o.K) == 0.0 and maxdiff(Vd, o.V) == 0.0
    for slot, seq, p0, ql, _ in items:
        assert int(lens[slot, seq]) == p0 + ql


def test_wave_attn_slot_offset(cuda_dev):
    items = [[0, b, 40 + b, 1, b] for b in range(2)]
    K, V, q, kn, vn = _wave_case(3, 3, 2, 64, 8, 2, 128, items, torch.bfloat16)
    out, Kd, _, lens = _run_wave(cuda_dev, K, V, q, kn, vn, items, 1, slot_offset=2)
    ref, o = _oracle_wave(K, V, q, kn, vn, items, slot_offset=2)
    assert maxdiff(out, ref) < TOL_BF16
    assert maxdiff(Kd, o.K) == 0.0
    assert int(lens[2, 0]) == 41 and int(lens[0, 0]) == 0


def test_wave_attn_empty_and_bad_items(cuda_dev):
    """Out-of-range items are skipped and reported through the device error
    word; the valid items of the same call are still exact."""
    from wavefront_decoding_b200 import attention as wa
    from wavefront_decoding_b200 import runtime as rt
    items_ok = [[0, 0, 10, 1, 0], [1, 1, 20, 1, 1]]
    K, V, q, kn, vn = _wave_case(9, 2, 2, 32, 4, 2, 64, items_ok + [[0, 0, 0, 1, 2]], torch.float32)
    bad = [[5, 0, 3, 1, 2]]  # slot out of range
    out, _, _, _ = _run_wave(cuda_dev, K, V, q, kn, vn, items_ok + bad, 1)
    from wavefront_decoding_b200._abi import WfdError
    with pytest.raises(WfdError):
        rt.read_device_error(cuda_dev)
    ref, _ = _oracle_wave(K, V, q, kn, vn, items_ok)
    assert maxdiff(out[:2], ref[:2]) < TOL_F32
    # an empty table is a no-op
    it = torch.zeros((0, 5), dtype=torch.int32, device=cuda_dev)
    wa.wave_attn(q.to(cuda_dev), kn.to(cuda_dev), vn.to(cuda_dev), K.to(cuda_dev), V.to(cuda_dev), it, 1)
    assert rt.read_device_error(cuda_dev) == 0


def test_wave_attn_many_items_balanced_split(cuda_dev):
    """More work items than CTAs, very uneven lengths: exercises the stream-K
    split, multi-CTA units and the last-arriver merge."""
    rng = np.random.default_rng(0)
    n_slots, B, S = 6, 16, 1024
    items = []
    for r in range(n_slots):
        for b in range(B):
            items.append([r, b, int(rng.integers(0, S - 1)), 1, len(items)])
    K, V, q, kn, vn = _wave_case(21, n_slots, B, S, 8, 2, 128, items, torch.bfloat16)
    ref, _ = _oracle_wave(K, V, q, kn, vn, items)
    small = [[0, 0, 700, 1, 0], [1, 3, 5, 1, 1], [5, 15, 1000, 1, 2]]
    Ks, Vs, qs, kns, vns = _wave_case(22, n_slots, B, S, 8, 2, 128, small, torch.float32)
    ref_s, _ = _oracle_wave(Ks, Vs, qs, kns, vns, small)
    for rep in range(3):
        # launches with other item counts / dtypes in between must not disturb
        # the split-K arrival counters the next launch relies on
        out, _, _, _ = _run_wave(cuda_dev, K, V, q, kn, vn, items, 1)
        assert maxdiff(out, ref) < TOL_BF16
        out_s, _, _, _ = _run_wave(cuda_dev, Ks, Vs, qs, kns, vns, small, 1)
        assert maxdiff(out_s, ref_s) < TOL_F32
    no_device_error(cuda_dev)


def _cfg2_inputs():
    """Config 2: B=8, R=8, Hq=16, Hkv=4, Dh=128, bf16; q (B,R,16,128), K, V
    (R,B,4096,4,128) ~ N(0,1) from seed 1 in that order; slot r of every
    sequence holds L_r = 4096 - r positions and one query at position L_r - 1."""
    g = gi.gen(1)
    B, R, H, Hkv, Dh, S = 8, 8, 16, 4, 128, 4096
    q = gi.randn((B, R, H, Dh), g, torch.bfloat16)
    K = gi.randn((R, B, S, Hkv, Dh), g, torch.bfloat16)
    V = gi.randn((R, B, S, Hkv, Dh), g, torch.bfloat16)
    items = [[r, b, S - r - 1, 1, b * R + r] for b in range(B) for r in range(R)]
    return q.reshape(B * R, H, Dh), K, V, items


def test_cfg2_full_size_vs_oracle(cuda_dev):
    from wavefront_decoding_b200 import attention as wa
    q, K, V, items = _cfg2_inputs()
    # the appended row is the row already in the cache: the op reads L_r keys
    kn = torch.stack([K[r, b, p] for r, b, p, _, _ in sorted(items, key=lambda t: t[4])])
    vn = torch.stack([V[r, b, p] for r, b, p, _, _ in sorted(items, key=lambda t: t[4])])
    Kd, Vd = K.to(cuda_dev), V.to(cuda_dev)
    it = torch.tensor(items, dtype=torch.int32, device=cuda_dev)
    out = wa.wave_attn(q.to(cuda_dev), kn.to(cuda_dev), vn.to(cuda_dev), Kd, Vd, it, 1)
    torch.cuda.synchronize()
    no_device_error(cuda_dev)
    out = out.float().cpu().numpy()
    worst = 0.0
    for r, b, p, _, row in items:
        ref = oattn.attn_varlen(q[row:row + 1], K[r, b, :p + 1], V[r, b, :p + 1], [0, 1], [0, p + 1])
        worst = max(worst, float(np.abs(out[row:row + 1] - ref).max()))
    assert worst < TOL_BF16, worst
    assert torch.equal(Kd.cpu(), K)  # rewriting the same rows leaves the cache unchanged


# ---------------------------------------------------------------------------
# tcgen05 tensor-core kernel (kernel=1): decode rows and verify windows
# ---------------------------------------------------------------------------
TC_CASES = [
    # (name, n_slots, B, S, H, Hkv, items)      Dh = 128 (Dh = 64 where the name ends in _d64), bf16
    ("tc_decode_gqa4", 4, 3, 300, 16, 4, [[r, b, 250 - 7 * r + b, 1, r * 3 + b] for r in range(4) for b in range(3)]),
    ("tc_first_and_full", 2, 2, 200, 8, 2, [[0, 0, 0, 1, 0], [1, 1, 199, 1, 1], [0, 1, 127, 1, 2], [1, 0, 128, 1, 3]]),
    ("tc_window8_gqa4", 3, 2, 400, 16, 4, [[r, b, 300 - 50 * r + 3 * b, 8, (r * 2 + b) * 8]
                                           for r in range(3) for b in range(2)]),
    ("tc_window_ragged", 2, 3, 300, 8, 2, [[0, 0, 5, 3, 0], [1, 2, 250, 8, 3], [0, 1, 130, 6, 11], [1, 0, 0, 2, 17]]),
    ("tc_window16_qgroups", 2, 2, 500, 16, 4, [[0, 0, 400, 16, 0], [1, 1, 37, 12, 16]]),
    ("tc_mha", 2, 2, 300, 4, 4, [[0, 0, 150, 1, 0], [1, 1, 260, 8, 1]]),
    ("tc_decode_mha_d64", 4, 3, 400, 6, 6, [[r, b, 390 - 9 * r - b, 1, r * 3 + b] for r in range(4) for b in range(3)]),
    ("tc_first_and_full_d64", 2, 2, 200, 4, 4, [[0, 0, 0, 1, 0], [1, 1, 199, 1, 1], [0, 1, 127, 1, 2],
                                                 [1, 0, 128, 1, 3]]),
    ("tc_window8_gqa4_d64", 3, 2, 400, 16, 4, [[r, b, 300 - 50 * r + 3 * b, 8, (r * 2 + b) * 8]
                                               for r in range(3) for b in range(2)]),
    ("tc_window_ragged_d64", 2, 3, 300, 8, 2, [[0, 0, 5, 3, 0], [1, 2, 250, 8, 3], [0, 1, 130, 6, 11],
                                                [1, 0, 0, 2, 17]]),
    ("tc_window16_qgroups_d64", 2, 2, 500, 16, 4, [[0, 0, 400, 16, 0], [1, 1, 37, 12, 16]]),
    # head_dim 64 with an even kv-head count runs as head pairs on the 128-dim kernel
    ("tc_window8_mha_pair_d64", 2, 3, 300, 6, 6, [[r, b, 200 - 30 * r + 7 * b, 8, (r * 3 + b) * 8]
                                                   for r in range(2) for b in range(3)]),
    ("tc_window4_gqa2_pair_d64", 3, 2, 300, 8, 4, [[0, 0, 10, 4, 0], [1, 1, 250, 3, 4], [2, 0, 0, 2, 7],
                                                    [2, 1, 131, 4, 9]]),
    ("tc_decode_mha_odd_d64", 2, 2, 300, 3, 3, [[r, b, 280 - 40 * r - b, 1, r * 2 + b] for r in range(2)
                                                 for b in range(2)]),
]


@pytest.mark.parametrize("case", TC_CASES, ids=[c[0] for c in TC_CASES])
def test_tc_kernel_vs_oracle(cuda_dev, case):
    name, n_slots, B, S, H, Hkv, items = case
    Dh = 64 if name.endswith("_d64") else 128
    K, V, q, kn, vn = _wave_case(sum(map(ord, name)), n_slots, B, S, H, Hkv, Dh, items, torch.bfloat16)
    max_q = max(it[3] for it in items)
    out, Kd, Vd, lens = _run_wave(cuda_dev, K, V, q, kn, vn, items, max_q, kernel=1)
    no_device_error(cuda_dev)
    ref, o = _oracle_wave(K, V, q, kn, vn, items)
    assert maxdiff(out, ref) < TOL_BF16
    assert maxdiff(Kd, o.K) == 0.0 and maxdiff(Vd, o.V) == 0.0
    for slot, seq, p0, ql, _ in items:
        assert int(lens[slot, seq]) == p0 + ql


@pytest.mark.parametrize("Dh,H,Hkv,max_ql", [(128, 16, 4, 8), (64, 12, 12, 8), (64, 12, 12, 1), (128, 16, 4, 1)])
def test_tc_kernel_balanced_split(cuda_dev, Dh, H, Hkv, max_ql):
    """Many units of very different lengths over the persistent grid; the
    second and third launches check the arrival counters were left zeroed."""
    rng = np.random.default_rng(3)
    n_slots, B, S = 4, 24, 2048
    items = []
    for r in range(n_slots):
        for b in range(B):
            ql = int(rng.integers(1, max_ql + 1))
            items.append([r, b, int(rng.integers(0, S - ql)), ql, 0])
    row = 0
    for it in items:
        it[4] = row
        row += it[3]
    K, V, q, kn, vn = _wave_case(31, n_slots, B, S, H, Hkv, Dh, items, torch.bfloat16)
    ref, _ = _oracle_wave(K, V, q, kn, vn, items)
    first = None
    for _ in range(3):
        out, _, _, _ = _run_wave(cuda_dev, K, V, q, kn, vn, items, max_ql, kernel=1)
        assert maxdiff(out, ref) < TOL_BF16
        # partials are merged in key order, whichever CTA arrives last: identical launches, identical bits
        if first is None:
            first = out.clone()
        else:
            assert torch.equal(out, first)
    no_device_error(cuda_dev)


def test_tc_varlen_packed_causal(cuda_dev):
    """Packed varlen (attn_varlen, causal windows) routed to the tensor cores."""
    from wavefront_decoding_b200 import attention as wa
    g = gi.gen(77)
    q_lens, k_lens = [8, 1, 8, 5], [700, 90, 8, 300]
    q = gi.randn((sum(q_lens), 16, 128), g, torch.bfloat16)
    k = gi.randn((sum(k_lens), 4, 128), g, torch.bfloat16)
    v = gi.randn((sum(k_lens), 4, 128), g, torch.bfloat16)
    cu_q = torch.tensor(np.concatenate([[0], np.cumsum(q_lens)]), dtype=torch.int32)
    cu_k = torch.tensor(np.concatenate([[0], np.cumsum(k_lens)]), dtype=torch.int32)
    ref = oattn.attn_varlen(q, k, v, cu_q, cu_k, causal=True)
    out = wa.attn_varlen(q.to(cuda_dev), k.to(cuda_dev), v.to(cuda_dev), cu_q.to(cuda_dev), cu_k.to(cuda_dev), 8,
                         max(k_lens), causal=True)
    no_device_error(cuda_dev)
    assert maxdiff(out, ref) < TOL_BF16


def test_tc_more_items_than_staged_and_append_blocks(cuda_dev):
    """4200 items: more than the plan kernel keeps in shared memory (its start
    records then search the global prefix) and many more than its window-append
    blocks (grid-stride); two out-of-range items are skipped and reported while
    every valid item is still exact and appended."""
    from wavefront_decoding_b200 import runtime as rt
    from wavefront_decoding_b200._abi import WfdError
    rng = np.random.default_rng(11)
    n_slots, B, S, H, Hkv, Dh = 2, 2100, 48, 4, 2, 128
    items = [[r, b, int(rng.integers(0, S - 1)), 1, r * B + b] for r in range(n_slots) for b in range(B)]
    K, V, q, kn, vn = _wave_case(41, n_slots, B, S, H, Hkv, Dh, items, torch.bfloat16)
    ref, o = _oracle_wave(K, V, q, kn, vn, items)
    bad = [list(items[7]), list(items[3001])]
    bad[0][0] = n_slots          # slot out of range
    bad[1][2] = S                # window past the slot
    run_items = [bad[0] if i == 7 else bad[1] if i == 3001 else it for i, it in enumerate(items)]
    out, Kd, Vd, lens = _run_wave(cuda_dev, K, V, q, kn, vn, run_items, 1, kernel=1)
    with pytest.raises(WfdError):
        rt.read_device_error(cuda_dev)
    keep = torch.ones(len(items), dtype=torch.bool)
    keep[7] = keep[3001] = False
    assert maxdiff(out.cpu()[keep], ref[keep.numpy()]) < TOL_BF16
    # appended rows: every valid item's window row is in place; the skipped items wrote nothing
    Kh = Kd.cpu()
    for i, (slot, seq, p0, ql, row) in enumerate(items):
        if keep[i]:
            assert torch.equal(Kh[slot, seq, p0], kn[row]), i
            assert int(lens[slot, seq]) == p0 + ql
    assert torch.equal(Kh[0, 7], K[0, 7])
    assert int(lens[0, 7]) == 0


def test_tc_bounded_wait_gives_up_and_next_launch_is_exact(cuda_dev):
    """Every CTA of the tcgen05 kernel is made to give up as a wait that ran out
    would, with its first K/V copies in flight (a test hook): the launch still
    returns, the error word reports a timeout (WFD_ERR_DEVICE_TIMEOUT), and the
    next launches, on the same workspace, are exact — the aborted launch drained
    its copies and MMAs and left the split-K arrival counters zeroed."""
    from wavefront_decoding_b200 import runtime as rt
    from wavefront_decoding_b200._abi import WfdError
    rng = np.random.default_rng(5)
    n_slots, B, S, H, Hkv = 3, 8, 1500, 16, 4
    items = []
    for r in range(n_slots):
        for b in range(B):
            ql = 1 if (r + b) % 2 else 8
            items.append([r, b, int(rng.integers(200, S - 8)), ql, 0])
    row = 0
    for it in items:
        it[4] = row
        row += it[3]
    K, V, q, kn, vn = _wave_case(55, n_slots, B, S, H, Hkv, 128, items, torch.bfloat16)
    ref, o = _oracle_wave(K, V, q, kn, vn, items)
    assert rt.read_device_error(cuda_dev) == 0
    rt.test_fail_waits(True)
    try:
        _run_wave(cuda_dev, K, V, q, kn, vn, items, 8, kernel=1)
    finally:
        rt.test_fail_waits(False)
    with pytest.raises(WfdError) as err:
        rt.read_device_error(cuda_dev)
    assert err.value.status == 16
    for _ in range(2):
        out, Kd, Vd, lens = _run_wave(cuda_dev, K, V, q, kn, vn, items, 8, kernel=1)
        no_device_error(cuda_dev)
        assert maxdiff(out, ref) < TOL_BF16
        assert maxdiff(Kd, o.K) == 0.0 and maxdiff(Vd, o.V) == 0.0


@pytest.mark.parametrize("Dh,H,Hkv", [(128, 16, 4), (64, 6, 6)], ids=["gqa4_d128", "mha_pair_d64"])
def test_tc_gapped_windows_vs_oracle(cuda_dev, Dh, H, Hkv):
    """Gapped windows (per-row positions, wfd_wave_attn_rows): the rows of one
    sequence on one slot at positions with gaps (stride 2, stride 3, irregular)
    form one window.  Outputs equal the oracle's one-window-per-row result (each
    row sees keys up to its own position, every row appended before any row
    attends), only the rows' own positions are written (bit-exact), and each
    slot length rises to the last row's position + 1.  The positions are read
    through a strided view (a table column), as the engine passes them."""
    from wavefront_decoding_b200 import attention as wa
    windows = [(0, 0, [400, 402, 404, 406]), (1, 1, [500, 503, 506]), (2, 2, [100, 101, 105, 106, 110]),
               (0, 3, [50]), (1, 0, [7, 9])]
    items, pos, row = [], [], 0
    for slot, seq, ps in windows:
        items.append([slot, seq, ps[0], len(ps), row])
        pos += ps
        row += len(ps)
    K, V, q, kn, vn = _wave_case(61 + Dh, 3, 4, 600, H, Hkv, Dh, items, torch.bfloat16)
    tab = torch.zeros((row, 6), dtype=torch.int32)
    tab[:, 1] = torch.tensor(pos, dtype=torch.int32)
    tabd = tab.to(cuda_dev)
    Kd, Vd = K.to(cuda_dev).contiguous(), V.to(cuda_dev).contiguous()
    lens = torch.zeros(K.shape[:2], dtype=torch.int32, device=cuda_dev)
    it = torch.tensor(items, dtype=torch.int32, device=cuda_dev)
    out = wa.wave_attn(q.to(cuda_dev), kn.to(cuda_dev), vn.to(cuda_dev), Kd, Vd, it, 5, lens=lens,
                       row_pos=tabd[:, 1])
    torch.cuda.synchronize()
    no_device_error(cuda_dev)
    per_row = [[slot, seq, p, 1, r] for (slot, seq, ps), base in zip(windows, [it_[4] for it_ in items])
               for r, p in zip(range(base, base + len(ps)), ps)]
    ref, o = _oracle_wave(K, V, q, kn, vn, per_row)
    assert maxdiff(out, ref) < TOL_BF16
    assert maxdiff(Kd, o.K) == 0.0 and maxdiff(Vd, o.V) == 0.0
    for slot, seq, ps in windows:
        assert int(lens[slot, seq]) == max(ps) + 1
    # the same table without per-row positions is a different (contiguous) window: not what was asked
    with pytest.raises(Exception):
        wa.wave_attn(q.to(cuda_dev).float(), kn.to(cuda_dev).float(), vn.to(cuda_dev).float(), Kd.float(),
                     Vd.float(), it, 5, row_pos=tabd[:, 1])  # fp32 has no gapped-window kernel
