"""Pin the CPU oracle to the reference: every golden vector produced by the
reference's own code (tests/golden/make_golden.py) must be reproduced by the
numpy restatement in oracle/."""
from __future__ import annotations

import json
import pathlib

import numpy as np
import pytest
import torch

import golden_inputs as gi
from oracle import attention as oattn
from oracle.kv_cache import SlotCacheOracle

TOL_F32 = 1e-5


def _check_inputs(golden, key, *ts):
    assert np.allclose(golden[key], gi.checksum(*ts), rtol=0, atol=1e-6 * max(1.0, np.abs(golden[key]).max())), \
        "regenerated inputs differ from the ones the golden file was made from (torch RNG changed?)"


@pytest.mark.parametrize("case", gi.VARLEN_CASES, ids=[c["name"] for c in gi.VARLEN_CASES])
def test_varlen(golden, case):
    q, k, v, cu_q, cu_k = gi.varlen_inputs(case)
    _check_inputs(golden, f"varlen/{case['name']}/checksum", q, k, v)
    out = oattn.attn_varlen(q, k, v, cu_q, cu_k, causal=case["causal"])
    ref = golden[f"varlen/{case['name']}/out"]
    # the reference ran SDPA in the input dtype; bf16 outputs carry bf16 rounding
    tol = TOL_F32 if case["dtype"] == "f32" else 8e-3
    assert np.abs(out - ref).max() < tol


def test_q1_padded(golden):
    q, k, v, cu_q, cu_k = gi.varlen_inputs(gi.Q1_PADDED_CASE)
    _check_inputs(golden, "q1_padded/checksum", q, k, v)
    out = oattn.attn_varlen(q, k, v, cu_q, cu_k, causal=False)
    assert np.abs(out - golden["q1_padded/out"]).max() < TOL_F32


@pytest.mark.parametrize("case", gi.DENSE_CASES, ids=[c["name"] for c in gi.DENSE_CASES])
def test_dense(golden, case):
    q, k, v = gi.dense_inputs(case)
    _check_inputs(golden, f"dense/{case['name']}/checksum", q, k, v)
    out = oattn.attn_dense(q, k, v, causal=case["causal"])
    assert np.abs(out - golden[f"dense/{case['name']}/out"]).max() < TOL_F32


def test_cutoff_multi(golden):
    q, k, v, qpos = gi.cutoff_inputs()
    _check_inputs(golden, "cutoff/checksum", q, k, v)
    out = oattn.attn_cutoff_multi(q, k, v, qpos)
    assert np.abs(out - golden["cutoff/out"]).max() < TOL_F32


def test_gate1_lengths(golden):
    K, V, q1, q8 = gi.gate1_inputs()
    _check_inputs(golden, "gate1/checksum", K, V, q1, q8)
    for n in gi.GATE1_LENGTHS:
        oa = oattn.attn_varlen(q1, K[:n], V[:n], [0, 1], [0, n], causal=False)
        ob = oattn.attn_varlen(q8, K[:n], V[:n], [0, 8], [0, n], causal=True)
        assert np.abs(oa - golden[f"gate1/a/{n}"]).max() < TOL_F32
        assert np.abs(ob - golden[f"gate1/b/{n}"]).max() < TOL_F32


def test_kv_script(golden):
    n_slots, B, S, Hkv, Dh = gi.KV_SCRIPT_GEOM
    c = SlotCacheOracle(n_slots, B, Hkv, Dh, S)
    log = json.loads((pathlib.Path(__file__).parent / "golden" / "reference_kv_log.json").read_text())
    for step, op in enumerate(gi.kv_script()):
        if op[0] == "prefill":
            c.write_prefill(op[1], op[2].numpy(), op[3].numpy())
        elif op[0] == "tokens":
            c.write_tokens(op[1], op[2], op[3], op[4].numpy(), op[5].numpy())
        elif op[0] == "drop":
            c.drop_positions_at_and_after(op[1], op[2])
        else:
            kp, vp, cu_k, max_k = c.gather_pack(op[1], op[2], op[3])
            assert np.array_equal(kp, golden[f"kv/pack{step}/k"])
            assert np.array_equal(vp, golden[f"kv/pack{step}/v"])
            assert np.array_equal(cu_k, golden[f"kv/pack{step}/cu_k"])
            assert max_k == int(golden[f"kv/pack{step}/max_k"])
        assert c.seqlen == log["seqlen"][step]
    assert np.array_equal(np.asarray(c.seqlen), golden["kv/seqlen_final"])


def test_write_tokens_overflow_raises():
    c = SlotCacheOracle(1, 1, 1, 16, 8)
    with pytest.raises(IndexError):
        c.write_tokens([0], [0], [8], np.zeros((1, 1, 16)), np.zeros((1, 1, 16)))


def test_cfg3_commit(golden):
    """Config-3 commit semantics: the oracle's window commit reproduces the
    reference's per-slot rollback lengths bit-exactly."""
    R, B, L0, W = 8, 32, 8192, 8
    a = gi.cfg3_accept()
    assert np.array_equal(a.numpy(), golden["cfg3/accept"])
    c = SlotCacheOracle(R, B, 1, 1, L0 + W)
    items = []
    for r in range(R):
        for b in range(B):
            items.append((r, b, L0 - r, W, (r * B + b) * W))
            c.seqlen[r][b] = L0 - r + W
    acc_rows, acc_count = c.commit_window(items, accept_len=[int(a[b]) for r in range(R) for b in range(B)])
    assert np.array_equal(np.asarray(c.seqlen), golden["cfg3/seqlen"])
    assert acc_count == [int(a[b]) for r in range(R) for b in range(B)]
    for i, (r, b, p0, ql, r0) in enumerate(items):
        for k in range(acc_count[i]):
            assert acc_rows[r0 + k] == r0 + k


def test_oracle_wave_equals_write_pack_varlen():
    """oracle.wave_attn == write_tokens + gather_pack + attn_varlen(causal) per item."""
    g = gi.gen(5)
    n_slots, B, S, Hkv, Dh, H = 2, 2, 40, 2, 64, 4
    c1 = SlotCacheOracle(n_slots, B, Hkv, Dh, S)
    c1.K[:] = gi.randn(c1.K.shape, g).numpy()
    c1.V[:] = gi.randn(c1.V.shape, g).numpy()
    items = np.array([[0, 0, 10, 1, 0], [1, 0, 20, 3, 1], [0, 1, 5, 2, 4]])
    q = gi.randn((6, H, Dh), g).numpy()
    kn = gi.randn((6, Hkv, Dh), g).numpy()
    vn = gi.randn((6, Hkv, Dh), g).numpy()
    out = c1.wave_attn(q, kn, vn, items)
    # explicit composition with full-prefix gathers
    for slot, seq, p0, ql, r0 in items:
        kp, vp, cu_k, _ = c1.gather_pack([slot], [seq], [p0 + ql - 1])
        ref = oattn.attn_varlen(q[r0:r0 + ql], kp, vp, [0, ql], cu_k, causal=True)
        assert np.abs(out[r0:r0 + ql] - ref).max() < 1e-12
        assert np.array_equal(c1.K[slot, seq, p0:p0 + ql], kn[r0:r0 + ql])
        assert c1.seqlen[slot][seq] >= p0 + ql
    # torch fp64 cross-check of one row
    qt = torch.tensor(q[1:4], dtype=torch.float64).unsqueeze(0).transpose(1, 2)
    kt = torch.tensor(c1.K[1, 0, :23], dtype=torch.float64).unsqueeze(0).transpose(1, 2)
    vt = torch.tensor(c1.V[1, 0, :23], dtype=torch.float64).unsqueeze(0).transpose(1, 2)
    mask = torch.arange(23)[None, :] <= (torch.arange(3)[:, None] + 20)
    ref = torch.nn.functional.scaled_dot_product_attention(qt, kt, vt, attn_mask=mask[None, None], enable_gqa=True)
    assert np.abs(out[1:4] - ref.transpose(1, 2)[0].numpy()).max() < 1e-10


# ---------------------------------------------------------------------------
# the timed CPU restatement (bench.py's cpu_baseline / reference arm) computes
# what the reference computes
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("case", [c for c in gi.VARLEN_CASES if c["dtype"] == "f32"],
                         ids=[c["name"] for c in gi.VARLEN_CASES if c["dtype"] == "f32"])
def test_cpu_path_varlen_matches_golden(golden, case):
    from oracle import cpu_path
    q, k, v, cu_q, cu_k = gi.varlen_inputs(case)
    out = cpu_path.attn_varlen_sdpa(q, k, v, cu_q, cu_k, case["causal"])
    assert float(np.abs(out.double().numpy() - golden[f"varlen/{case['name']}/out"]).max()) < 1e-5


@pytest.mark.parametrize("windows", [False, True], ids=["decode", "windows"])
def test_cpu_path_wave_step_matches_oracle(windows):
    """write_tokens + gather_pack + SDPA varlen on the host, fp32: the same
    outputs (1e-5) and cache contents (exact) as the oracle's wave step."""
    from oracle import cpu_path
    g = gi.gen(19)
    n_slots, B, S, H, Hkv, Dh = 3, 2, 80, 8, 2, 64
    if windows:
        items = [[0, 0, 40, 4, 0], [1, 1, 70, 1, 4], [2, 0, 10, 8, 5], [2, 1, 0, 3, 13]]
    else:
        items = [[r, b, 60 - 9 * r - b, 1, r * B + b] for r in range(n_slots) for b in range(B)]
    rows = max(it[4] + it[3] for it in items)
    K = gi.randn((n_slots, B, S, Hkv, Dh), g, torch.float32)
    V = gi.randn((n_slots, B, S, Hkv, Dh), g, torch.float32)
    q = gi.randn((rows, H, Dh), g, torch.float32)
    kn = gi.randn((rows, Hkv, Dh), g, torch.float32)
    vn = gi.randn((rows, Hkv, Dh), g, torch.float32)
    o = SlotCacheOracle(n_slots, B, Hkv, Dh, S)
    o.K[:] = K.numpy()
    o.V[:] = V.numpy()
    ref = o.wave_attn(q.numpy(), kn.numpy(), vn.numpy(), items)
    Kc, Vc = K.clone(), V.clone()
    out = cpu_path.wave_step(Kc, Vc, q, kn, vn, items).double().numpy()
    order = [it[4] + j for it in items for j in range(it[3])]   # wave_step packs rows in item order
    assert float(np.abs(out - ref[order]).max()) < 1e-5
    assert np.array_equal(Kc.numpy(), o.K) and np.array_equal(Vc.numpy(), o.V)
