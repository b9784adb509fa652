"""GPU parity of the KV-slot kernels (append, prefill, rollback, accept commit,
gather) against the reference's golden session and the oracle — bit-exact."""
from __future__ import annotations

import json
import pathlib

import numpy as np
import pytest
import torch

import golden_inputs as gi
from oracle.kv_cache import SlotCacheOracle

pytestmark = pytest.mark.gpu


def test_kv_script_matches_reference(cuda_dev, golden):
    from wavefront_decoding_b200.kv_cache import SlotKVCache
    n_slots, B, S, Hkv, Dh = gi.KV_SCRIPT_GEOM
    c = SlotKVCache(n_slots, B, Hkv, Dh, S, torch.float32, cuda_dev)
    log = json.loads((pathlib.Path(__file__).parent / "golden" / "reference_kv_log.json").read_text())
    for step, op in enumerate(gi.kv_script()):
        if op[0] == "prefill":
            c.write_prefill(op[1], op[2].to(cuda_dev), op[3].to(cuda_dev))
        elif op[0] == "tokens":
            c.write_tokens(op[1], op[2], op[3], op[4].to(cuda_dev), op[5].to(cuda_dev))
        elif op[0] == "drop":
            c.drop_positions_at_and_after(op[1], op[2])
        else:
            kp, vp, cu_k, max_k = c.gather_pack(op[1], op[2], op[3])
            assert np.array_equal(kp.cpu().numpy(), golden[f"kv/pack{step}/k"])
            assert np.array_equal(vp.cpu().numpy(), golden[f"kv/pack{step}/v"])
            assert np.array_equal(cu_k.cpu().numpy(), golden[f"kv/pack{step}/cu_k"])
            assert max_k == int(golden[f"kv/pack{step}/max_k"])
        assert c.seqlen == log["seqlen"][step], step
    from wavefront_decoding_b200 import runtime as rt
    assert rt.read_device_error(cuda_dev) == 0


def test_write_tokens_overflow_raises(cuda_dev):
    from wavefront_decoding_b200.kv_cache import SlotKVCache
    c = SlotKVCache(1, 1, 1, 16, 8, torch.bfloat16, cuda_dev)
    with pytest.raises(IndexError):
        c.write_tokens([0], [0], [8], torch.zeros((1, 1, 16), dtype=torch.bfloat16, device=cuda_dev),
                       torch.zeros((1, 1, 16), dtype=torch.bfloat16, device=cuda_dev))


def _filled_cache(dev, n_slots, B, S, Hkv, Dh, seed, dtype=torch.bfloat16):
    from wavefront_decoding_b200.kv_cache import SlotKVCache
    g = gi.gen(seed)
    c = SlotKVCache(n_slots, B, Hkv, Dh, S, dtype, dev)
    K = gi.randn(c.K.shape, g, dtype)
    V = gi.randn(c.V.shape, g, dtype)
    c.K.copy_(K)
    c.V.copy_(V)
    o = SlotCacheOracle(n_slots, B, Hkv, Dh, S)
    o.K[:] = K.float().numpy()
    o.V[:] = V.float().numpy()
    return c, o


def test_commit_window_prefix(cuda_dev):
    c, o = _filled_cache(cuda_dev, 3, 4, 64, 2, 64, 5)
    items = [[r, b, 20 + r + b, 6, (r * 4 + b) * 6] for r in range(3) for b in range(4)]
    acc = torch.randint(0, 7, (12,), generator=gi.gen(6)).tolist()
    for it in items:
        c.lens[it[0], it[1]] = it[2] + it[3]
        o.seqlen[it[0]][it[1]] = it[2] + it[3]
    acc_rows, acc_count = c.commit_window(torch.tensor(items, dtype=torch.int32), accept_len=torch.tensor(acc))
    ref_rows, ref_count = o.commit_window(items, accept_len=acc)
    assert c.seqlen == o.seqlen
    assert acc_count.cpu().tolist() == ref_count
    rows = acc_rows.cpu().tolist()
    for k, v in ref_rows.items():
        assert rows[k] == v
    assert np.array_equal(c.K.float().cpu().numpy(), o.K)


def test_commit_window_mask_compacts(cuda_dev):
    """Non-prefix accept masks move the accepted K/V rows down in place."""
    c, o = _filled_cache(cuda_dev, 2, 2, 48, 2, 128, 8)
    items = [[0, 0, 10, 8, 0], [1, 1, 30, 5, 8], [1, 0, 0, 3, 13]]
    mask = np.zeros(16, dtype=np.uint8)
    mask[[1, 2, 5, 7]] = 1          # item 0: rows 1,2,5,7 -> positions 10..13
    mask[[8, 12]] = 1               # item 1: rows 0,4
    mask[[13, 14, 15]] = 1          # item 2: all (prefix, no move)
    acc_rows, acc_count = c.commit_window(torch.tensor(items, dtype=torch.int32), accept_mask=torch.tensor(mask))
    ref_rows, ref_count = o.commit_window(items, accept_mask=mask)
    assert acc_count.cpu().tolist() == ref_count == [4, 2, 3]
    rows = acc_rows.cpu().tolist()
    for k, v in ref_rows.items():
        assert rows[k] == v
    assert np.array_equal(c.K.float().cpu().numpy(), o.K)
    assert np.array_equal(c.V.float().cpu().numpy(), o.V)
    assert c.seqlen[0][0] == 14 and c.seqlen[1][1] == 32 and c.seqlen[1][0] == 3


def test_cfg3_commit_lengths(cuda_dev, golden):
    """Config 3 commit: 8 slots x 32 sequences, 8-row windows at 8192-r, accepted
    a_b ~ U{0..8} (seed 3) -> slot lengths bit-exact with the reference's rollback."""
    from wavefront_decoding_b200.kv_cache import SlotKVCache
    R, B, L0, W = 8, 32, 8192, 8
    c = SlotKVCache(R, B, 1, 8, L0 + W, torch.bfloat16, cuda_dev)
    a = gi.cfg3_accept()
    items = torch.tensor([[r, b, L0 - r, W, (r * B + b) * W] for r in range(R) for b in range(B)], dtype=torch.int32)
    c.lens.copy_(torch.tensor([[L0 - r + W] * B for r in range(R)], dtype=torch.int32))
    acc_rows, acc_count = c.commit_window(items, accept_len=a.repeat(R).to(torch.int32))
    assert np.array_equal(np.asarray(c.seqlen), golden["cfg3/seqlen"])
    assert acc_count.cpu().tolist() == a.repeat(R).tolist()
    rows = acc_rows.cpu().numpy()
    for i in range(R * B):
        r0 = i * W
        n = int(a[i % B])
        assert rows[r0:r0 + n].tolist() == list(range(r0, r0 + n))


def test_drop_many(cuda_dev):
    from wavefront_decoding_b200.kv_cache import SlotKVCache
    c = SlotKVCache(4, 3, 1, 8, 100, torch.bfloat16, cuda_dev)
    c.lens.copy_(torch.tensor([[50, 60, 70]] * 4, dtype=torch.int32))
    c.lens[2, 1] = 40
    c.drop_many(torch.tensor([-1, 45, 10], dtype=torch.int32))
    assert c.seqlen == [[50, 45, 10], [50, 45, 10], [50, 40, 10], [50, 45, 10]]
