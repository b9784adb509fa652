"""Configs 3 and 5 at their own geometry: the inputs bench.py times, checked.

Config 3 (verify + commit): B=32, R=8, Hq=32 / Hkv=8, Dh=128, bf16; slot r holds
8192 - r positions and gets an 8-row bottom-right-causal window; q, K, V ~ N(0,1)
drawn on the device from seed 2 (bench.cfg3_device_inputs); accepted lengths
U{0..8} from seed 3.  The test appends NEW window rows (a separate seed), so the
fused append is visible, then compares a deterministic sample of 16
(sequence, slot) items with the float64 oracle (reference semantics:
write_tokens -> gather_pack -> attn_varlen(causal=True), batch_kv_cache.py:61-96,
fa4_attention.py:369-381), checks every appended row and every slot length bit
for bit, and the accept commit (drop_positions_at_and_after semantics,
batch_kv_cache.py:99-105) bit for bit.

Config 5 geometry at small batch: B=2, R=16, Hq=32 / Hkv=8, Dh=128, slot r holds
32768 - r positions plus an 8-row window: units of 256 tiles, 64-bit byte offsets
(the cache is 1.07 GB per tensor) and the config-5 work split over the
persistent grid.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import bench
from oracle import attention as oattn

pytestmark = pytest.mark.gpu

TOL_BF16 = 2e-2


def _run_config(dev, base, batch, n_sample, sample_seed, alpha=None):
    from wavefront_decoding_b200 import attention as wa
    from wavefront_decoding_b200 import runtime as rt
    from wavefront_decoding_b200.kv_cache import SlotKVCache
    c, q, K, V, _, _, items, acc = bench.cfg3_device_inputs(dev, base["seed"], batch, base, alpha)
    W, L0 = c["W"], c["L0"]
    g = torch.Generator(device=dev).manual_seed(1000 + base["seed"])
    kn = torch.randn((q.shape[0], c["Hkv"], c["Dh"]), generator=g, device=dev, dtype=torch.bfloat16)
    vn = torch.randn((q.shape[0], c["Hkv"], c["Dh"]), generator=g, device=dev, dtype=torch.bfloat16)
    sample = sorted(np.random.default_rng(sample_seed).choice(len(items), n_sample, replace=False).tolist())
    before = {i: (K[items[i][0], items[i][1], :items[i][2]].cpu(), V[items[i][0], items[i][1], :items[i][2]].cpu())
              for i in sample}
    cache = SlotKVCache.wrap(K, V)
    cache.lens.copy_(torch.tensor([[L0 - r] * c["B"] for r in range(c["R"])], dtype=torch.int32))
    itd = torch.tensor(items, dtype=torch.int32, device=dev)
    out = wa.wave_attn(q, kn, vn, K, V, itd, W, lens=cache.lens)
    torch.cuda.synchronize()
    assert rt.read_device_error(dev) == 0
    # every slot length rose to the end of its window
    lens = cache.lens.cpu()
    for r, b, p0, ql, _ in items:
        assert int(lens[r, b]) == p0 + ql
    # every appended row, bit for bit
    idx_r = torch.tensor([r for r, b, p, w, _ in items for j in range(w)], device=dev)
    idx_b = torch.tensor([b for r, b, p, w, _ in items for j in range(w)], device=dev)
    idx_p = torch.tensor([p + j for r, b, p, w, _ in items for j in range(w)], device=dev)
    assert torch.equal(K[idx_r, idx_b, idx_p], kn) and torch.equal(V[idx_r, idx_b, idx_p], vn)
    # sampled items against the oracle, over the untouched prefix plus the window
    worst = 0.0
    out_h = out.float().cpu().numpy()
    for i in sample:
        r, b, p0, ql, row = items[i]
        kp, vp = before[i]
        assert torch.equal(K[r, b, :p0].cpu(), kp)  # the prefix was read in place, never written
        kfull = torch.cat([kp, kn[row:row + ql].cpu()])
        vfull = torch.cat([vp, vn[row:row + ql].cpu()])
        ref = oattn.attn_varlen(q[row:row + ql].cpu(), kfull, vfull, [0, ql], [0, p0 + ql], causal=True)
        worst = max(worst, float(np.abs(out_h[row:row + ql] - ref).max()))
    assert worst < TOL_BF16, worst
    # accept commit: lengths pos0 + a_b, accepted rows kept in place (a prefix of each window)
    acc_rows, acc_cnt = cache.commit_window(itd, accept_len=acc, n_rows=q.shape[0])
    torch.cuda.synchronize()
    assert rt.read_device_error(dev) == 0
    a = acc.cpu().tolist()
    assert acc_cnt.cpu().tolist() == a
    lens = cache.lens.cpu()
    rows = acc_rows.cpu().tolist()
    for i, (r, b, p0, ql, row) in enumerate(items):
        assert int(lens[r, b]) == p0 + a[i]
        assert rows[row:row + a[i]] == list(range(row, row + a[i]))
    for i in sample:
        r, b, p0, ql, row = items[i]
        assert torch.equal(K[r, b, p0:p0 + a[i]].cpu(), kn[row:row + a[i]].cpu())
        assert torch.equal(V[r, b, p0:p0 + a[i]].cpu(), vn[row:row + a[i]].cpu())
    return c, a, items


def test_cfg3_full_geometry_vs_oracle(cuda_dev):
    c, a, items = _run_config(cuda_dev, bench.CFG3, None, 16, 2)
    assert c["B"] == 32 and c["R"] == 8 and c["H"] == 32 and c["Hkv"] == 8 and len(items) == 256
    # accepted lengths: U{0..8} from seed 3, one per sequence, the same in every slot
    accept = torch.randint(0, 9, (32,), generator=torch.Generator().manual_seed(3)).tolist()
    assert a == [accept[b] for _, b, _, _, _ in items]


@pytest.mark.parametrize("alpha", [0.5, 0.8])
def test_cfg5_geometry_small_batch_vs_oracle(cuda_dev, alpha):
    c, a, _ = _run_config(cuda_dev, bench.CFG5, 2, 6, 5, alpha=alpha)
    assert c["R"] == 16 and c["L0"] == 32768 and c["B"] == 2
    torch.cuda.empty_cache()
