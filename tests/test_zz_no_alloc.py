"""The no-allocation entry point (wfd_wave_attn_static) against the regular one.

wfd_wave_attn_static exists for callers that cannot allocate device memory at
call time (serving runtimes with a memory plan fixed at start-up, where an
allocation mid-request can synchronise the device or fail under memory
pressure; foreign-language hosts that hold device pointers but no device
allocator): it runs the same tensor-core wavefront kernel on a fixed array
inside the library instead of a caller workspace.  This test calls both entry
points through the C ABI on identical inputs, twice in a row with different
shapes (the second call must not be disturbed by what the first left in the
shared array), and requires the same outputs (and both within the bf16
tolerance of the float64 oracle), appended K/V rows and slot lengths; the
device's free memory does not move across the second call.  It lives in its own
file, collected last.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

import golden_inputs as gi
from oracle.kv_cache import SlotCacheOracle

pytestmark = pytest.mark.gpu

TOL_BF16 = 2e-2


def _inputs(seed, n_slots, B, S, H, Hkv, items):
    g = gi.gen(seed)
    K = gi.randn((n_slots, B, S, Hkv, 128), g, torch.bfloat16)
    V = gi.randn((n_slots, B, S, Hkv, 128), g, torch.bfloat16)
    n_rows = max(it[4] + it[3] for it in items)
    q = gi.randn((n_rows, H, 128), g, torch.bfloat16)
    kn = gi.randn((n_rows, Hkv, 128), g, torch.bfloat16)
    vn = gi.randn((n_rows, Hkv, 128), g, torch.bfloat16)
    return K, V, q, kn, vn


def _call(lib, fn_name, dev, K, V, q, kn, vn, items, max_q, H, Hkv, ws=None):
    from wavefront_decoding_b200 import runtime as rt
    Kd, Vd = K.to(dev).contiguous(), V.to(dev).contiguous()
    qd, knd, vnd = q.to(dev), kn.to(dev), vn.to(dev)
    out = torch.zeros_like(qd)
    lens = torch.zeros(K.shape[:2], dtype=torch.int32, device=dev)
    it = torch.tensor(items, dtype=torch.int32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    n_slots, B, S = K.shape[:3]
    common = (qd.data_ptr(), knd.data_ptr(), vnd.data_ptr(), Kd.data_ptr(), Vd.data_ptr(), out.data_ptr(),
              lens.data_ptr(), it.data_ptr(), len(items), max_q, 0, qd.shape[0], n_slots, B, S, H, Hkv, 128, 0, 0.0)
    stream = rt.stream_ptr(dev)
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info(dev)[0]
    if fn_name == "wfd_wave_attn_static":
        st = lib.wfd_wave_attn_static(*common, err.data_ptr(), stream)
    else:
        st = lib.wfd_wave_attn(*common, ws[0].data_ptr(), ws[1], err.data_ptr(), stream)
    assert st == 0, st
    torch.cuda.synchronize()
    free1 = torch.cuda.mem_get_info(dev)[0]
    assert int(err.item()) == 0
    return out, Kd, Vd, lens, free0 - free1


def test_static_entry_point_matches_regular(cuda_dev):
    from wavefront_decoding_b200 import _abi
    from wavefront_decoding_b200 import runtime as rt
    lib = _abi.load()
    rng = np.random.default_rng(11)
    calls = [
        # call 1: decode rows of a wave over 4 slots x 6 sequences, GQA 4:1
        (41, 4, 6, 1024, 16, 4, [[r, b, int(rng.integers(0, 1000)), 1, r * 6 + b] for r in range(4) for b in range(6)], 1),
        # call 2: 8-row verify windows, GQA 4:1 with 32 query heads, other sizes
        (42, 3, 5, 2100, 32, 8, [[r, b, 2000 - 37 * r - b, 8, (r * 5 + b) * 8] for r in range(3) for b in range(5)], 8),
    ]
    ws = rt.workspace(cuda_dev, 64, 128)
    for k, (seed, n_slots, B, S, H, Hkv, items, max_q) in enumerate(calls):
        K, V, q, kn, vn = _inputs(seed, n_slots, B, S, H, Hkv, items)
        out_s, Ks, Vs, lens_s, used = _call(lib, "wfd_wave_attn_static", cuda_dev, K, V, q, kn, vn, items, max_q, H,
                                            Hkv)
        if k > 0:
            assert used == 0, used  # nothing allocated on the device by the call
        out_r, Kr, Vr, lens_r, _ = _call(lib, "wfd_wave_attn", cuda_dev, K, V, q, kn, vn, items, max_q, H, Hkv,
                                         ws=ws)
        diff = float((out_s.float() - out_r.float()).abs().max())
        assert diff < TOL_BF16, diff
        assert float(out_s.float().abs().max()) > 0.0
        assert torch.equal(Ks, Kr) and torch.equal(Vs, Vr)
        assert torch.equal(lens_s, lens_r)
        # and both against the float64 oracle of the reference semantics
        o = SlotCacheOracle(n_slots, B, Hkv, 128, S)
        o.K[:] = K.float().numpy()
        o.V[:] = V.float().numpy()
        ref = o.wave_attn(q.float().numpy(), kn.float().numpy(), vn.float().numpy(), items)
        assert float(np.abs(out_s.float().cpu().numpy() - ref).max()) < TOL_BF16
        assert np.array_equal(Ks.float().cpu().numpy(), o.K)


def test_static_entry_point_rejects_out_of_range(cuda_dev):
    from wavefront_decoding_b200 import _abi
    lib = _abi.load()
    null = ctypes.c_void_p(0)
    # fp32 is not served by the fixed-workspace variant; too many items neither
    assert lib.wfd_wave_attn_static(null, null, null, null, null, null, null, null, 1, 1, 0, 1, 1, 1, 1, 4, 4, 128, 1,
                                    0.0, null, null) == 2
    assert lib.wfd_wave_attn_static(null, null, null, null, null, null, null, null, 4097, 1, 0, 1, 1, 1, 1, 4, 4, 128,
                                    0, 0.0, null, null) == 3
