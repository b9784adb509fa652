"""Fused looped-LM block kernels (RMSNorm, RoPE + QKV split, SwiGLU gate)
against plain fp32 torch arithmetic of the same op."""
from __future__ import annotations

import pytest
import torch

import golden_inputs as gi

pytestmark = pytest.mark.gpu


def _tol(dt):
    return 1e-5 if dt == torch.float32 else 2e-2


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("n,d", [(1, 256), (37, 512), (200, 1536)])
def test_rmsnorm(cuda_dev, dt, n, d):
    from wavefront_decoding_b200 import fused
    g = gi.gen(31)
    x = (torch.randn((n, d), generator=g) * 3).to(dt).to(cuda_dev)
    w = (torch.rand((d,), generator=g) + 0.5).to(dt).to(cuda_dev)
    y = fused.rmsnorm(x, w, 1e-6)
    xf = x.float()
    ref = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6) * w.float()
    assert (y.float() - ref).abs().max().item() <= _tol(dt) * max(1.0, ref.abs().max().item())


def _rope_ref(x, pos, cos, sin, interleaved):
    xf = x.float()
    c, s = cos[pos][:, None, :], sin[pos][:, None, :]
    if interleaved:
        a, b = xf[..., 0::2], xf[..., 1::2]
        return torch.stack((a * c - b * s, a * s + b * c), dim=-1).flatten(-2)
    h = x.shape[-1] // 2
    a, b = xf[..., :h], xf[..., h:]
    return torch.cat((a * c - b * s, b * c + a * s), dim=-1)


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("interleaved", [False, True])
@pytest.mark.parametrize("H,Hkv,Dh", [(8, 8, 64), (16, 4, 128), (24, 24, 64)])
def test_rope_split(cuda_dev, dt, interleaved, H, Hkv, Dh):
    from wavefront_decoding_b200 import fused
    g = gi.gen(32)
    n, S = 45, 300
    qkv = torch.randn((n, (H + 2 * Hkv) * Dh), generator=g).to(dt).to(cuda_dev)
    inv = 1.0 / (10000.0 ** (torch.arange(0, Dh, 2, dtype=torch.float64) / Dh))
    ang = torch.outer(torch.arange(S, dtype=torch.float64), inv)
    cos, sin = ang.cos().float().to(cuda_dev), ang.sin().float().to(cuda_dev)
    # positions as a strided column of an int32 table (as the engine passes them)
    tab = torch.randint(0, S, (n, 3), generator=g, dtype=torch.int32).to(cuda_dev)
    pos = tab[:, 1]
    q, k, v = fused.rope_split(qkv, cos, sin, H, Hkv, Dh, pos=pos, interleaved=interleaved)
    qs, ks, vs = torch.split(qkv, [H * Dh, Hkv * Dh, Hkv * Dh], dim=-1)
    pl = pos.long()
    tol = _tol(dt) * 4
    assert (q.float() - _rope_ref(qs.reshape(n, H, Dh), pl, cos, sin, interleaved)).abs().max().item() <= tol
    assert (k.float() - _rope_ref(ks.reshape(n, Hkv, Dh), pl, cos, sin, interleaved)).abs().max().item() <= tol
    assert torch.equal(v, vs.reshape(n, Hkv, Dh))
    # period form: rows are L consecutive positions per sequence
    L = 9
    q2, k2, _ = fused.rope_split(qkv, cos, sin, H, Hkv, Dh, pos_period=L, interleaved=interleaved)
    pp = torch.arange(n, device=cuda_dev) % L
    assert (q2.float() - _rope_ref(qs.reshape(n, H, Dh), pp, cos, sin, interleaved)).abs().max().item() <= tol


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
def test_silu_mul(cuda_dev, dt):
    from wavefront_decoding_b200 import fused
    g = gi.gen(33)
    gu = (torch.randn((70, 2 * 4096), generator=g) * 2).to(dt).to(cuda_dev)
    out = fused.silu_mul(gu)
    a, b = gu.float().split(4096, dim=-1)
    ref = torch.nn.functional.silu(a) * b
    assert (out.float() - ref).abs().max().item() <= _tol(dt) * max(1.0, ref.abs().max().item())


def test_rope_bad_position_sets_error(cuda_dev):
    from wavefront_decoding_b200 import _abi, fused
    from wavefront_decoding_b200 import runtime as rt
    assert rt.read_device_error(cuda_dev) == 0
    qkv = torch.zeros((2, 3 * 64), device=cuda_dev)
    cos = torch.ones((4, 32), device=cuda_dev)
    sin = torch.zeros((4, 32), device=cuda_dev)
    pos = torch.tensor([1, 7], dtype=torch.int32, device=cuda_dev)   # 7 >= 4 table rows
    fused.rope_split(qkv, cos, sin, 1, 1, 64, pos=pos)
    with pytest.raises(_abi.WfdError):
        rt.read_device_error(cuda_dev)           # reads and clears the word
    assert rt.read_device_error(cuda_dev) == 0


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
def test_row_plumbing(cuda_dev, dt):
    from wavefront_decoding_b200 import fused
    g = gi.gen(34)
    a = torch.randn((50, 256), generator=g).to(dt).to(cuda_dev)
    b = torch.randn((50, 256), generator=g).to(dt).to(cuda_dev)
    tab = torch.randint(0, 50, (17, 3), generator=g, dtype=torch.int32).to(cuda_dev)
    idx = tab[:, 1]                                    # strided int32 column
    il = idx.long()
    assert torch.equal(fused.gather_rows(a, idx), a[il])
    assert torch.equal(fused.gather_rows(a, idx, b=b), (a.float()[il] + b.float()[il]).to(dt))
    uniq = torch.randperm(50, generator=g)[:17].to(torch.int32).to(cuda_dev)
    dst, zero = a.clone(), b.clone()
    src = torch.randn((17, 256), generator=g).to(dt).to(cuda_dev)
    fused.scatter_rows(src, uniq, dst, zero=zero)
    ref_d, ref_z = a.clone(), b.clone()
    ref_d[uniq.long()] = src
    ref_z[uniq.long()] = 0
    assert torch.equal(dst, ref_d) and torch.equal(zero, ref_z)


def test_items_from_table_and_argmax(cuda_dev):
    from wavefront_decoding_b200 import fused
    g = gi.gen(35)
    tab = torch.randint(0, 1000, (33, 8), generator=g, dtype=torch.int32).to(cuda_dev)
    items = torch.empty((33, 5), dtype=torch.int32, device=cuda_dev)
    fused.items_from_table(tab, 4, 3, 1, 5, items)
    ref = torch.stack([tab[:, 4], tab[:, 3], tab[:, 1], tab[:, 5],
                       torch.arange(33, dtype=torch.int32, device=cuda_dev)], dim=1)
    assert torch.equal(items, ref)
    for dt in (torch.float32, torch.bfloat16):
        x = torch.randn((9, 50304), generator=g).to(dt).to(cuda_dev)
        x[3, 100] = x[3, 2000] = x[3].max() + 1        # a tie: the first index wins, as torch.argmax
        out = torch.empty(9, dtype=torch.int32, device=cuda_dev)
        fused.argmax_rows(x, out)
        assert torch.equal(out.long(), x.float().argmax(dim=-1))
        assert int(out[3]) == 100
    # vector path (V % 8 == 0, aligned), scalar path (odd V, or a row base off
    # the 16-byte boundary), ties inside one 8-element vector and across the
    # unrolled loads, and the maximum at the last element
    for dt in (torch.float32, torch.bfloat16):
        for V in (8, 7, 4104, 40000, 50303):
            base = torch.randn(5 * V + 1, generator=g).to(dt).to(cuda_dev)
            for x in (base[:5 * V].view(5, V), base[1:].view(5, V)):
                x[0, V - 1] = x[0].max() + 1
                m = x[1].max() + 1
                x[1, min(3, V - 1)] = x[1, min(5, V - 1)] = x[1, V // 2] = m
                x[2, V // 3] = x[2, V - 1] = x[2].max() + 1
                out = torch.empty(5, dtype=torch.int32, device=cuda_dev)
                fused.argmax_rows(x, out)
                assert torch.equal(out.long(), x.float().argmax(dim=-1)), (dt, V, x.data_ptr() % 16)


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("n", [1, 7, 64, 300])
@pytest.mark.parametrize("interleaved", [False, True])
def test_rope_split_with_folded_norm(cuda_dev, dt, n, interleaved):
    """wfd_rope_split_norm: rope_split of s_r * qkv_r, s_r = rsqrt(mean(x_r^2) + eps)
    from the pre-norm rows x (a strided view), against fp32 torch."""
    from wavefront_decoding_b200 import fused
    g = gi.gen(33)
    H, Hkv, Dh, d, S = 8, 4, 64, 512, 300
    qkv = torch.randn((n, (H + 2 * Hkv) * Dh), generator=g).to(dt).to(cuda_dev)
    xbig = (torch.randn((n, d + 64), generator=g) * 3).to(dt).to(cuda_dev)
    x = xbig[:, :d]                                   # row stride d + 64
    inv = 1.0 / (10000.0 ** (torch.arange(0, Dh, 2, dtype=torch.float64) / Dh))
    ang = torch.outer(torch.arange(S, dtype=torch.float64), inv)
    cos, sin = ang.cos().float().to(cuda_dev), ang.sin().float().to(cuda_dev)
    pos = torch.randint(0, S, (n,), generator=g, dtype=torch.int32).to(cuda_dev)
    q, k, v = fused.rope_split(qkv, cos, sin, H, Hkv, Dh, pos=pos, interleaved=interleaved, norm_x=x,
                               norm_eps=1e-6)
    xf = x.float()
    sc = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6)
    y = qkv.float() * sc
    pl = pos.long()
    tol = _tol(dt) * 4
    ref_q = _rope_ref(y[:, :H * Dh].view(n, H, Dh), pl, cos, sin, interleaved)
    ref_k = _rope_ref(y[:, H * Dh:(H + Hkv) * Dh].view(n, Hkv, Dh), pl, cos, sin, interleaved)
    ref_v = y[:, (H + Hkv) * Dh:].view(n, Hkv, Dh)
    for got, ref in ((q, ref_q), (k, ref_k), (v, ref_v)):
        assert (got.float() - ref).abs().max().item() <= tol * max(1.0, ref.abs().max().item())


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("n", [1, 9, 300])
def test_silu_mul_with_folded_norm(cuda_dev, dt, n):
    from wavefront_decoding_b200 import fused
    g = gi.gen(34)
    dff, d = 1536, 512
    gu = torch.randn((n, 2 * dff), generator=g).to(dt).to(cuda_dev)
    x = (torch.randn((n, d), generator=g) * 2).to(dt).to(cuda_dev)
    out = fused.silu_mul(gu, norm_x=x, norm_eps=1e-6)
    sc = torch.rsqrt(x.float().pow(2).mean(-1, keepdim=True) + 1e-6)
    gg, uu = gu.float()[:, :dff] * sc, gu.float()[:, dff:] * sc
    ref = torch.nn.functional.silu(gg) * uu
    assert (out.float() - ref).abs().max().item() <= _tol(dt) * 4 * max(1.0, ref.abs().max().item())


def test_folded_norm_model_matches_explicit_norm(cuda_dev):
    """The bf16 looped LM with folded norms against the same model with explicit
    RMSNorm launches: q / k / v and the block output agree within bf16 rounding."""
    from wavefront_decoding_b200.looped_lm import LoopedLM, LoopedLMConfig
    cfg = LoopedLMConfig(vocab=512, d_model=256, n_heads=4, n_kv_heads=2, head_dim=64, d_ff=512, n_prelude=1,
                         n_core=2, n_coda=1, T_total=4)
    m = LoopedLM(cfg, seed=3, dtype=torch.bfloat16, device="cuda")
    assert m.fold_norms
    m.rope_tables(64)
    blk = m.core[0]
    blk.norm1 = (torch.rand(cfg.d_model, generator=gi.gen(35)) + 0.5).to(torch.bfloat16).to(cuda_dev)
    blk.norm2 = (torch.rand(cfg.d_model, generator=gi.gen(36)) + 0.5).to(torch.bfloat16).to(cuda_dev)
    m._fold()
    x = torch.randn((10, cfg.d_model), generator=gi.gen(37)).to(torch.bfloat16).to(cuda_dev)
    pos = torch.arange(10, dtype=torch.int32, device=cuda_dev) * 3
    folded = m.qkv(blk, x, pos=pos)
    attn = torch.randn((10, cfg.n_heads, cfg.head_dim), generator=gi.gen(38)).to(torch.bfloat16).to(cuda_dev)
    out_f = m.finish_block(blk, x.clone(), attn)
    m.fold_norms = False
    explicit = m.qkv(blk, x, pos=pos)
    out_e = m.finish_block(blk, x.clone(), attn)
    for a, b in zip(folded, explicit):
        assert (a.float() - b.float()).abs().max().item() <= 3e-2 * max(1.0, b.float().abs().max().item())
    assert (out_f.float() - out_e.float()).abs().max().item() <= 3e-2 * max(1.0, out_e.float().abs().max().item())
