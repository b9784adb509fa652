"""The fused skinny linear kernel (wfd_linear, tcgen05) against plain fp32 torch
arithmetic of the same op: RMSNorm (weight folded into W) -> x @ W, then the
plain / residual / SwiGLU / RoPE + split epilogues, at the looped-LM shapes of
configs 1 and 4 and a GQA head_dim-128 shape, row counts 1 .. 100 (one to two
row blocks, one and several k ranges per feature tile).  bf16 storage, fp32
accumulation; tolerance 2e-2 x max(1, |ref|max).  Also: a row's bits do not
depend on the other rows of the call, and repeated calls are identical."""
from __future__ import annotations

import pytest
import torch

import golden_inputs as gi

pytestmark = pytest.mark.gpu

TOL = 2e-2
EPS = 1e-6


def _close(y, ref):
    err = (y.float() - ref).abs().max().item()
    assert err <= TOL * max(1.0, ref.abs().max().item()), err


def _inputs(dev, n, K, F, seed, std=0.02):
    g = gi.gen(seed)
    x = (torch.randn((n, K), generator=g) * 2).to(torch.bfloat16).to(dev)
    w = (torch.randn((K, F), generator=g) * std).to(torch.bfloat16).to(dev)
    norm = (torch.rand((K,), generator=g) + 0.5).to(torch.bfloat16).to(dev)
    return x, w, norm


def _normed(x, norm):
    xf = x.float()
    return xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + EPS) * norm.float()


ROWS = [1, 5, 16, 17, 40, 64, 100]


@pytest.mark.parametrize("n", ROWS)
@pytest.mark.parametrize("K,F", [(1536, 1536), (512, 1536), (1536, 50304), (4096, 1536)])
def test_plain_and_row_norm(cuda_dev, n, K, F):
    from wavefront_decoding_b200 import fused
    x, w, norm = _inputs(cuda_dev, n, K, F, 40 + n)
    _close(fused.linear(x, w), x.float() @ w.float())
    y = fused.linear(x, fused.fold_norm(w, norm), norm_eps=EPS)
    _close(y, _normed(x, norm) @ w.float())


@pytest.mark.parametrize("n", ROWS)
@pytest.mark.parametrize("K,F", [(1536, 1536), (4096, 1536), (512, 512)])
def test_residual(cuda_dev, n, K, F):
    from wavefront_decoding_b200 import fused
    x, w, _ = _inputs(cuda_dev, n, K, F, 50 + n)
    res = torch.randn((n, F), generator=gi.gen(51)).to(torch.bfloat16).to(cuda_dev)
    ref = res.float() + x.float() @ w.float()
    out = res.clone()
    fused.linear_residual(x, w, out)
    _close(out, ref)


@pytest.mark.parametrize("n", ROWS)
@pytest.mark.parametrize("K,dff", [(1536, 4096), (512, 1536)])
def test_swiglu(cuda_dev, n, K, dff):
    from wavefront_decoding_b200 import fused
    x, w, norm = _inputs(cuda_dev, n, K, 2 * dff, 60 + n)
    gu = (_normed(x, norm) @ w.float()).to(torch.bfloat16).float()   # the unfused chain stores gu in bf16
    g, u = gu[:, :dff], gu[:, dff:]
    ref = torch.nn.functional.silu(g) * u
    y = fused.linear_swiglu(x, fused.interleave_gate_up(fused.fold_norm(w, norm)), norm_eps=EPS)
    assert y.shape == (n, dff)
    _close(y, ref)


def _rope_ref(y, pos, cos, sin, interleaved):
    c, s = cos[pos][:, None, :], sin[pos][:, None, :]
    if interleaved:
        a, b = y[..., 0::2], y[..., 1::2]
        return torch.stack((a * c - b * s, a * s + b * c), dim=-1).flatten(-2)
    h = y.shape[-1] // 2
    a, b = y[..., :h], y[..., h:]
    return torch.cat((a * c - b * s, b * c + a * s), dim=-1)


@pytest.mark.parametrize("n", [1, 17, 64, 100])
@pytest.mark.parametrize("interleaved", [False, True])
@pytest.mark.parametrize("K,H,Hkv,Dh", [(1536, 24, 24, 64), (512, 8, 8, 64), (1024, 16, 4, 128)])
def test_rope_split(cuda_dev, n, interleaved, K, H, Hkv, Dh):
    from wavefront_decoding_b200 import fused
    F = (H + 2 * Hkv) * Dh
    x, w, norm = _inputs(cuda_dev, n, K, F, 70 + n)
    S = 2048
    inv = 1.0 / (10000.0 ** (torch.arange(0, Dh, 2, dtype=torch.float64) / Dh))
    ang = torch.outer(torch.arange(S, dtype=torch.float64), inv)
    cos, sin = ang.cos().float().to(cuda_dev), ang.sin().float().to(cuda_dev)
    tab = torch.randint(0, S, (n, 6), generator=gi.gen(71), dtype=torch.int32).to(cuda_dev)
    pos = tab[:, 1]                                                    # a strided column, as the engine passes
    q, k, v = fused.linear_rope(x, fused.fold_norm(w, norm), cos, sin, H, Hkv, Dh, pos=pos,
                                interleaved=interleaved, norm_eps=EPS)
    y = (_normed(x, norm) @ w.float()).to(torch.bfloat16).float()     # the unfused chain stores qkv in bf16
    pl = pos.long()
    qr = _rope_ref(y[:, :H * Dh].view(n, H, Dh), pl, cos, sin, interleaved)
    kr = _rope_ref(y[:, H * Dh:(H + Hkv) * Dh].view(n, Hkv, Dh), pl, cos, sin, interleaved)
    vr = y[:, (H + Hkv) * Dh:].view(n, Hkv, Dh)
    _close(q, qr)
    _close(k, kr)
    _close(v, vr)
    # prompt rows: position r % period
    q2, _, _ = fused.linear_rope(x, fused.fold_norm(w, norm), cos, sin, H, Hkv, Dh, pos_period=7,
                                 interleaved=interleaved, norm_eps=EPS)
    _close(q2, _rope_ref(y[:, :H * Dh].view(n, H, Dh), torch.arange(n, device=cuda_dev) % 7, cos, sin, interleaved))


def test_rows_independent_and_repeatable(cuda_dev):
    """Row r's output bits are the same whatever the other rows of the call
    (16-, 32- and 64-column MMAs, one or two row blocks), and for repeated calls."""
    from wavefront_decoding_b200 import fused
    x, w, norm = _inputs(cuda_dev, 100, 1536, 4608, 80)
    wf = fused.fold_norm(w, norm)
    full = fused.linear(x, wf, norm_eps=EPS)
    assert torch.equal(full, fused.linear(x, wf, norm_eps=EPS))
    for n in (5, 16, 17, 33, 64):
        assert torch.equal(fused.linear(x[:n].contiguous(), wf, norm_eps=EPS), full[:n]), n
    # residual and SwiGLU modes too
    res = torch.randn((100, 1536), generator=gi.gen(81)).to(torch.bfloat16).to(cuda_dev)
    a = res.clone()
    fused.linear_residual(x, w[:, :1536].contiguous(), a)
    b = res[:9].clone()
    fused.linear_residual(x[:9].contiguous(), w[:, :1536].contiguous(), b)
    assert torch.equal(a[:9], b)


def test_bad_position_sets_error_bit(cuda_dev):
    """A position outside the cos / sin tables is caught by the kernel's bounds
    check (error bit, position 0 used), never read out of bounds."""
    from wavefront_decoding_b200 import _abi, fused
    from wavefront_decoding_b200 import runtime as rt
    H, Hkv, Dh, K = 8, 8, 64, 512
    x, w, _ = _inputs(cuda_dev, 4, K, (H + 2 * Hkv) * Dh, 91)
    cos = torch.ones((16, Dh // 2), device=cuda_dev)
    sin = torch.zeros((16, Dh // 2), device=cuda_dev)
    rt.read_device_error(cuda_dev)
    pos = torch.tensor([0, 3, 40, 5], dtype=torch.int32, device=cuda_dev)
    fused.linear_rope(x, w, cos, sin, H, Hkv, Dh, pos=pos)
    with pytest.raises(_abi.WfdError):
        rt.read_device_error(cuda_dev)
    assert rt.read_device_error(cuda_dev) == 0
