"""Fused block helpers of the looped LM on libwfd_b200 (CUDA tensors only).

rmsnorm     one launch per call instead of up-cast / pow / mean / rsqrt / mul / down-cast
rope_split  fused-QKV output -> contiguous q, k (RoPE at per-row positions) and v
silu_mul    SwiGLU gate silu(g) * u
gather_rows / scatter_rows / items_from_table / argmax_rows: state-pool row
            plumbing and greedy ids by int32 indices (no int64 index tensors)
All arithmetic is fp32; storage bf16 or fp32.  No CPU path: CPU tensors raise.
"""
from __future__ import annotations

import torch

from . import _abi
from . import runtime as rt


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float, out: torch.Tensor | None = None) -> torch.Tensor:
    """x (..., d) contiguous; returns x * rsqrt(mean(x^2) + eps) * w."""
    dev = rt.require_cuda(x, w)
    d = x.shape[-1]
    if not x.is_contiguous():
        x = x.contiguous()
    if out is None:
        out = torch.empty_like(x)
    n = x.numel() // d if d else 0
    st = _abi.load().wfd_rmsnorm(x.data_ptr(), w.data_ptr(), out.data_ptr(), n, d, float(eps),
                                 rt.dtype_code(x.dtype), rt.stream_ptr(dev))
    _abi.check(st, "wfd_rmsnorm")
    return out


def rope_split(qkv: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, n_heads: int, n_kv_heads: int, head_dim: int,
               *, pos: torch.Tensor | None = None, pos_period: int = 0, interleaved: bool = False):
    """qkv (n, (H + 2 Hkv) Dh) -> q (n, H, Dh), k (n, Hkv, Dh) rotated, v (n, Hkv, Dh).

    pos: int32 positions, one per row (a strided column view is fine), or None
    with pos_period = L for rows that are L consecutive positions per sequence."""
    dev = rt.require_cuda(qkv, cos, sin)
    n = qkv.shape[0]
    if not qkv.is_contiguous():
        qkv = qkv.contiguous()
    assert qkv.shape[1] == (n_heads + 2 * n_kv_heads) * head_dim
    assert cos.dtype == torch.float32 and sin.dtype == torch.float32 and cos.is_contiguous() and sin.is_contiguous()
    q = torch.empty((n, n_heads, head_dim), dtype=qkv.dtype, device=dev)
    k = torch.empty((n, n_kv_heads, head_dim), dtype=qkv.dtype, device=dev)
    v = torch.empty((n, n_kv_heads, head_dim), dtype=qkv.dtype, device=dev)
    if pos is not None:
        assert pos.dtype == torch.int32 and pos.dim() == 1 and pos.shape[0] >= n
        pptr, pstride = pos.data_ptr(), pos.stride(0)
    else:
        assert pos_period > 0
        pptr, pstride = None, 0
    st = _abi.load().wfd_rope_split(qkv.data_ptr(), cos.data_ptr(), sin.data_ptr(), pptr, pstride, pos_period,
                                    cos.shape[0], q.data_ptr(), k.data_ptr(), v.data_ptr(), n, n_heads, n_kv_heads,
                                    head_dim, 1 if interleaved else 0, rt.dtype_code(qkv.dtype),
                                    rt.error_word(dev).data_ptr(), rt.stream_ptr(dev))
    _abi.check(st, "wfd_rope_split")
    return q, k, v


def silu_mul(gu: torch.Tensor) -> torch.Tensor:
    """gu (..., 2 dff) = [g | u] -> silu(g) * u (..., dff)."""
    dev = rt.require_cuda(gu)
    if not gu.is_contiguous():
        gu = gu.contiguous()
    dff = gu.shape[-1] // 2
    out = torch.empty((*gu.shape[:-1], dff), dtype=gu.dtype, device=dev)
    n = gu.numel() // (2 * dff) if dff else 0
    st = _abi.load().wfd_silu_mul(gu.data_ptr(), out.data_ptr(), n, dff, rt.dtype_code(gu.dtype), rt.stream_ptr(dev))
    _abi.check(st, "wfd_silu_mul")
    return out


def _idx(idx: torch.Tensor):
    assert idx.dtype == torch.int32 and idx.dim() == 1
    return idx.data_ptr(), idx.stride(0)


def gather_rows(a: torch.Tensor, idx: torch.Tensor, b: torch.Tensor | None = None,
                out: torch.Tensor | None = None) -> torch.Tensor:
    """out[i] = a[idx[i]] (+ b[idx[i]]); a, b (rows, d) contiguous, idx int32 (n,) (strided ok)."""
    dev = rt.require_cuda(a, idx, b)
    n, d = idx.shape[0], a.shape[1]
    if out is None:
        out = torch.empty((n, d), dtype=a.dtype, device=dev)
    ip, istr = _idx(idx)
    st = _abi.load().wfd_gather_rows(a.data_ptr(), None if b is None else b.data_ptr(), ip, istr, out.data_ptr(), n,
                                     d, a.shape[0], rt.dtype_code(a.dtype), rt.error_word(dev).data_ptr(),
                                     rt.stream_ptr(dev))
    _abi.check(st, "wfd_gather_rows")
    return out


def scatter_rows(src: torch.Tensor, idx: torch.Tensor, dst: torch.Tensor, zero: torch.Tensor | None = None) -> None:
    """dst[idx[i]] = src[i] (and zero[idx[i]] = 0)."""
    dev = rt.require_cuda(src, idx, dst, zero)
    if not src.is_contiguous():
        src = src.contiguous()
    ip, istr = _idx(idx)
    st = _abi.load().wfd_scatter_rows(src.data_ptr(), ip, istr, dst.data_ptr(),
                                      None if zero is None else zero.data_ptr(), idx.shape[0], dst.shape[1],
                                      dst.shape[0], rt.dtype_code(dst.dtype), rt.error_word(dev).data_ptr(),
                                      rt.stream_ptr(dev))
    _abi.check(st, "wfd_scatter_rows")


def items_from_table(tab: torch.Tensor, c_slot: int, c_seq: int, c_pos: int, c_qlen: int,
                     items: torch.Tensor) -> None:
    """items[i] = (tab[i, c_slot], tab[i, c_seq], tab[i, c_pos], tab[i, c_qlen], i)."""
    dev = rt.require_cuda(tab, items)
    assert tab.dtype == torch.int32 and tab.is_contiguous() and items.shape == (tab.shape[0], 5)
    st = _abi.load().wfd_items_from_table(tab.data_ptr(), tab.shape[1], c_slot, c_seq, c_pos, c_qlen,
                                          items.data_ptr(), tab.shape[0], rt.stream_ptr(dev))
    _abi.check(st, "wfd_items_from_table")


def argmax_rows(x: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    """out[r] = first index of the maximum of x[r] (int32), x (n, V) contiguous."""
    dev = rt.require_cuda(x, out)
    assert x.is_contiguous() and out.dtype == torch.int32
    st = _abi.load().wfd_argmax_rows(x.data_ptr(), out.data_ptr(), x.shape[0], x.shape[1], rt.dtype_code(x.dtype),
                                     rt.stream_ptr(dev))
    _abi.check(st, "wfd_argmax_rows")
    return out

