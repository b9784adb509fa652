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


def _norm_rows(norm_x: torch.Tensor, n: int):
    """(pointer, row stride, width) of the pre-norm rows x of a folded RMSNorm."""
    if norm_x.dim() != 2 or norm_x.shape[0] != n or norm_x.stride(1) != 1:
        raise ValueError(f"norm_x must be ({n}, d) rows with unit column stride, got {tuple(norm_x.shape)}")
    return norm_x.data_ptr(), norm_x.stride(0), norm_x.shape[1]


def rope_split(qkv: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, n_heads: int, n_kv_heads: int, head_dim: int,
               *, pos: torch.Tensor | None = None, pos_period: int = 0, interleaved: bool = False,
               norm_x: torch.Tensor | None = None, norm_eps: float = 0.0):
    """qkv (n, (H + 2 Hkv) Dh) -> q (n, H, Dh), k (n, Hkv, Dh) rotated, v (n, Hkv, Dh).

    pos: int32 positions, one per row (a strided column view is fine), or None
    with pos_period = L for rows that are L consecutive positions per sequence.
    norm_x: the rows x the QKV GEMM read when an RMSNorm is folded into its weight
    (fold_norm): every row of qkv is first scaled by rsqrt(mean(x^2) + norm_eps)."""
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
    if norm_x is not None:
        assert norm_x.dtype == qkv.dtype
        xp, ldx, d = _norm_rows(norm_x, n)
        st = _abi.load().wfd_rope_split_norm(qkv.data_ptr(), xp, ldx, d, float(norm_eps), cos.data_ptr(),
                                             sin.data_ptr(), pptr, pstride, pos_period, cos.shape[0], q.data_ptr(),
                                             k.data_ptr(), v.data_ptr(), n, n_heads, n_kv_heads, head_dim,
                                             1 if interleaved else 0, rt.dtype_code(qkv.dtype),
                                             rt.error_word(dev).data_ptr(), rt.stream_ptr(dev))
        _abi.check(st, "wfd_rope_split_norm")
        return q, k, v
    st = _abi.load().wfd_rope_split(qkv.data_ptr(), cos.data_ptr(), sin.data_ptr(), pptr, pstride, pos_period,
                                    cos.shape[0], q.data_ptr(), k.data_ptr(), v.data_ptr(), n, n_heads, n_kv_heads,
                                    head_dim, 1 if interleaved else 0, rt.dtype_code(qkv.dtype),
                                    rt.error_word(dev).data_ptr(), rt.stream_ptr(dev))
    _abi.check(st, "wfd_rope_split")
    return q, k, v


def silu_mul(gu: torch.Tensor, *, norm_x: torch.Tensor | None = None, norm_eps: float = 0.0) -> torch.Tensor:
    """gu (..., 2 dff) = [g | u] -> silu(g) * u (..., dff).  norm_x: the rows the
    gate/up GEMM read when an RMSNorm is folded into its weight (fold_norm): g and
    u are first scaled by rsqrt(mean(x^2) + norm_eps) of their row."""
    dev = rt.require_cuda(gu)
    if not gu.is_contiguous():
        gu = gu.contiguous()
    dff = gu.shape[-1] // 2
    out = torch.empty((*gu.shape[:-1], dff), dtype=gu.dtype, device=dev)
    n = gu.numel() // (2 * dff) if dff else 0
    if norm_x is not None:
        assert norm_x.dtype == gu.dtype
        xp, ldx, d = _norm_rows(norm_x, n)
        st = _abi.load().wfd_silu_mul_norm(gu.data_ptr(), xp, ldx, d, float(norm_eps), out.data_ptr(), n, dff,
                                           rt.dtype_code(gu.dtype), rt.stream_ptr(dev))
        _abi.check(st, "wfd_silu_mul_norm")
        return out
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



# ---------------------------------------------------------------------------
# skinny linear layers on the tensor cores (wfd_linear): a few rows times a
# weight matrix, with the block's RMSNorm / residual / SwiGLU / RoPE fused in
# ---------------------------------------------------------------------------
def fold_norm(w: torch.Tensor, norm: torch.Tensor) -> torch.Tensor:
    """W' = diag(norm) W (rows of W scaled by the RMSNorm weight), for a linear
    call with the row norm on: s_r x_r . W' == (x_r * s_r * norm) . W."""
    return (norm.float()[:, None] * w.float()).to(w.dtype).contiguous()


def interleave_gate_up(wgu: torch.Tensor) -> torch.Tensor:
    """(K, 2 dff) = [gate | up] -> columns interleaved per 64 (gate 64j.., then up
    64j..), the layout the SwiGLU mode of wfd_linear reads (dff % 64 == 0)."""
    K, two_dff = wgu.shape
    dff = two_dff // 2
    assert dff % 64 == 0
    return wgu.view(K, 2, dff // 64, 64).permute(0, 2, 1, 3).reshape(K, two_dff).contiguous()


def _linear(x: torch.Tensor, w: torch.Tensor, mode: int, *, out=None, norm_eps=None, q=None, k=None, v=None,
            rope=None) -> None:
    import ctypes
    dev = rt.require_cuda(x, w)
    if x.dtype != torch.bfloat16 or w.dtype != torch.bfloat16:
        raise TypeError("wfd_linear takes bf16 rows and weights")
    if x.dim() != 2 or w.dim() != 2 or x.shape[1] != w.shape[0] or x.stride(1) != 1 or not w.is_contiguous():
        raise ValueError(f"wfd_linear: x {tuple(x.shape)} (row-major rows) against W {tuple(w.shape)} (contiguous)")
    n, K = x.shape
    p = _abi.wfd_linear_params()
    p.x, p.w, p.ldx = x.data_ptr(), w.data_ptr(), x.stride(0)
    p.n_rows, p.K, p.F = n, K, w.shape[1]
    p.mode = mode
    p.row_norm = 0 if norm_eps is None else 1
    p.eps = 0.0 if norm_eps is None else float(norm_eps)
    if out is not None:
        if out.dtype != torch.bfloat16 or out.dim() != 2 or out.stride(1) != 1 or out.shape[0] != n:
            raise ValueError("wfd_linear: out must be bf16 (n_rows, width) rows")
        p.out, p.ldo = out.data_ptr(), out.stride(0)
    if rope is not None:
        cos, sin, H, Hkv, Dh, pos, pos_period, interleaved = rope
        p.q, p.k, p.v = q.data_ptr(), k.data_ptr(), v.data_ptr()
        p.cos_tab, p.sin_tab, p.max_pos = cos.data_ptr(), sin.data_ptr(), cos.shape[0]
        p.H, p.Hkv, p.Dh, p.rope_style = H, Hkv, Dh, 1 if interleaved else 0
        if pos is not None:
            assert pos.dtype == torch.int32 and pos.dim() == 1 and pos.shape[0] >= n
            p.pos, p.pos_stride = pos.data_ptr(), pos.stride(0)
        else:
            assert pos_period > 0
            p.pos_period = pos_period
    p.err = rt.error_word(dev).data_ptr()
    _abi.check(_abi.load().wfd_linear(ctypes.byref(p), rt.stream_ptr(dev)), "wfd_linear")


def linear(x: torch.Tensor, w: torch.Tensor, out: torch.Tensor | None = None,
           norm_eps: float | None = None) -> torch.Tensor:
    """out (n, F) = x (n, K) @ w (K, F); with norm_eps each row is first scaled by
    rsqrt(mean(x^2) + eps) (an RMSNorm whose weight is folded into w: fold_norm)."""
    if out is None:
        out = torch.empty((x.shape[0], w.shape[1]), dtype=x.dtype, device=x.device)
    _linear(x, w, _abi.WFD_LINEAR_PLAIN, out=out, norm_eps=norm_eps)
    return out


def linear_residual(x: torch.Tensor, w: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    """out (n, F) += x (n, K) @ w (K, F), in place."""
    _linear(x, w, _abi.WFD_LINEAR_RESIDUAL, out=out)
    return out


def linear_swiglu(x: torch.Tensor, w_il: torch.Tensor, norm_eps: float | None = None,
                  out: torch.Tensor | None = None) -> torch.Tensor:
    """silu(g) * u (n, dff) of g | u = x @ W for W given in the interleaved layout
    of interleave_gate_up (optionally row-normed: fold_norm before interleaving)."""
    if out is None:
        out = torch.empty((x.shape[0], w_il.shape[1] // 2), dtype=x.dtype, device=x.device)
    _linear(x, w_il, _abi.WFD_LINEAR_SWIGLU, out=out, norm_eps=norm_eps)
    return out


def linear_rope(x: torch.Tensor, w: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, n_heads: int,
                n_kv_heads: int, head_dim: int, *, pos: torch.Tensor | None = None, pos_period: int = 0,
                interleaved: bool = False, norm_eps: float | None = None):
    """q (n, H, Dh), k, v (n, Hkv, Dh) of the fused QKV projection x @ w with RoPE
    at each row's position (as rope_split on the bf16 projection)."""
    n = x.shape[0]
    assert cos.dtype == torch.float32 and sin.dtype == torch.float32 and cos.is_contiguous() and sin.is_contiguous()
    q = torch.empty((n, n_heads, head_dim), dtype=x.dtype, device=x.device)
    k = torch.empty((n, n_kv_heads, head_dim), dtype=x.dtype, device=x.device)
    v = torch.empty((n, n_kv_heads, head_dim), dtype=x.dtype, device=x.device)
    _linear(x, w, _abi.WFD_LINEAR_ROPE, norm_eps=norm_eps, q=q, k=k, v=v,
            rope=(cos, sin, n_heads, n_kv_heads, head_dim, pos, pos_period, interleaved))
    return q, k, v
