"""Attention backend with the reference's call surface, on libwfd_b200 kernels.

Mirrors `src/decoding/fa4_attention.py` of the reference (same function names,
argument meaning, shapes and contract checks) so a reference call site can be
pointed at this module unchanged, plus `wave_attn`, the slot-native wavefront
op that replaces the write_tokens -> gather_pack -> attn_varlen sequence.

Layouts (reference fa4_attention.py:187-300):
  attn_dense        q (B, Tq, H, Dh), k/v (B, Tk, Hkv, Dh)        -> (B, Tq, H, Dh)
  attn_cutoff_multi q (1, nq, H, Dh), k/v (1, Tk, Hkv, Dh), qpos  -> (1, nq, H, Dh)
  attn_varlen       q (total_q, H, Dh), k/v (total_k, Hkv, Dh), cu_q/cu_k (n+1,) int32
Semantics: scale 1/sqrt(Dh); GQA head h reads kv head h // (H/Hkv); causal means
bottom-right aligned (row r of a (q_len, k_len) segment sees keys <= k_len-q_len+r).
There is one implementation (CUDA, sm_100a); nothing here computes on the CPU.
`attn_varlen` and `wave_attn` go through the dispatcher ops `torch.ops.wfd.*`
(ops.py), which a call site can also use directly.
"""
from __future__ import annotations

import torch

from . import _abi
from . import ops as _ops
from . import runtime as rt

# The reference selects among "torch" | "fa4" | "sdpa" (fa4_attention.py:107-118).
# Those names are accepted so that its call sites run unchanged; every name runs
# the same libwfd_b200 kernels.
_BACKEND_NAMES = ("wfd", "torch", "fa4", "sdpa")
_BACKEND = "wfd"


def set_backend(name: str) -> None:
    """Reference `set_backend` (fa4_attention.py:107-114): asserts a known name."""
    global _BACKEND
    assert name in _BACKEND_NAMES
    _BACKEND = name


def backend() -> str:
    return _BACKEND


_heads = _ops.heads
_i32 = _ops.i32


def attn_varlen(q, k, v, cu_q, cu_k, max_q, max_k, causal: bool = False, *, scale: float | None = None,
                out: torch.Tensor | None = None):
    """Reference `attn_varlen` (fa4_attention.py:301-317), through the
    dispatcher op torch.ops.wfd.attn (torch.ops.wfd.attn_out with `out`).
    causal=False: every row of a segment sees the whole segment; causal=True:
    bottom-right causal per segment.  cu_q / cu_k may be device tensors whose
    contents change between CUDA-graph replays (the graph engine's
    lengths-as-data contract, graph_blocks.py:5-11); max_q / max_k are upper
    bounds."""
    dev = rt.require_cuda(q, k, v)
    if q.dim() != 3 or k.dim() != 3 or v.shape != k.shape:
        raise ValueError("attn_varlen expects q (total_q, H, Dh), k/v (total_k, Hkv, Dh)")
    _heads(q, k)
    if q.dtype != k.dtype or k.dtype != v.dtype:
        raise TypeError("q, k, v must share a dtype")
    cu_q, cu_k = _i32(cu_q, dev), _i32(cu_k, dev)
    if cu_k.numel() != cu_q.numel():
        raise ValueError("cu_q and cu_k must have the same number of segments")
    if out is None:
        return torch.ops.wfd.attn(q, k, v, cu_q, cu_k, int(max_q), int(max_k), bool(causal), scale)
    torch.ops.wfd.attn_out(q, k, v, cu_q, cu_k, int(max_q), int(max_k), bool(causal), scale, out)
    return out


def attn_varlen_q1_padded(q, k, v, cu_k, max_k):
    """Reference `attn_varlen_q1_padded` (fa4_attention.py:320-342): n
    single-query segments, each row attending its whole segment.  The reference
    duplicates rows to dodge FA2 tile downgrades; the wavefront kernel reads
    single-query segments at full bandwidth, so no padding is needed."""
    n = q.shape[0]
    cu_q = torch.arange(0, n + 1, dtype=torch.int32, device=q.device)
    return attn_varlen(q, k, v, cu_q, cu_k, 1, max_k, causal=False)


def attn_segments(q, k, v, q_row0, q_len, k_row0, k_len, max_q, causal: bool, *, scale: float | None = None,
                  out: torch.Tensor | None = None):
    """Explicit-segment attention (segments may share key rows)."""
    dev = rt.require_cuda(q, k, v)
    H, Hkv, Dh = _heads(q, k)
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    q_row0, q_len, k_row0, k_len = (_i32(t, dev) for t in (q_row0, q_len, k_row0, k_len))
    n = q_row0.numel()
    if out is None:
        out = torch.empty_like(q)
    ws, wsb = rt.workspace(dev, n, Dh)
    st = _abi.load().wfd_attn_segments(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
                                       q_row0.data_ptr(), q_len.data_ptr(), k_row0.data_ptr(), k_len.data_ptr(), n,
                                       int(max_q), q.shape[0], k.shape[0], H, Hkv, Dh, rt.dtype_code(q.dtype),
                                       1 if causal else 0, float(scale or 0.0), ws.data_ptr(), wsb,
                                       rt.error_word(dev).data_ptr(), rt.stream_ptr(dev))
    _abi.check(st, "wfd_attn_segments")
    return out


# Query rows per segment from which dense attention runs on the prompt kernel
# (query-major tcgen05 tiles of 128 rows) instead of the decode / verify kernels.
PREFILL_MIN_ROWS = 64


def attn_prefill(q, k, v, *, causal: bool, scale: float | None = None, out: torch.Tensor | None = None):
    """Dense prompt attention on the tcgen05 prompt kernel (wfd_attn_prefill):
    q (B, Tq, H, Dh), k / v (B, Tk, Hkv, Dh), bf16, Dh 64 or 128; causal is
    bottom-right aligned.  The prompt pass of every layer (write_prefill +
    attn_dense, ouro_blocks_batch.py:123-144)."""
    dev = rt.require_cuda(q, k, v)
    B, Tq, H, Dh = q.shape
    Tk, Hkv = k.shape[1], k.shape[2]
    _heads(q, k)
    if v.shape != k.shape or k.shape[0] != B:
        raise ValueError("attn_prefill expects q (B, Tq, H, Dh), k / v (B, Tk, Hkv, Dh)")
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    if out is None:
        out = torch.empty_like(q)
    st = _abi.load().wfd_attn_prefill(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), B, Tq, Tk, H, Hkv, Dh,
                                      rt.dtype_code(q.dtype), 1 if causal else 0, float(scale or 0.0),
                                      rt.error_word(dev).data_ptr(), rt.stream_ptr(dev))
    _abi.check(st, "wfd_attn_prefill")
    return out


def attn_dense(q, k, v, *, causal: bool):
    """Reference `attn_dense` (fa4_attention.py:191-232): per batch element,
    Tq=1 or causal=False sees the whole prefix; causal is bottom-right aligned
    (Tq == Tk is the ordinary causal mask).  bf16 prompts (Tq >= 64, head_dim
    64 / 128) run on the prompt kernel, everything else on the varlen path."""
    rt.require_cuda(q, k, v)
    B, Tq, H, Dh = q.shape
    Tk = k.shape[1]
    if q.dtype == torch.bfloat16 and Dh in (64, 128) and Tq >= PREFILL_MIN_ROWS:
        return attn_prefill(q, k, v, causal=bool(causal) and Tq > 1)
    qf = q.reshape(B * Tq, H, Dh)
    kf = k.reshape(B * Tk, k.shape[2], Dh)
    vf = v.reshape(B * Tk, v.shape[2], Dh)
    cu_q = torch.arange(0, B * Tq + 1, Tq, dtype=torch.int32, device=q.device)
    cu_k = torch.arange(0, B * Tk + 1, Tk, dtype=torch.int32, device=q.device)
    out = attn_varlen(qf, kf, vf, cu_q, cu_k, Tq, Tk, causal=bool(causal) and Tq > 1)
    return out.view(B, Tq, H, Dh)


def attn_cutoff_multi(q, k, v, qpos):
    """Reference `attn_cutoff_multi` (fa4_attention.py:240-291): nq queries at
    disjoint absolute positions sharing one slot; query m sees keys
    j <= qpos[m].  Contract (asserted as in the reference, :262): Tk == max(qpos)+1."""
    rt.require_cuda(q, k, v)
    pos = qpos if isinstance(qpos, list) else torch.as_tensor(qpos).tolist()
    B, nq, H, Dh = q.shape
    Tk = k.shape[1]
    assert Tk == max(pos) + 1, "attn_cutoff_multi expects K sliced to max(qpos)+1"
    assert B == 1
    dev = q.device
    q_row0 = torch.arange(nq, dtype=torch.int32)
    q_len = torch.ones(nq, dtype=torch.int32)
    k_row0 = torch.zeros(nq, dtype=torch.int32)
    k_len = torch.tensor([p + 1 for p in pos], dtype=torch.int32)
    out = attn_segments(q.reshape(nq, H, Dh), k.reshape(Tk, k.shape[2], Dh), v.reshape(Tk, v.shape[2], Dh),
                        q_row0.to(dev), q_len.to(dev), k_row0.to(dev), k_len.to(dev), 1, causal=False)
    return out.view(1, nq, H, Dh)


def wave_attn(q, k_new, v_new, k_cache, v_cache, items, max_q: int, *, lens=None, slot_offset: int = 0,
              out: torch.Tensor | None = None, scale: float | None = None, kernel: int = -1,
              row_pos: torch.Tensor | None = None):
    """Wavefront decode / verify attention with the K/V append fused, through
    the dispatcher op torch.ops.wfd.wave_attn (torch.ops.wfd.wave_attn_out with
    `out`).

    q (n_rows, H, Dh); k_new / v_new (n_rows, Hkv, Dh); k_cache / v_cache
    (n_slots, n_seqs, max_seq, Hkv, Dh); items: device int32 (n_items, 5) rows of
    (slot, seq, pos0, q_len, q_row0); lens: optional device int32 (n_slots,
    n_seqs).  Row j of an item writes its K/V at pos0+j of (slot+slot_offset, seq)
    and attends positions [0, pos0+j].  kernel: -1 auto, 0 CUDA-core decode,
    1 tcgen05 verify.  row_pos (int32, one position per q row, any stride):
    gapped windows, row j of an item at row_pos[q_row0 + j] instead of pos0 + j
    (tcgen05 kernel only)."""
    rt.require_cuda(q, k_new, v_new, k_cache, v_cache, items)
    if out is None:
        return torch.ops.wfd.wave_attn(q, k_new, v_new, k_cache, v_cache, items, int(max_q), lens, int(slot_offset),
                                       scale, int(kernel), row_pos)
    torch.ops.wfd.wave_attn_out(q, k_new, v_new, k_cache, v_cache, items, int(max_q), lens, int(slot_offset), scale,
                                int(kernel), row_pos, out)
    return out
