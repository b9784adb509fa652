"""PyTorch custom ops over libwfd_b200: the dispatcher-level drop-in for the
reference's attention backend and KV-slot commits.

Registered in the `wfd` namespace with torch.library (schemas below), each with
a CUDA kernel (a libwfd_b200 launch on the current stream) and a fake (meta)
kernel, so the ops trace under FakeTensor / torch.compile and capture into CUDA
graphs.  Mutated arguments are declared in the schemas (`Tensor(a!)`): the KV
cache and the slot lengths.  There is no CPU kernel: a CPU tensor fails in the
dispatcher.

  wfd::attn(q, k, v, cu_q, cu_k, max_q, max_k, causal=False, scale=None) -> out
      packed varlen attention, bottom-right causal per segment.  Replaces the
      graph engine's torch.ops.aten._flash_attention_forward(q, K, V, cu_q,
      cu_k, max_q, max_k, 0.0, causal, False)[0] (graph_blocks.py:37-43) and
      fa4_attention.attn_varlen (fa4_attention.py:301-317).
  wfd::attn_out(..., Tensor(a!) out) -> ()            the same into `out`
  wfd::wave_attn(q, k_new, v_new, k_cache!, v_cache!, items, max_q,
                 lens!?=None, slot_offset=0, scale=None, kernel=-1, row_pos=None) -> out
      write_tokens + gather_pack + attn_varlen of one wavefront tick in one
      launch pair (batch_kv_cache.py:61-96, ouro_blocks_batch.py:207-231);
      row_pos (int32, one per q row, any stride) gives gapped windows their
      rows' positions (ouro_blocks_batch.py:184-205 pads such runs instead).
  wfd::wave_attn_out(..., Tensor(d!) out) -> ()
  wfd::commit(k_cache!, v_cache!, lens!, items, accept_len?, accept_mask?,
              slot_offset, n_rows) -> (acc_rows, acc_count)
      verify-window accept commit with in-place compaction
      (scheduler_batch.py:472-499 semantics, drop_positions_at_and_after
      rollback, batch_kv_cache.py:99-105).
  wfd::commit_out(..., Tensor(d!) acc_rows, Tensor(e!) acc_count) -> ()
  wfd::commit_drop(lens!, drop_pos) -> ()
      batched drop_positions_at_and_after (drop_pos[b] = -1 keeps sequence b).
"""
from __future__ import annotations

import torch

from . import _abi
from . import runtime as rt

_LIB = torch.library.Library("wfd", "DEF")

_SCHEMAS = {
    "attn": "attn(Tensor q, Tensor k, Tensor v, Tensor cu_q, Tensor cu_k, int max_q, int max_k, bool causal=False, "
            "float? scale=None) -> Tensor",
    "attn_out": "attn_out(Tensor q, Tensor k, Tensor v, Tensor cu_q, Tensor cu_k, int max_q, int max_k, bool causal, "
                "float? scale, Tensor(a!) out) -> ()",
    "wave_attn": "wave_attn(Tensor q, Tensor k_new, Tensor v_new, Tensor(a!) k_cache, Tensor(b!) v_cache, "
                 "Tensor items, int max_q, Tensor(c!)? lens=None, int slot_offset=0, float? scale=None, "
                 "int kernel=-1, Tensor? row_pos=None) -> Tensor",
    "wave_attn_out": "wave_attn_out(Tensor q, Tensor k_new, Tensor v_new, Tensor(a!) k_cache, Tensor(b!) v_cache, "
                     "Tensor items, int max_q, Tensor(c!)? lens, int slot_offset, float? scale, int kernel, "
                     "Tensor? row_pos, Tensor(d!) out) -> ()",
    "commit": "commit(Tensor(a!) k_cache, Tensor(b!) v_cache, Tensor(c!) lens, Tensor items, Tensor? accept_len, "
              "Tensor? accept_mask, int slot_offset, int n_rows) -> (Tensor, Tensor)",
    "commit_out": "commit_out(Tensor(a!) k_cache, Tensor(b!) v_cache, Tensor(c!) lens, Tensor items, "
                  "Tensor? accept_len, Tensor? accept_mask, int slot_offset, Tensor(d!) acc_rows, "
                  "Tensor(e!) acc_count) -> ()",
    "commit_drop": "commit_drop(Tensor(a!) lens, Tensor drop_pos) -> ()",
}
for _schema in _SCHEMAS.values():
    _LIB.define(_schema)


# ---------------------------------------------------------------------------
# argument checks shared by the kernels
# ---------------------------------------------------------------------------
def heads(q: torch.Tensor, k: torch.Tensor) -> tuple[int, int, int]:
    H, Dh = q.shape[-2], q.shape[-1]
    Hkv = k.shape[-2]
    if k.shape[-1] != Dh:
        raise ValueError(f"head_dim mismatch: q {Dh} vs k {k.shape[-1]}")
    if H % Hkv != 0:
        raise ValueError(f"query heads {H} not a multiple of kv heads {Hkv}")
    return H, Hkv, Dh


def i32(t, device) -> torch.Tensor:
    t = torch.as_tensor(t)
    if t.dtype != torch.int32 or t.device != device:
        t = t.to(device=device, dtype=torch.int32)
    return t.contiguous()


def _check_varlen(q, k, v, cu_q, cu_k):
    dev = rt.require_cuda(q, k, v, cu_q, cu_k)
    if q.dim() != 3 or k.dim() != 3 or v.shape != k.shape:
        raise ValueError("attn expects q (total_q, H, Dh), k/v (total_k, Hkv, Dh)")
    heads(q, k)
    if q.dtype != k.dtype or k.dtype != v.dtype:
        raise TypeError("q, k, v must share a dtype")
    if cu_q.dtype != torch.int32 or cu_k.dtype != torch.int32 or cu_q.numel() != cu_k.numel():
        raise ValueError("cu_q / cu_k must be int32 with the same number of segments + 1")
    return dev


def _check_wave(q, k_new, v_new, k_cache, v_cache, items, lens):
    dev = rt.require_cuda(q, k_new, v_new, k_cache, v_cache, items, lens)
    if k_cache.dim() != 5 or v_cache.shape != k_cache.shape:
        raise ValueError("k_cache / v_cache must be (n_slots, n_seqs, max_seq, Hkv, Dh)")
    n_slots, n_seqs, _, Hkv, Dh = k_cache.shape
    if q.dim() != 3 or q.shape[2] != Dh or k_new.shape != (q.shape[0], Hkv, Dh) or v_new.shape != k_new.shape:
        raise ValueError("q (n_rows, H, Dh) and k_new / v_new (n_rows, Hkv, Dh) must match the cache")
    if not (k_cache.is_contiguous() and v_cache.is_contiguous()):
        raise ValueError("k_cache / v_cache must be contiguous")
    if items.dtype != torch.int32 or items.dim() != 2 or items.shape[1] != 5 or not items.is_contiguous():
        raise ValueError("items must be a contiguous int32 (n_items, 5) device tensor")
    if lens is not None and (lens.dtype != torch.int32 or tuple(lens.shape) != (n_slots, n_seqs)):
        raise ValueError("lens must be int32 (n_slots, n_seqs)")
    return dev


def _check_commit(k_cache, v_cache, lens, items, accept_len, accept_mask):
    dev = rt.require_cuda(k_cache, v_cache, lens, items, accept_len, accept_mask)
    if (accept_len is None) == (accept_mask is None):
        raise ValueError("give exactly one of accept_len / accept_mask")
    if k_cache.dim() != 5 or v_cache.shape != k_cache.shape:
        raise ValueError("k_cache / v_cache must be (n_slots, n_seqs, max_seq, Hkv, Dh)")
    if lens.dtype != torch.int32 or tuple(lens.shape) != tuple(k_cache.shape[:2]):
        raise ValueError("lens must be int32 (n_slots, n_seqs)")
    if items.dtype != torch.int32 or items.dim() != 2 or items.shape[1] != 5 or not items.is_contiguous():
        raise ValueError("items must be a contiguous int32 (n_items, 5) device tensor")
    if accept_len is not None and accept_len.dtype != torch.int32:
        raise ValueError("accept_len must be int32")
    if accept_mask is not None and accept_mask.dtype != torch.uint8:
        raise ValueError("accept_mask must be uint8")
    return dev


# ---------------------------------------------------------------------------
# CUDA kernels (libwfd_b200 launches on the current stream)
# ---------------------------------------------------------------------------
def _attn_out_cuda(q, k, v, cu_q, cu_k, max_q, max_k, causal, scale, out):
    dev = _check_varlen(q, k, v, cu_q, cu_k)
    H, Hkv, Dh = heads(q, k)
    if out.shape != q.shape or out.dtype != q.dtype or not out.is_contiguous():
        raise ValueError("out must be a contiguous tensor shaped like q")
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    cu_q, cu_k = cu_q.contiguous(), cu_k.contiguous()
    n = cu_q.numel() - 1
    ws, wsb = rt.workspace(dev, n, Dh)
    st = _abi.load().wfd_attn_varlen(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), cu_q.data_ptr(),
                                     cu_k.data_ptr(), n, int(max_q), q.shape[0], k.shape[0], H, Hkv, Dh,
                                     rt.dtype_code(q.dtype), 1 if causal else 0, float(scale or 0.0), ws.data_ptr(),
                                     wsb, rt.error_word(dev).data_ptr(), rt.stream_ptr(dev))
    _abi.check(st, "wfd_attn_varlen")


def _attn_cuda(q, k, v, cu_q, cu_k, max_q, max_k, causal=False, scale=None):
    out = torch.empty(q.shape, dtype=q.dtype, device=q.device)
    _attn_out_cuda(q, k, v, cu_q, cu_k, max_q, max_k, causal, scale, out)
    return out


def _wave_attn_out_cuda(q, k_new, v_new, k_cache, v_cache, items, max_q, lens, slot_offset, scale, kernel, row_pos,
                        out):
    dev = _check_wave(q, k_new, v_new, k_cache, v_cache, items, lens)
    n_slots, n_seqs, max_seq, Hkv, Dh = k_cache.shape
    if out.shape != q.shape or out.dtype != q.dtype or not out.is_contiguous():
        raise ValueError("out must be a contiguous tensor shaped like q")
    rp_stride = 1
    if row_pos is not None:
        if row_pos.dtype != torch.int32 or row_pos.dim() != 1 or row_pos.numel() < q.shape[0] or \
                row_pos.device != dev or row_pos.stride(0) < 1:
            raise ValueError("row_pos must be an int32 device vector with one position per q row")
        rp_stride = row_pos.stride(0)
    q, k_new, v_new = q.contiguous(), k_new.contiguous(), v_new.contiguous()
    n = items.shape[0]
    ws, wsb = rt.workspace(dev, n, Dh)
    st = _abi.load().wfd_wave_attn_rows(
        int(kernel), q.data_ptr(), k_new.data_ptr(), v_new.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
        out.data_ptr(), rt.ptr(lens), items.data_ptr(), n, int(max_q), rt.ptr(row_pos), rp_stride, int(slot_offset),
        q.shape[0], n_slots, n_seqs, max_seq, q.shape[1], Hkv, Dh, rt.dtype_code(q.dtype), float(scale or 0.0),
        ws.data_ptr(), wsb, rt.error_word(dev).data_ptr(), rt.stream_ptr(dev))
    _abi.check(st, "wfd_wave_attn")


def _wave_attn_cuda(q, k_new, v_new, k_cache, v_cache, items, max_q, lens=None, slot_offset=0, scale=None,
                    kernel=-1, row_pos=None):
    out = torch.empty(q.shape, dtype=q.dtype, device=q.device)
    _wave_attn_out_cuda(q, k_new, v_new, k_cache, v_cache, items, max_q, lens, slot_offset, scale, kernel, row_pos,
                        out)
    return out


def _commit_out_cuda(k_cache, v_cache, lens, items, accept_len, accept_mask, slot_offset, acc_rows, acc_count):
    dev = _check_commit(k_cache, v_cache, lens, items, accept_len, accept_mask)
    if acc_rows.dtype != torch.int32 or acc_count.dtype != torch.int32:
        raise ValueError("acc_rows / acc_count must be int32")
    if acc_count.numel() < items.shape[0]:
        raise ValueError("acc_count needs one entry per item")
    if accept_len is not None and accept_len.numel() < items.shape[0]:
        raise ValueError("accept_len needs one entry per item")
    n_slots, n_seqs, max_seq, Hkv, Dh = k_cache.shape
    al = None if accept_len is None else accept_len.contiguous()
    am = None if accept_mask is None else accept_mask.contiguous()
    # q rows both row-indexed arrays cover: the kernel skips (and reports) windows past them
    n_rows = acc_rows.numel() if am is None else min(acc_rows.numel(), am.numel())
    st = _abi.load().wfd_commit_window(k_cache.data_ptr(), v_cache.data_ptr(), lens.data_ptr(), items.data_ptr(),
                                       items.shape[0], rt.ptr(al), rt.ptr(am), acc_rows.data_ptr(),
                                       acc_count.data_ptr(), n_rows, int(slot_offset), n_slots, n_seqs, max_seq, Hkv,
                                       Dh, rt.dtype_code(k_cache.dtype), rt.error_word(dev).data_ptr(),
                                       rt.stream_ptr(dev))
    _abi.check(st, "wfd_commit_window")


def _commit_cuda(k_cache, v_cache, lens, items, accept_len, accept_mask, slot_offset, n_rows):
    acc_rows = torch.full((int(n_rows),), -1, dtype=torch.int32, device=k_cache.device)
    acc_count = torch.zeros((items.shape[0],), dtype=torch.int32, device=k_cache.device)
    _commit_out_cuda(k_cache, v_cache, lens, items, accept_len, accept_mask, slot_offset, acc_rows, acc_count)
    return acc_rows, acc_count


def _commit_drop_cuda(lens, drop_pos):
    dev = rt.require_cuda(lens, drop_pos)
    if lens.dtype != torch.int32 or lens.dim() != 2 or drop_pos.dtype != torch.int32 or \
            drop_pos.numel() != lens.shape[1]:
        raise ValueError("lens int32 (n_slots, n_seqs), drop_pos int32 (n_seqs,)")
    st = _abi.load().wfd_commit_drop(lens.data_ptr(), drop_pos.contiguous().data_ptr(), lens.shape[0], lens.shape[1],
                                     rt.stream_ptr(dev))
    _abi.check(st, "wfd_commit_drop")


_LIB.impl("attn", _attn_cuda, "CUDA")
_LIB.impl("attn_out", _attn_out_cuda, "CUDA")
_LIB.impl("wave_attn", _wave_attn_cuda, "CUDA")
_LIB.impl("wave_attn_out", _wave_attn_out_cuda, "CUDA")
_LIB.impl("commit", _commit_cuda, "CUDA")
_LIB.impl("commit_out", _commit_out_cuda, "CUDA")
_LIB.impl("commit_drop", _commit_drop_cuda, "CUDA")


# ---------------------------------------------------------------------------
# fake (meta) kernels: shapes and dtypes only
# ---------------------------------------------------------------------------
@torch.library.register_fake("wfd::attn")
def _attn_fake(q, k, v, cu_q, cu_k, max_q, max_k, causal=False, scale=None):
    return torch.empty_like(q)


@torch.library.register_fake("wfd::attn_out")
def _attn_out_fake(q, k, v, cu_q, cu_k, max_q, max_k, causal, scale, out):
    return None


@torch.library.register_fake("wfd::wave_attn")
def _wave_attn_fake(q, k_new, v_new, k_cache, v_cache, items, max_q, lens=None, slot_offset=0, scale=None, kernel=-1,
                    row_pos=None):
    return torch.empty_like(q)


@torch.library.register_fake("wfd::wave_attn_out")
def _wave_attn_out_fake(q, k_new, v_new, k_cache, v_cache, items, max_q, lens, slot_offset, scale, kernel, row_pos,
                        out):
    return None


@torch.library.register_fake("wfd::commit")
def _commit_fake(k_cache, v_cache, lens, items, accept_len, accept_mask, slot_offset, n_rows):
    return (k_cache.new_empty((n_rows,), dtype=torch.int32), k_cache.new_empty((items.shape[0],), dtype=torch.int32))


@torch.library.register_fake("wfd::commit_out")
def _commit_out_fake(k_cache, v_cache, lens, items, accept_len, accept_mask, slot_offset, acc_rows, acc_count):
    return None


@torch.library.register_fake("wfd::commit_drop")
def _commit_drop_fake(lens, drop_pos):
    return None
