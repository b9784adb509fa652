"""KV slot cache for the wavefront hot path.

Same storage contract as the reference's `BatchStaticKVCache`
(src/decoding/batch_kv_cache.py:28-105):

    K, V : (n_slots, B, max_seq_len, Hkv, Dh)     buffer index == absolute position

with the logical lengths kept ON THE DEVICE (`lens`, int32 (n_slots, B)) instead
of a host list, so appends, rollbacks and commits can run inside CUDA graphs.
`seqlen` gives the reference's host view (it synchronises).  Every mutation is
a libwfd_b200 kernel: append (write_tokens), prefill write, rollback
(drop_positions_at_and_after) and the window accept/compact commit.
"""
from __future__ import annotations


import torch

from . import _abi
from . import attention as _attn
from . import ops as _ops
from . import runtime as rt


class SlotKVCache:
    def __init__(self, n_slots: int, batch_size: int, n_kv_head: int, head_dim: int, max_seq_len: int,
                 dtype: torch.dtype, device: torch.device):
        self.n_slots = n_slots
        self.B = batch_size
        self.S = max_seq_len
        self.n_kv_head = n_kv_head
        self.head_dim = head_dim
        self.dtype = dtype
        self.device = torch.device(device)
        rt.dtype_code(dtype)
        shape = (n_slots, batch_size, max_seq_len, n_kv_head, head_dim)
        self.K = torch.zeros(shape, dtype=dtype, device=self.device)
        self.V = torch.zeros(shape, dtype=dtype, device=self.device)
        self.lens = torch.zeros((n_slots, batch_size), dtype=torch.int32, device=self.device)

    @classmethod
    def wrap(cls, K: torch.Tensor, V: torch.Tensor, lens: torch.Tensor | None = None) -> "SlotKVCache":
        """Adopt existing (n_slots, B, S, Hkv, Dh) K / V tensors (e.g. a reference
        BatchStaticKVCache's .K / .V) without copying."""
        if K.dim() != 5 or V.shape != K.shape or not (K.is_contiguous() and V.is_contiguous()):
            raise ValueError("K, V must be contiguous (n_slots, B, max_seq_len, Hkv, Dh) tensors")
        rt.dtype_code(K.dtype)
        self = cls.__new__(cls)
        self.n_slots, self.B, self.S, self.n_kv_head, self.head_dim = K.shape
        self.dtype, self.device, self.K, self.V = K.dtype, K.device, K, V
        if lens is None:
            lens = torch.zeros((self.n_slots, self.B), dtype=torch.int32, device=K.device)
        if lens.dtype != torch.int32 or tuple(lens.shape) != (self.n_slots, self.B):
            raise ValueError("lens must be int32 (n_slots, B)")
        self.lens = lens
        return self

    # ------------------------------------------------------------------
    @property
    def nbytes(self) -> int:
        return (self.K.numel() + self.V.numel()) * self.K.element_size()

    @property
    def seqlen(self) -> list[list[int]]:
        """Host copy of the logical lengths, shaped like the reference's
        `seqlen[slot][b]` (batch_kv_cache.py:44).  Synchronises."""
        return self.lens.cpu().tolist()

    def _geom(self):
        return (self.n_slots, self.B, self.S, self.n_kv_head, self.head_dim, rt.dtype_code(self.dtype))

    def _stream(self) -> int:
        return rt.stream_ptr(self.device)

    # ------------------------------------------------------------------
    def write_prefill(self, slot: int, k: torch.Tensor, v: torch.Tensor) -> None:
        """k, v: (B, L, Hkv, Dh) prompt K/V at positions [0, L) (batch_kv_cache.py:51-59)."""
        L = k.shape[1]
        assert L <= self.S
        if k.shape != (self.B, L, self.n_kv_head, self.head_dim) or v.shape != k.shape:
            raise ValueError("write_prefill expects k, v of shape (B, L, Hkv, Dh)")
        k, v = k.contiguous(), v.contiguous()
        st = _abi.load().wfd_write_prefill(k.data_ptr(), v.data_ptr(), self.K.data_ptr(), self.V.data_ptr(),
                                           self.lens.data_ptr(), int(slot), L, *self._geom(), self._stream())
        _abi.check(st, "wfd_write_prefill")

    def write_tokens(self, slots, seq_ids, positions, k: torch.Tensor, v: torch.Tensor, *, slot_offset: int = 0) -> None:
        """Scatter n rows k, v (n, Hkv, Dh) to (slots[i], seq_ids[i], positions[i])
        (batch_kv_cache.py:61-73).  Host lists are bounds-checked here with the
        reference's IndexError; device index tensors are checked in the kernel."""
        n = k.shape[0]
        if isinstance(positions, list):
            for p in positions:
                if p >= self.S:
                    raise IndexError(f"position {p} exceeds max_seq_len={self.S}")
        sl = _ops.i32(slots, self.device)
        sq = _ops.i32(seq_ids, self.device)
        ps = _ops.i32(positions, self.device)
        k, v = k.contiguous(), v.contiguous()
        st = _abi.load().wfd_append(k.data_ptr(), v.data_ptr(), self.K.data_ptr(), self.V.data_ptr(),
                                    self.lens.data_ptr(), sl.data_ptr(), sq.data_ptr(), ps.data_ptr(), n,
                                    int(slot_offset), *self._geom(), rt.error_word(self.device).data_ptr(),
                                    self._stream())
        _abi.check(st, "wfd_append")

    def gather_pack(self, slots, seq_ids, uptos):
        """Pack n prefixes [(slot, b, 0..upto)] -> (k_pack, v_pack, cu_k, max_k)
        (batch_kv_cache.py:75-96).  API parity only: the wavefront op reads the
        slots in place and never packs."""
        lengths = [u + 1 for u in uptos]
        cu_host = [0]
        for ln in lengths:
            cu_host.append(cu_host[-1] + ln)
        total = cu_host[-1]
        k_pack = torch.empty((total, self.n_kv_head, self.head_dim), dtype=self.dtype, device=self.device)
        v_pack = torch.empty_like(k_pack)
        cu_k = torch.tensor(cu_host, dtype=torch.int32, device=self.device)
        sl = _ops.i32(slots, self.device)
        sq = _ops.i32(seq_ids, self.device)
        st = _abi.load().wfd_gather_pack(self.K.data_ptr(), self.V.data_ptr(), k_pack.data_ptr(), v_pack.data_ptr(),
                                         sl.data_ptr(), sq.data_ptr(), cu_k.data_ptr(), len(lengths), *self._geom(),
                                         rt.error_word(self.device).data_ptr(), self._stream())
        _abi.check(st, "wfd_gather_pack")
        return k_pack, v_pack, cu_k, max(lengths)

    # ------------------------------------------------------------------
    def drop_positions_at_and_after(self, b: int, position: int) -> None:
        """Per-sequence rollback (batch_kv_cache.py:99-105): every slot of sequence
        b keeps min(len, position) entries; buffers are untouched."""
        drop = torch.full((self.B,), -1, dtype=torch.int32)
        drop[b] = position
        self.drop_many(drop.to(self.device))

    def drop_many(self, drop_pos: torch.Tensor) -> None:
        """Batched rollback: drop_pos (B,) int32 device tensor, -1 = keep
        (torch.ops.wfd.commit_drop)."""
        torch.ops.wfd.commit_drop(self.lens, _ops.i32(drop_pos, self.device))

    def commit_window(self, items: torch.Tensor, *, accept_len: torch.Tensor | None = None,
                      accept_mask: torch.Tensor | None = None, slot_offset: int = 0, n_rows: int | None = None,
                      out: tuple[torch.Tensor, torch.Tensor] | None = None):
        """Accept commit of verify windows.  Returns (acc_rows, acc_count):
        acc_rows[q_row0 + k] = q row of the k-th accepted row of an item (rows
        past the count are left untouched: -1 when allocated here),
        acc_count[i] = accepted rows of item i.  Accepted K/V rows are compacted
        in place to pos0, pos0+1, ...  `out` supplies preallocated (acc_rows,
        acc_count) int32 tensors (nothing is allocated then, e.g. under graph
        capture)."""
        if (accept_len is None) == (accept_mask is None):
            raise ValueError("give exactly one of accept_len / accept_mask")
        items = _ops.i32(items, self.device).reshape(-1, 5)
        n = items.shape[0]
        al = None if accept_len is None else _ops.i32(accept_len, self.device)
        am = None
        if accept_mask is not None:
            am = torch.as_tensor(accept_mask).to(device=self.device, dtype=torch.uint8).contiguous()
        if out is not None:
            acc_rows, acc_count = out
            torch.ops.wfd.commit_out(self.K, self.V, self.lens, items, al, am, int(slot_offset), acc_rows, acc_count)
            return (acc_rows if n_rows is None else acc_rows[:n_rows]), acc_count[:n]
        if n_rows is None:
            n_rows = int((items[:, 4] + items[:, 3]).max().item()) if n else 0
        return torch.ops.wfd.commit(self.K, self.V, self.lens, items, al, am, int(slot_offset), int(n_rows))

    # ------------------------------------------------------------------
    def wave_attn(self, q, k_new, v_new, items, max_q: int, *, slot_offset: int = 0, out=None, kernel: int = -1,
                  update_lens: bool = True):
        """Fused append + wavefront attention over this cache's slots."""
        return _attn.wave_attn(q, k_new, v_new, self.K, self.V, items, max_q,
                               lens=self.lens if update_lens else None, slot_offset=slot_offset, out=out,
                               kernel=kernel)
