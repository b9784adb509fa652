"""Numpy restatement of the reference's batched KV slot cache (test oracle).

Reference: src/decoding/batch_kv_cache.py
  BatchStaticKVCache.__init__              :28-44   K/V (n_slots, B, S, Hkv, Dh), seqlen[slot][b]
  write_prefill                            :51-59
  write_tokens                             :61-73   flat index (slot*B + b)*S + pos; seqlen = max(seqlen, pos+1)
  gather_pack                              :75-96   copy of positions [0, upto] per segment + cu_k
  drop_positions_at_and_after              :99-105  seqlen[s][b] = min(seqlen[s][b], pos)
plus the two compositions the wavefront op fuses:
  wave_attn      write_tokens -> gather_pack -> attn_varlen(causal=True) per
                 (slot, seq) window, as OuroBlocksBatch.advance_union
                 (ouro_blocks_batch.py:207-231) issues them for grouped segments;
  commit_window  the DtV accept cascade (scheduler_batch.py:472-499): keep the
                 accepted window rows, roll the slot back to pos0 + accepted.
"""
from __future__ import annotations

import numpy as np

from . import attention as oattn


class SlotCacheOracle:
    def __init__(self, n_slots: int, batch_size: int, n_kv_head: int, head_dim: int, max_seq_len: int,
                 dtype=np.float32):
        self.n_slots, self.B, self.S = n_slots, batch_size, max_seq_len
        self.n_kv_head, self.head_dim = n_kv_head, head_dim
        shape = (n_slots, batch_size, max_seq_len, n_kv_head, head_dim)
        self.K = np.zeros(shape, dtype=dtype)
        self.V = np.zeros(shape, dtype=dtype)
        self.seqlen = [[0] * batch_size for _ in range(n_slots)]

    def write_prefill(self, slot: int, k: np.ndarray, v: np.ndarray) -> None:
        L = k.shape[1]
        assert L <= self.S
        self.K[slot][:, :L] = k
        self.V[slot][:, :L] = v
        for b in range(self.B):
            self.seqlen[slot][b] = max(self.seqlen[slot][b], L)

    def write_tokens(self, slots, seq_ids, positions, k: np.ndarray, v: np.ndarray) -> None:
        for i, (sl, b, p) in enumerate(zip(slots, seq_ids, positions)):
            if p >= self.S:
                raise IndexError(f"position {p} exceeds max_seq_len={self.S}")
            self.K[sl, b, p] = k[i]
            self.V[sl, b, p] = v[i]
            if p + 1 > self.seqlen[sl][b]:
                self.seqlen[sl][b] = p + 1

    def gather_pack(self, slots, seq_ids, uptos):
        lengths = [u + 1 for u in uptos]
        cu = [0]
        for ln in lengths:
            cu.append(cu[-1] + ln)
        kp = np.concatenate([self.K[sl, b, : u + 1] for sl, b, u in zip(slots, seq_ids, uptos)], axis=0)
        vp = np.concatenate([self.V[sl, b, : u + 1] for sl, b, u in zip(slots, seq_ids, uptos)], axis=0)
        return kp, vp, np.asarray(cu, dtype=np.int32), max(lengths)

    def drop_positions_at_and_after(self, b: int, position: int) -> None:
        for sl in range(self.n_slots):
            if self.seqlen[sl][b] > position:
                self.seqlen[sl][b] = position

    # ------------------------------------------------------------------
    def wave_attn(self, q: np.ndarray, k_new: np.ndarray, v_new: np.ndarray, items, slot_offset: int = 0):
        """items: rows (slot, seq, pos0, q_len, q_row0).  Writes every window row,
        then attends each item's rows bottom-right causally over [0, pos0+q_len)."""
        items = [tuple(int(x) for x in it) for it in np.asarray(items).reshape(-1, 5)]
        for slot, seq, pos0, ql, r0 in items:
            rows = list(range(r0, r0 + ql))
            self.write_tokens([slot + slot_offset] * ql, [seq] * ql, [pos0 + j for j in range(ql)],
                              k_new[rows], v_new[rows])
        out = np.zeros(q.shape, dtype=np.float64)
        for slot, seq, pos0, ql, r0 in items:
            if ql == 0:
                continue
            kp, vp, cu_k, _ = self.gather_pack([slot + slot_offset], [seq], [pos0 + ql - 1])
            cu_q = np.asarray([0, ql])
            out[r0:r0 + ql] = oattn.attn_varlen(q[r0:r0 + ql], kp, vp, cu_q, cu_k, causal=True)
        return out

    def commit_window(self, items, accept_len=None, accept_mask=None, slot_offset: int = 0):
        """Accepted rows keep their K/V, compacted to pos0, pos0+1, ...; the slot
        length becomes pos0 + n_accepted.  Returns (acc_rows dict q_row0+k -> row,
        acc_count list)."""
        items = [tuple(int(x) for x in it) for it in np.asarray(items).reshape(-1, 5)]
        acc_rows, acc_count = {}, []
        for i, (slot, seq, pos0, ql, r0) in enumerate(items):
            s = slot + slot_offset
            if accept_len is not None:
                keep = [j for j in range(ql) if j < int(accept_len[i])]
            else:
                keep = [j for j in range(ql) if accept_mask[r0 + j]]
            for rk, j in enumerate(keep):
                self.K[s, seq, pos0 + rk] = self.K[s, seq, pos0 + j]
                self.V[s, seq, pos0 + rk] = self.V[s, seq, pos0 + j]
                acc_rows[r0 + rk] = r0 + j
            acc_count.append(len(keep))
            self.seqlen[s][seq] = pos0 + len(keep)
        return acc_rows, acc_count
