"""The reference's CPU execution of one wavefront attention step, restated in
torch for timing on the host cores (bench.py cpu_baseline / --impl reference).

Per layer the reference issues (OuroBlocksBatch.advance_union,
ouro_blocks_batch.py:207-231, HuginnBlocksBatch._union_attn,
huginn_blocks_batch.py:254-285):
  1. BatchStaticKVCache.write_tokens  (batch_kv_cache.py:61-73)   flat index_copy_
  2. BatchStaticKVCache.gather_pack   (batch_kv_cache.py:75-96)   repeat_interleave + index_select copy
  3. fa4_attention.attn_varlen        (fa4_attention.py:301-317); on CPU the "torch"
     backend falls back to the per-segment SDPA loop _attn_varlen_sdpa
     (fa4_attention.py:348-381) because aten._flash_attention_forward has no CPU kernel
The same three steps are written out below on the same tensor layouts, in the
inputs' dtype, with torch's intra-op thread pool.  This is a baseline to time,
not a checker.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F


def write_tokens(K: torch.Tensor, V: torch.Tensor, slots, seqs, positions, k: torch.Tensor, v: torch.Tensor):
    n_slots, B, S, Hkv, Dh = K.shape
    flat = [(sl * B + b) * S + p for sl, b, p in zip(slots, seqs, positions)]
    idx = torch.tensor(flat, dtype=torch.long)
    K.view(-1, Hkv, Dh).index_copy_(0, idx, k)
    V.view(-1, Hkv, Dh).index_copy_(0, idx, v)


def gather_pack(K: torch.Tensor, V: torch.Tensor, slots, seqs, uptos):
    n_slots, B, S, Hkv, Dh = K.shape
    lengths = [u + 1 for u in uptos]
    starts = [(sl * B + b) * S for sl, b in zip(slots, seqs)]
    cu = [0]
    for ln in lengths:
        cu.append(cu[-1] + ln)
    len_t = torch.tensor(lengths, dtype=torch.long)
    start_t = torch.tensor(starts, dtype=torch.long)
    cu_prev = torch.tensor(cu[:-1], dtype=torch.long)
    offs = torch.repeat_interleave(start_t - cu_prev, len_t)
    flat = offs + torch.arange(cu[-1], dtype=torch.long)
    return (K.view(-1, Hkv, Dh).index_select(0, flat), V.view(-1, Hkv, Dh).index_select(0, flat),
            torch.tensor(cu, dtype=torch.int32), max(lengths))


def attn_varlen_sdpa(q, k, v, cu_q, cu_k, causal: bool):
    cq, ck = cu_q.tolist(), cu_k.tolist()
    outs = []
    for i in range(len(cq) - 1):
        qi = q[cq[i]:cq[i + 1]].unsqueeze(0).transpose(1, 2)
        ki = k[ck[i]:ck[i + 1]].unsqueeze(0).transpose(1, 2)
        vi = v[ck[i]:ck[i + 1]].unsqueeze(0).transpose(1, 2)
        Tq, Tk = qi.shape[2], ki.shape[2]
        gqa = qi.shape[1] != ki.shape[1]
        if causal and Tq != Tk:
            ri = torch.arange(Tq).unsqueeze(1)
            cj = torch.arange(Tk).unsqueeze(0)
            o = F.scaled_dot_product_attention(qi, ki, vi, attn_mask=(cj <= ri + (Tk - Tq))[None, None],
                                               enable_gqa=gqa)
        else:
            o = F.scaled_dot_product_attention(qi, ki, vi, is_causal=causal, enable_gqa=gqa)
        outs.append(o.transpose(1, 2)[0])
    return torch.cat(outs, dim=0)


@torch.no_grad()
def wave_step(K, V, q, k_new, v_new, items):
    """One layer's wavefront attention for `items` rows (slot, seq, pos0, q_len,
    q_row0) with every q_len == 1 (decode) or a window (causal)."""
    slots, seqs, pos, rows = [], [], [], []
    for sl, b, p0, ql, r0 in items:
        for j in range(ql):
            slots.append(sl)
            seqs.append(b)
            pos.append(p0 + j)
            rows.append(r0 + j)
    ridx = torch.tensor(rows, dtype=torch.long)
    write_tokens(K, V, slots, seqs, pos, k_new.index_select(0, ridx), v_new.index_select(0, ridx))
    causal = any(it[3] > 1 for it in items)
    g_slots = [it[0] for it in items]
    g_seqs = [it[1] for it in items]
    g_upto = [it[2] + it[3] - 1 for it in items]
    kp, vp, cu_k, _ = gather_pack(K, V, g_slots, g_seqs, g_upto)
    q_lens = [it[3] for it in items]
    cu_q = torch.tensor([0] + list(torch.tensor(q_lens).cumsum(0).tolist()), dtype=torch.int32)
    qp = q.index_select(0, torch.tensor([it[4] + j for it in items for j in range(it[3])], dtype=torch.long))
    return attn_varlen_sdpa(qp, kp, vp, cu_q, cu_k, causal)
