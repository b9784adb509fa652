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


# ---------------------------------------------------------------------------
# the whole decode loop: the reference's batched looped-LM blocks on the host
# ---------------------------------------------------------------------------
def random_weights(dims: dict, seed: int, dtype=torch.bfloat16, std: float = 0.02) -> dict:
    """Random-init weights of the looped LM (the layout oracle.looped_lm reads:
    embed, prelude / core / coda blocks of norm1, wqkv, wo, norm2, wgu, wd,
    final_norm, lm_head).  Only shapes matter for timing."""
    g = torch.Generator().manual_seed(seed)
    d, H, Hkv, Dh, F_ = dims["d_model"], dims["n_heads"], dims["n_kv_heads"], dims["head_dim"], dims["d_ff"]

    def w(*shape, scale=1.0):
        return (torch.randn(shape, generator=g) * (std * scale)).to(dtype)

    def blk():
        return {"norm1": torch.ones(d, dtype=dtype), "wqkv": w(d, (H + 2 * Hkv) * Dh),
                "wo": w(H * Dh, d, scale=0.7071), "norm2": torch.ones(d, dtype=dtype),
                "wgu": w(d, 2 * F_), "wd": w(F_, d, scale=0.7071)}

    return {"embed": w(dims["vocab"], d, scale=50.0), "final_norm": torch.ones(d, dtype=dtype),
            "lm_head": w(d, dims["vocab"]), "prelude": [blk() for _ in range(dims["n_prelude"])],
            "core": [blk() for _ in range(dims["n_core"])], "coda": [blk() for _ in range(dims["n_coda"])]}


class LoopedBlocksCPU:
    """The reference's batched looped-LM blocks, run on the host cores.

    The four calls its batch scheduler makes (scheduler_batch.py:123-159 prefill,
    then prelude_union / advance_union / coda_argmax_union per tick) with the
    Parcae split into prelude, looped core and coda (parcae_blocks.py:284-309
    prelude, :310-390 one core step over the union, :476-518 coda) and the
    batched union body of ouro_blocks_batch.py:173-243: per layer RMSNorm, fused
    QKV projection, RoPE at each row's position, then
      write_tokens   (batch_kv_cache.py:61-73)  every row's K / V into its slot,
      gather_pack    (batch_kv_cache.py:75-96)  each row's slot prefix [0, pos] copied out,
      attn_varlen    (fa4_attention.py:369-381) the per-segment SDPA loop (q_len 1),
    o_proj + residual, RMSNorm, SwiGLU + residual.  The prompt pass is
    write_prefill + causal attn_dense per layer (ouro_blocks_batch.py:123-144).
    The cache is BatchStaticKVCache's (n_slots, B, S, Hkv, Dh) tensors; slots as
    in the package (prelude i -> i, core (depth r, layer l) -> n_prelude +
    (r % s) * n_core + l, coda i -> n_prelude + s * n_core + i).

    `synthetic_prompt=True` skips the prompt pass: the slots' prompt rows hold
    random K / V and the first token of each sequence is its last prompt id.
    The decode work per tick is unchanged (it never reads values back into
    control flow other than the greedy ids); bench.py times the decode region
    only."""

    def __init__(self, W: dict, cfg: dict, batch: int, max_seq: int, dtype=torch.bfloat16,
                 synthetic_prompt: bool = False, seed: int = 0):
        self.W, self.cfg, self.B, self.S, self.dtype = W, cfg, batch, max_seq, dtype
        self.H, self.Hkv, self.Dh = cfg["n_heads"], cfg["n_kv_heads"], cfg["head_dim"]
        self.T_total = cfg["T_total"]
        self.n_prelude, self.n_core, self.n_coda = len(W["prelude"]), len(W["core"]), len(W["coda"])
        s = int(cfg.get("kv_budget_s", 0) or 0)
        self.n_depth = s if 0 < s < self.T_total else self.T_total
        self.n_slots = self.n_prelude + self.n_depth * self.n_core + self.n_coda
        self.K = torch.zeros((self.n_slots, batch, max_seq, self.Hkv, self.Dh), dtype=dtype)
        self.V = torch.zeros_like(self.K)
        self.seqlen = [[0] * batch for _ in range(self.n_slots)]
        self.synthetic_prompt = synthetic_prompt
        self.seed = seed
        tab = torch.float64 if dtype == torch.float64 else torch.float32
        inv = 1.0 / (cfg["rope_theta"] ** (torch.arange(0, self.Dh, 2, dtype=torch.float64) / self.Dh))
        ang = torch.outer(torch.arange(max_seq, dtype=torch.float64), inv)
        self.cos, self.sin = ang.cos().to(tab), ang.sin().to(tab)

    # slots -------------------------------------------------------------
    def slot_prelude(self, i: int) -> int:
        return i

    def slot_core(self, r: int, l: int) -> int:
        return self.n_prelude + (r % self.n_depth) * self.n_core + l

    def slot_coda(self, i: int) -> int:
        return self.n_prelude + self.n_depth * self.n_core + i

    # math --------------------------------------------------------------
    def _rms(self, x, w):
        xf = x.to(self.cos.dtype)
        y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.cfg["norm_eps"])
        return y.to(x.dtype) * w

    def _rope(self, x, pos):
        """x (n, h, Dh) at positions pos (n,) (long)."""
        c, s = self.cos[pos][:, None, :], self.sin[pos][:, None, :]
        xf = x.to(c.dtype)
        if self.cfg.get("rope_style", "half") == "interleaved":
            a, b = xf[..., 0::2], xf[..., 1::2]
            y = torch.stack((a * c - b * s, a * s + b * c), dim=-1).flatten(-2)
        else:
            h = self.Dh // 2
            x1, x2 = xf[..., :h], xf[..., h:]
            y = torch.cat((x1 * c - x2 * s, x2 * c + x1 * s), dim=-1)
        return y.to(x.dtype)

    def _qkv(self, blk, x, pos):
        H, Hkv, Dh = self.H, self.Hkv, self.Dh
        n = x.shape[0]
        h = self._rms(x, blk["norm1"]) @ blk["wqkv"]
        q, k, v = torch.split(h, [H * Dh, Hkv * Dh, Hkv * Dh], dim=-1)
        return (self._rope(q.reshape(n, H, Dh), pos), self._rope(k.reshape(n, Hkv, Dh), pos),
                v.reshape(n, Hkv, Dh))

    def _finish(self, blk, x, o):
        x = x + o.reshape(x.shape[0], -1) @ blk["wo"]
        gu = self._rms(x, blk["norm2"]) @ blk["wgu"]
        g, u = gu.split(self.cfg["d_ff"], dim=-1)
        return x + (F.silu(g) * u) @ blk["wd"]

    def _union_block(self, blk, x, slots, seqs, positions, pos):
        q, k, v = self._qkv(blk, x, pos)
        write_tokens(self.K, self.V, slots, seqs, positions, k, v)
        for sl, b, p in zip(slots, seqs, positions):
            if self.seqlen[sl][b] <= p:
                self.seqlen[sl][b] = p + 1
        kp, vp, cu_k, _ = gather_pack(self.K, self.V, slots, seqs, positions)
        cu_q = torch.arange(len(positions) + 1, dtype=torch.int32)
        return self._finish(blk, x, attn_varlen_sdpa(q, kp, vp, cu_q, cu_k, causal=False))

    def _dense_block(self, blk, x, slot):
        """Prompt pass of one layer over (B, L, d): write_prefill, causal attn_dense."""
        B, L, d = x.shape
        pos = torch.arange(L).repeat(B)
        q, k, v = self._qkv(blk, x.reshape(B * L, d), pos)
        q, k, v = (t.reshape(B, L, t.shape[1], self.Dh) for t in (q, k, v))
        self.K[slot, :B, :L] = k
        self.V[slot, :B, :L] = v
        o = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
                                           is_causal=True, enable_gqa=self.H != self.Hkv).transpose(1, 2)
        return self._finish(blk, x.reshape(B * L, d), o.reshape(B * L, -1)).reshape(B, L, d)

    # the scheduler's interface ------------------------------------------
    @torch.no_grad()
    def prefill(self, prompt_ids: torch.Tensor):
        B, L = prompt_ids.shape
        assert B == self.B, f"prefill expects (B={self.B}, L) prompt ids"
        for row in self.seqlen:
            row[:] = [L] * B
        if self.synthetic_prompt:
            g = torch.Generator().manual_seed(self.seed)
            blockk = torch.randn((1, 1, L, self.Hkv, self.Dh), generator=g).to(self.dtype)
            blockv = torch.randn((1, 1, L, self.Hkv, self.Dh), generator=g).to(self.dtype)
            self.K[:, :, :L].copy_(blockk.expand(self.n_slots, B, L, self.Hkv, self.Dh))
            self.V[:, :, :L].copy_(blockv.expand(self.n_slots, B, L, self.Hkv, self.Dh))
            logits = torch.zeros((B, self.W["lm_head"].shape[1]))
            logits[torch.arange(B), prompt_ids[:, -1].long()] = 1.0
            return self, logits
        W = self.W
        x = W["embed"][prompt_ids.long()]
        for i, blk in enumerate(W["prelude"]):
            x = self._dense_block(blk, x, self.slot_prelude(i))
        e, h = x, torch.zeros_like(x)
        for r in range(self.T_total):
            h = h + e
            for l, blk in enumerate(W["core"]):
                h = self._dense_block(blk, h, self.slot_core(r, l))
        for i, blk in enumerate(W["coda"]):
            h = self._dense_block(blk, h, self.slot_coda(i))
        return self, (self._rms(h[:, -1], W["final_norm"]) @ W["lm_head"]).float()

    def drop_positions_at_and_after(self, b: int, position: int) -> None:
        """BatchStaticKVCache.drop_positions_at_and_after (batch_kv_cache.py:98-105):
        only the lengths move; rows at and after `position` are rewritten before
        any row at those positions attends."""
        for row in self.seqlen:
            if row[b] > position:
                row[b] = position

    @torch.no_grad()
    def prelude_union(self, seq_ids, toks, cache) -> None:
        positions = [t.position for t in toks]
        pos = torch.tensor(positions, dtype=torch.long)
        x = self.W["embed"][torch.tensor([t.token_id for t in toks], dtype=torch.long)]
        for i, blk in enumerate(self.W["prelude"]):
            x = self._union_block(blk, x, [self.slot_prelude(i)] * len(toks), seq_ids, positions, pos)
        zero = torch.zeros_like(x[0])
        for i, t in enumerate(toks):
            t.static_state = x[i]
            t.hidden = zero
            t.step = 0

    @torch.no_grad()
    def advance_union(self, seq_ids, toks, cache) -> None:
        positions = [t.position for t in toks]
        pos = torch.tensor(positions, dtype=torch.long)
        h = torch.stack([t.hidden for t in toks]) + torch.stack([t.static_state for t in toks])
        for l, blk in enumerate(self.W["core"]):
            h = self._union_block(blk, h, [self.slot_core(t.step, l) for t in toks], seq_ids, positions, pos)
        for i, t in enumerate(toks):
            t.hidden = h[i]
            t.step += 1

    @torch.no_grad()
    def coda_argmax_union(self, seq_ids, toks, cache) -> list:
        positions = [t.position for t in toks]
        pos = torch.tensor(positions, dtype=torch.long)
        x = torch.stack([t.hidden for t in toks])
        for i, blk in enumerate(self.W["coda"]):
            x = self._union_block(blk, x, [self.slot_coda(i)] * len(toks), seq_ids, positions, pos)
        logits = self._rms(x, self.W["final_norm"]) @ self.W["lm_head"]
        return logits.float().argmax(dim=-1).tolist()
