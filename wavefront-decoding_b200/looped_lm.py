"""Random-init looped (recurrent-depth) language model whose attention runs on
the wavefront kernels.

Architecture (the P / R / C split of the reference's looped models,
src/decoding/blocks.py:22-116, parcae_blocks.py:283-518,
huginn_blocks_batch.py:1-31):
  P  embedding -> n_prelude blocks; its output e is the loop's injected input
  R  one loop step: x <- x + e (additive input injection), then n_core blocks
  C  n_coda blocks -> final RMSNorm -> lm_head
Block: RMSNorm -> fused QKV -> RoPE -> attention over this block's KV slot ->
o_proj -> residual -> RMSNorm -> SwiGLU -> residual.
KV slots (kv_cache.py:12-15 of the reference): prelude layer i -> i; core
(depth r, layer l) -> n_prelude + r * n_core + l; coda layer i ->
n_prelude + T_total * n_core + i.

Weights are plain tensors; GEMMs are cuBLAS (torch.matmul / addmm, residual adds
in the GEMM epilogue), attention and the element-wise block work (RMSNorm, RoPE
+ QKV split, SwiGLU gate) are libwfd_b200 kernels.  Prefill attention (the
one-shot prompt pass) uses torch's fused SDPA; every decode-time attention uses
the wavefront kernels.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from . import attention
from . import fused


@dataclass
class LoopedLMConfig:
    vocab: int = 32000
    d_model: int = 512
    n_heads: int = 8
    n_kv_heads: int = 8
    head_dim: int = 64
    d_ff: int = 1536
    n_prelude: int = 1
    n_core: int = 2
    n_coda: int = 1
    T_total: int = 4          # loop depth R
    rope_theta: float = 10000.0
    rope_style: str = "half"  # "half": dims i, i + Dh/2 rotate together; "interleaved": dims 2i, 2i+1
    norm_eps: float = 1e-6
    init_std: float = 0.02
    # KV sharing across loop depths (parcae_blocks.py:77-81,114-120,
    # ouro_blocks_batch.py:15-18,66-78): with a budget 0 < s < T_total, core
    # depth r keeps its K/V in depth slot r % s (the last depth to write a
    # position wins) and the cache holds s depth slots instead of T_total.
    # 0 = off (one slot per depth, lossless).
    kv_budget_s: int = 0

    @property
    def n_depth_slots(self) -> int:
        s = self.kv_budget_s
        return s if 0 < s < self.T_total else self.T_total

    @property
    def n_slots(self) -> int:
        return self.n_prelude + self.n_depth_slots * self.n_core + self.n_coda

    def slot_prelude(self, i: int) -> int:
        return i

    def core_slot_base(self, r: int) -> int:
        """First core slot of loop depth r, relative to the prelude slots (r % s * n_core)."""
        return (r % self.n_depth_slots) * self.n_core

    def slot_core(self, r: int, l: int) -> int:
        return self.n_prelude + self.core_slot_base(r) + l

    def slot_coda(self, i: int) -> int:
        return self.n_prelude + self.n_depth_slots * self.n_core + i

    def n_params(self) -> int:
        d, Dh = self.d_model, self.head_dim
        per_layer = d * (self.n_heads + 2 * self.n_kv_heads) * Dh + self.n_heads * Dh * d + 3 * d * self.d_ff + 2 * d
        return 2 * self.vocab * d + d + (self.n_prelude + self.n_core + self.n_coda) * per_layer


# the configurations BASELINE.json names
CONFIG1 = LoopedLMConfig()  # vocab 32000, d 512, 8 x 64, SwiGLU 1536, prelude 1 / core 2 x R=4 / coda 1
CONFIG4 = LoopedLMConfig(vocab=50304, d_model=1536, n_heads=24, n_kv_heads=24, head_dim=64, d_ff=4096,
                         n_prelude=2, n_core=4, n_coda=2, T_total=8)


class Block:
    def __init__(self, cfg: LoopedLMConfig, g: torch.Generator, dtype, device):
        d, Dh, H, Hkv = cfg.d_model, cfg.head_dim, cfg.n_heads, cfg.n_kv_heads
        std = cfg.init_std

        def w(*shape, scale=1.0):
            return (torch.randn(shape, generator=g) * (std * scale)).to(dtype=dtype, device=device)

        self.norm1 = torch.ones(d, dtype=dtype, device=device)
        self.wqkv = w(d, (H + 2 * Hkv) * Dh)
        self.wo = w(H * Dh, d, scale=1.0 / math.sqrt(2.0))
        self.norm2 = torch.ones(d, dtype=dtype, device=device)
        self.wgu = w(d, 2 * cfg.d_ff)
        self.wd = w(cfg.d_ff, d, scale=1.0 / math.sqrt(2.0))


class LoopedLM:
    def __init__(self, cfg: LoopedLMConfig, seed: int = 0, dtype=torch.bfloat16, device="cuda"):
        self.cfg = cfg
        self.dtype = dtype
        self.device = torch.device(device)
        g = torch.Generator().manual_seed(seed)
        d = cfg.d_model
        self.embed = (torch.randn((cfg.vocab, d), generator=g) * 1.0).to(dtype=dtype, device=self.device)
        self.prelude = [Block(cfg, g, dtype, self.device) for _ in range(cfg.n_prelude)]
        self.core = [Block(cfg, g, dtype, self.device) for _ in range(cfg.n_core)]
        self.coda = [Block(cfg, g, dtype, self.device) for _ in range(cfg.n_coda)]
        self.final_norm = torch.ones(d, dtype=dtype, device=self.device)
        self.lm_head = (torch.randn((d, cfg.vocab), generator=g) * (1.0 / math.sqrt(d))).to(dtype=dtype,
                                                                                           device=self.device)
        self._rope_cache = None
        # bf16: every RMSNorm is folded into the linear layer after it (its weight
        # multiplied into that layer's rows, its row scale applied by the kernel that
        # follows the GEMM), one launch fewer per norm; fp32 keeps the explicit norm,
        # the reference's own arithmetic
        self.fold_norms = dtype == torch.bfloat16
        self._fold()

    def _fold(self) -> None:
        if not self.fold_norms:
            return
        for blk in self.prelude + self.core + self.coda:
            blk.wqkv_n = fused.fold_norm(blk.wqkv, blk.norm1)
            blk.wgu_n = fused.fold_norm(blk.wgu, blk.norm2)
        self.lm_head_n = fused.fold_norm(self.lm_head, self.final_norm)

    def load_weights(self, W: dict) -> "LoopedLM":
        """Replace every weight from a dict of tensors: embed (V, d), final_norm (d),
        lm_head (d, V), and lists prelude / core / coda of per-block dicts with
        norm1, wqkv (d, (H + 2 Hkv) Dh), wo (H Dh, d), norm2, wgu (d, 2 d_ff), wd (d_ff, d)."""
        def put(t, ref):
            assert tuple(t.shape) == tuple(ref.shape), (tuple(t.shape), tuple(ref.shape))
            return t.to(dtype=self.dtype, device=self.device).contiguous()

        self.embed = put(W["embed"], self.embed)
        self.final_norm = put(W["final_norm"], self.final_norm)
        self.lm_head = put(W["lm_head"], self.lm_head)
        for name in ("prelude", "core", "coda"):
            blocks = getattr(self, name)
            assert len(W[name]) == len(blocks)
            for blk, wb in zip(blocks, W[name]):
                for k in ("norm1", "wqkv", "wo", "norm2", "wgu", "wd"):
                    setattr(blk, k, put(wb[k], getattr(blk, k)))
        self._fold()
        return self

    # ------------------------------------------------------------------
    def rope_tables(self, max_seq: int):
        """(max_seq, Dh/2) fp32 cos / sin tables (grown on demand, kept on the device)."""
        if self._rope_cache is None or self._rope_cache[0].shape[0] < max_seq:
            Dh = self.cfg.head_dim
            inv = 1.0 / (self.cfg.rope_theta ** (torch.arange(0, Dh, 2, dtype=torch.float64) / Dh))
            t = torch.arange(max_seq, dtype=torch.float64)
            ang = torch.outer(t, inv)
            self._rope_cache = (ang.cos().float().contiguous().to(self.device),
                                ang.sin().float().contiguous().to(self.device))
        return self._rope_cache

    def rmsnorm(self, x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        return fused.rmsnorm(x, w, self.cfg.norm_eps)

    def qkv(self, blk: Block, x: torch.Tensor, pos: torch.Tensor | None = None, pos_period: int = 0):
        """Norm, fused QKV projection, RoPE.  x (n, d) with positions `pos` (int32,
        one per row), or x (B, L, d) at positions 0..L-1 (pos_period = L).
        Returns contiguous q (.., H, Dh), k / v (.., Hkv, Dh)."""
        cfg = self.cfg
        lead = x.shape[:-1]
        cos, sin = self._rope_cache
        if self.fold_norms:
            x2 = x.reshape(-1, cfg.d_model)
            q, k, v = fused.rope_split(x2 @ blk.wqkv_n, cos, sin, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, pos=pos,
                                       pos_period=pos_period, interleaved=cfg.rope_style == "interleaved",
                                       norm_x=x2, norm_eps=cfg.norm_eps)
        else:
            h = self.rmsnorm(x, blk.norm1).reshape(-1, cfg.d_model)
            q, k, v = fused.rope_split(h @ blk.wqkv, cos, sin, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, pos=pos,
                                       pos_period=pos_period, interleaved=cfg.rope_style == "interleaved")
        return (q.view(*lead, cfg.n_heads, cfg.head_dim), k.view(*lead, cfg.n_kv_heads, cfg.head_dim),
                v.view(*lead, cfg.n_kv_heads, cfg.head_dim))

    def finish_block(self, blk: Block, x: torch.Tensor, attn: torch.Tensor) -> torch.Tensor:
        """x + o_proj(attn), then x + SwiGLU(norm(x)); the residual adds ride on the
        GEMMs (beta = 1), which update the residual stream x IN PLACE (x must be
        contiguous and owned by the caller) and return it."""
        cfg = self.cfg
        shp = x.shape
        x2 = x.view(-1, cfg.d_model)
        x2.addmm_(attn.reshape(-1, cfg.n_heads * cfg.head_dim), blk.wo)
        if self.fold_norms:
            a = fused.silu_mul(x2 @ blk.wgu_n, norm_x=x2, norm_eps=cfg.norm_eps)
        else:
            a = fused.silu_mul(self.rmsnorm(x2, blk.norm2) @ blk.wgu)
        return x2.addmm_(a, blk.wd).view(shp)

    def logits(self, x: torch.Tensor) -> torch.Tensor:
        return (self.rmsnorm(x.contiguous(), self.final_norm) @ self.lm_head).float()

    def greedy_ids(self, x: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        """out (int32) = argmax of each row's logits (first maximum), without an fp32 copy.
        With folded norms the final RMSNorm's weight sits in lm_head_n and its row
        scale, positive, leaves the argmax unchanged: it is not computed."""
        if self.fold_norms:
            return fused.argmax_rows(x.contiguous() @ self.lm_head_n, out)
        return fused.argmax_rows(self.rmsnorm(x.contiguous(), self.final_norm) @ self.lm_head, out)

    # ------------------------------------------------------------------
    @torch.no_grad()
    def prefill_dense(self, ids: torch.Tensor, cache) -> torch.Tensor:
        """Prompt pass for every sequence at positions [0, L): fills every KV
        slot and returns the full-depth logits at the last position (B, V)."""
        cfg = self.cfg
        B, L = ids.shape
        self.rope_tables(max(L, cache.S))

        def dense_block(blk, x, slot):
            q, k, v = self.qkv(blk, x, pos_period=L)                     # (B, L, H|Hkv, Dh)
            cache.write_prefill(slot, k, v)
            o = attention.attn_dense(q, k, v, causal=True)               # (B, L, H, Dh), libwfd kernels
            return self.finish_block(blk, x, o)

        x = self.embed[ids]
        for i, blk in enumerate(self.prelude):
            x = dense_block(blk, x, cfg.slot_prelude(i))
        e = x
        h = torch.zeros_like(e)
        for r in range(cfg.T_total):
            h = h + e
            for l, blk in enumerate(self.core):
                h = dense_block(blk, h, cfg.slot_core(r, l))
        x = h
        for i, blk in enumerate(self.coda):
            x = dense_block(blk, x, cfg.slot_coda(i))
        return self.logits(x[:, -1])
