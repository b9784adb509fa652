"""A tiny parcae-shaped looped LM for driving the reference's `ParcaeBlocks`
(test infrastructure; written from scratch, no parcae_lm source is available).

It exposes exactly the surface `ParcaeBlocks` and `ar_generate_parcae_blocks`
touch (src/decoding/parcae_blocks.py:74-302, ar_baseline.py:30-81,
fa4_attention.py:140-160, kv_cache.py:75-92):
  config.{clip_qkv, qk_bias, rope_settings.use_rope, qk_norm, prelude_norm,
          init.logit_scale, init.get_std, logit_softcap, n_embd,
          num_attention_heads, num_key_value_heads}
  transformer.{wte, prelude, ln_prelude, core_block, adapter, C, coda, ln_f},
  lm_head, freqs_cis, emb_scale, value_embeds, core_block_forward(...),
  blocks callable as block(x, freqs, mask, past_key_values=, step_idx=, ve=)
  that store K/V through `cache.update`.
Math (config 1 of the benchmark): RMSNorm, separate q/k/v projections,
complex-pair RoPE (dims 2i, 2i+1 rotate together), causal attention, SwiGLU,
additive input injection adapter(x, e) = x + e, identity C, no prelude norm,
logit scale 1, no softcap.  Weights: PyTorch default initialisation after
`torch.manual_seed(seed)`.

`to_looped_weights` maps the weights onto the product model
(wavefront_decoding_b200.looped_lm.LoopedLM, rope_style="interleaved").
"""
from __future__ import annotations

from types import SimpleNamespace

import torch
import torch.nn as nn
import torch.nn.functional as F

MAX_SEQ = 2048


def apply_rotary_emb_complex_like(q, k, freqs_cis):
    """q (B, T, H, Dh), k (B, T, Hkv, Dh); freqs_cis (1, T, Dh/2, 2) = (cos, sin).
    Each pair (x[2i], x[2i+1]) is multiplied by e^{i * angle_i} (complex-pair RoPE)."""
    c = freqs_cis[..., 0].unsqueeze(2)
    s = freqs_cis[..., 1].unsqueeze(2)

    def rot(x):
        xf = x.float().reshape(*x.shape[:-1], x.shape[-1] // 2, 2)
        a, b = xf[..., 0], xf[..., 1]
        return torch.stack((a * c - b * s, a * s + b * c), dim=-1).flatten(-2).to(x.dtype)

    return rot(q), rot(k)


def qk_norm(x):
    raise RuntimeError("qk_norm is off in this fixture")


def freqs_table(head_dim: int, max_seq: int, theta: float = 10000.0) -> torch.Tensor:
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float64) / head_dim))
    ang = torch.outer(torch.arange(max_seq, dtype=torch.float64), inv)
    return torch.stack((ang.cos(), ang.sin()), dim=-1).float().unsqueeze(0)    # (1, S, Dh/2, 2)


class RMSNorm(nn.Module):
    def __init__(self, d: int, eps: float = 1e-6):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(d))
        self.eps = eps

    def forward(self, x):
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps) * self.weight.float()).to(x.dtype)


class Attention(nn.Module):
    def __init__(self, d: int, n_head: int, n_kv_head: int):
        super().__init__()
        self.n_head, self.n_kv_head, self.head_dim = n_head, n_kv_head, d // n_head
        self.c_q = nn.Linear(d, n_head * self.head_dim, bias=False)
        self.c_k = nn.Linear(d, n_kv_head * self.head_dim, bias=False)
        self.c_v = nn.Linear(d, n_kv_head * self.head_dim, bias=False)
        self.c_proj = nn.Linear(n_head * self.head_dim, d, bias=False)
        self.ve_gate = None
        self.ve_gate_channels = 0

    def forward(self, x, freqs, cache, step_idx):
        B, T, _ = x.shape
        q = self.c_q(x).view(B, T, self.n_head, self.head_dim)
        k = self.c_k(x).view(B, T, self.n_kv_head, self.head_dim)
        v = self.c_v(x).view(B, T, self.n_kv_head, self.head_dim)
        q, k = apply_rotary_emb_complex_like(q, k, freqs)
        K, V = cache.update(k.transpose(1, 2), v.transpose(1, 2), step_idx)   # (B, Hkv, S, Dh)
        S = K.shape[2]
        # query row t sits at absolute position S - T + t and sees keys <= it
        keep = torch.arange(S)[None, :] <= (torch.arange(T)[:, None] + (S - T))
        o = F.scaled_dot_product_attention(q.transpose(1, 2), K, V, attn_mask=keep,
                                           enable_gqa=self.n_head != self.n_kv_head)
        return self.c_proj(o.transpose(1, 2).reshape(B, T, -1))


class SwiGLU(nn.Module):
    def __init__(self, d: int, d_ff: int):
        super().__init__()
        self.d_ff = d_ff
        self.fc = nn.Linear(d, 2 * d_ff, bias=False)
        self.proj = nn.Linear(d_ff, d, bias=False)

    def forward(self, x):
        g, u = self.fc(x).split(self.d_ff, dim=-1)
        return self.proj(F.silu(g) * u)


class Block(nn.Module):
    def __init__(self, d, n_head, n_kv_head, d_ff):
        super().__init__()
        self.norm_1 = RMSNorm(d)
        self.attn = Attention(d, n_head, n_kv_head)
        self.norm_2 = RMSNorm(d)
        self.mlp = SwiGLU(d, d_ff)

    def forward(self, x, freqs, mask=None, past_key_values=None, step_idx=None, ve=None):
        x = x + self.attn(self.norm_1(x), freqs, past_key_values, step_idx)
        return x + self.mlp(self.norm_2(x))


class Adapter(nn.Module):
    def forward(self, x, e):
        return x + e


class ParcaeFixture(nn.Module):
    def __init__(self, vocab=32000, d=512, n_head=8, n_kv_head=8, d_ff=1536, n_prelude=1, n_core=2, n_coda=1,
                 seed: int = 0):
        super().__init__()
        torch.manual_seed(seed)
        self.config = SimpleNamespace(
            clip_qkv=None, qk_bias=False, rope_settings=SimpleNamespace(use_rope=True), qk_norm=False,
            prelude_norm=False, logit_softcap=None, n_embd=d, num_attention_heads=n_head,
            num_key_value_heads=n_kv_head, d_ff=d_ff,
            init=SimpleNamespace(logit_scale=1.0, get_std=lambda name: 0.02))
        self.transformer = nn.ModuleDict(dict(
            wte=nn.Embedding(vocab, d),
            prelude=nn.ModuleList([Block(d, n_head, n_kv_head, d_ff) for _ in range(n_prelude)]),
            ln_prelude=RMSNorm(d),
            core_block=nn.ModuleList([Block(d, n_head, n_kv_head, d_ff) for _ in range(n_core)]),
            adapter=Adapter(),
            C=nn.Identity(),
            coda=nn.ModuleList([Block(d, n_head, n_kv_head, d_ff) for _ in range(n_coda)]),
            ln_f=RMSNorm(d),
        ))
        self.lm_head = nn.Linear(d, vocab, bias=False)
        self.register_buffer("freqs_cis", freqs_table(d // n_head, MAX_SEQ), persistent=False)
        self.emb_scale = 1.0
        self.value_embeds = nn.ModuleDict()
        self._current_input_ids = None

    def initialize_state(self, input_embeds):
        return torch.zeros_like(input_embeds)

    def core_block_forward(self, x, input_embeds, freqs_cis, mask, step=None, total_steps=None,
                           past_key_values=None, step_idx_base=0):
        x = self.transformer.adapter(x, input_embeds)
        for l, blk in enumerate(self.transformer.core_block):
            x = blk(x, freqs_cis, mask, past_key_values=past_key_values,
                    step_idx=torch.tensor(step_idx_base + l, dtype=torch.long))
        return x


def to_looped_weights(m: ParcaeFixture) -> dict:
    """float32 CPU weights in the layout of looped_lm.LoopedLM.load_weights."""
    def t(w):
        return w.detach().float().t().contiguous()

    def blk(b):
        a = b.attn
        return {"norm1": b.norm_1.weight.detach().float().clone(),
                "wqkv": torch.cat([t(a.c_q.weight), t(a.c_k.weight), t(a.c_v.weight)], dim=1),
                "wo": t(a.c_proj.weight), "norm2": b.norm_2.weight.detach().float().clone(),
                "wgu": t(b.mlp.fc.weight), "wd": t(b.mlp.proj.weight)}

    tr = m.transformer
    return {"embed": tr.wte.weight.detach().float().clone(), "final_norm": tr.ln_f.weight.detach().float().clone(),
            "lm_head": t(m.lm_head.weight), "prelude": [blk(b) for b in tr.prelude],
            "core": [blk(b) for b in tr.core_block], "coda": [blk(b) for b in tr.coda]}


def looped_config(m: ParcaeFixture, T_total: int, kv_budget_s: int = 0):
    """The product model config matching the fixture (kv_budget_s: the
    reference blocks' KV-sharing budget, 0 = off)."""
    from wavefront_decoding_b200.looped_lm import LoopedLMConfig
    c = m.config
    tr = m.transformer
    return LoopedLMConfig(vocab=tr.wte.num_embeddings, d_model=c.n_embd, n_heads=c.num_attention_heads,
                          n_kv_heads=c.num_key_value_heads, head_dim=c.n_embd // c.num_attention_heads,
                          d_ff=c.d_ff, n_prelude=len(tr.prelude), n_core=len(tr.core_block), n_coda=len(tr.coda),
                          T_total=T_total, rope_style="interleaved", norm_eps=1e-6, kv_budget_s=kv_budget_s)


def weight_sums(m: ParcaeFixture) -> list[float]:
    """float64 sums of a few weights: detects a change of the seeded initialisation."""
    tr = m.transformer
    ws = [tr.wte.weight, tr.prelude[0].attn.c_q.weight, tr.core_block[-1].mlp.fc.weight, m.lm_head.weight]
    return [float(w.detach().double().sum()) for w in ws]


def config1_prompt(seed: int = 0, length: int = 128, vocab: int = 32000) -> torch.Tensor:
    return torch.randint(0, vocab, (length,), generator=torch.Generator().manual_seed(seed))

