"""Plain sequential loop decoding of the looped LM, recomputed from scratch for
every token in float64 on the CPU (test oracle).

The reference's sequential baseline (`ar_generate_parcae_blocks`,
src/decoding/ar_baseline.py:132-193) runs, per token, the prelude, T_total
loop steps of the core and the coda with KV caching per (layer, depth) slot.
Caching only stores values that a full causal recompute over the whole
sequence produces again, so this oracle recomputes the whole sequence at every
step: the engine's slot bookkeeping (which depth's K/V lives where, rollback,
wave ordering) has nothing to hide behind.

Weights come as plain tensors (the names of looped_lm.LoopedLM); the math is
the same architecture: prelude -> (h <- h + e; core) x T_total -> coda ->
RMSNorm -> lm_head, blocks = RMSNorm / QKV / rotate-half RoPE / causal GQA
attention / o_proj / RMSNorm / SwiGLU.
"""
from __future__ import annotations

import math

import torch


def _rms(x, w, eps):
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w


def _rope(x, pos, theta, style="half"):
    """Pairs (i, i + Dh/2) ("half") or (2i, 2i + 1) ("interleaved") rotate by angle
    pos * theta^(-2i/Dh)."""
    Dh = x.shape[-1]
    inv = 1.0 / (theta ** (torch.arange(0, Dh, 2, dtype=torch.float64) / Dh))
    ang = torch.outer(pos.double(), inv)            # (T, Dh/2)
    c, s = ang.cos()[:, None, :], ang.sin()[:, None, :]
    if style == "interleaved":
        a, b = x[..., 0::2], x[..., 1::2]
        return torch.stack((a * c - b * s, a * s + b * c), dim=-1).flatten(-2)
    x1, x2 = x[..., : Dh // 2], x[..., Dh // 2:]
    return torch.cat((x1 * c - x2 * s, x2 * c + x1 * s), dim=-1)


def _block(blk, x, cfg, kv_out=None):
    """One block over positions [0, T); appends the stored (post-RoPE) K and the
    V, each (T, Hkv, Dh), to kv_out when given."""
    T = x.shape[0]
    H, Hkv, Dh = cfg["n_heads"], cfg["n_kv_heads"], cfg["head_dim"]
    pos = torch.arange(T)
    h = _rms(x, blk["norm1"], cfg["norm_eps"]) @ blk["wqkv"]
    q, k, v = torch.split(h, [H * Dh, Hkv * Dh, Hkv * Dh], dim=-1)
    style = cfg.get("rope_style", "half")
    q = _rope(q.reshape(T, H, Dh), pos, cfg["rope_theta"], style)
    k = _rope(k.reshape(T, Hkv, Dh), pos, cfg["rope_theta"], style)
    v = v.reshape(T, Hkv, Dh)
    if kv_out is not None:
        kv_out.append((k, v))
    G = H // Hkv
    k = k.repeat_interleave(G, dim=1)
    v = v.repeat_interleave(G, dim=1)
    s = torch.einsum("qhd,khd->hqk", q, k) / math.sqrt(Dh)
    mask = torch.arange(T)[None, :] <= torch.arange(T)[:, None]
    s = s.masked_fill(~mask[None], float("-inf"))
    o = torch.einsum("hqk,khd->qhd", torch.softmax(s, dim=-1), v).reshape(T, H * Dh)
    x = x + o @ blk["wo"]
    gu = _rms(x, blk["norm2"], cfg["norm_eps"]) @ blk["wgu"]
    g, u = gu.split(cfg["d_ff"], dim=-1)
    return x + (torch.nn.functional.silu(g) * u) @ blk["wd"]


def last_logits(W: dict, cfg: dict, ids: torch.Tensor, draft_depth: int | None = None) -> torch.Tensor:
    """Logits at the last position of `ids` after the full T_total loop steps.
    With draft_depth d, the last position leaves the loop after d steps instead
    (a draft): its coda attends to the earlier positions' full-depth coda K/V
    and to its own depth-d row, as the draft C pass of a wavefront does
    (parcae_blocks.py:472-518, the draft copy is taken at step == T_draft,
    :567-573)."""
    x = W["embed"][ids]
    for blk in W["prelude"]:
        x = _block(blk, x, cfg)
    e = x
    h = torch.zeros_like(e)
    h_draft = None
    for r in range(cfg["T_total"]):
        h = h + e
        for blk in W["core"]:
            h = _block(blk, h, cfg)
        if draft_depth is not None and r + 1 == draft_depth:
            h_draft = h[-1:].clone()
    x = h if h_draft is None else torch.cat((h[:-1], h_draft))
    for blk in W["coda"]:
        x = _block(blk, x, cfg)
    return _rms(x[-1], W["final_norm"], cfg["norm_eps"]) @ W["lm_head"]


def slot_kv(W: dict, cfg: dict, ids: torch.Tensor) -> list[tuple[torch.Tensor, torch.Tensor]]:
    """K / V that every slot holds for positions [0, len(ids)) after sequential
    decoding, indexed by slot id: prelude layer i -> i, core (depth r, layer l)
    -> n_prelude + r * n_core + l, coda layer i -> n_prelude + T_total * n_core + i
    (kv_cache.py:12-15).  A causal recompute produces exactly the entries that
    incremental decoding caches."""
    kv = []
    x = W["embed"][ids]
    for blk in W["prelude"]:
        x = _block(blk, x, cfg, kv)
    e = x
    h = torch.zeros_like(e)
    for _ in range(cfg["T_total"]):
        h = h + e
        for blk in W["core"]:
            h = _block(blk, h, cfg, kv)
    for blk in W["coda"]:
        h = _block(blk, h, cfg, kv)
    return kv


def greedy_generate(W: dict, cfg: dict, prompt: list[int], n_new: int) -> list[int]:
    """First token from the prompt, then n_new - 1 more, each by full recompute."""
    ids = list(prompt)
    out = []
    for _ in range(n_new):
        tok = int(last_logits(W, cfg, torch.tensor(ids)).argmax())
        out.append(tok)
        ids.append(tok)
    return out


def weights_from(model) -> tuple[dict, dict]:
    """float64 CPU copies of a looped_lm.LoopedLM's weights and its config."""
    def f(t):
        return t.detach().to("cpu", torch.float64)

    def blk(b):
        return {k: f(getattr(b, k)) for k in ("norm1", "wqkv", "wo", "norm2", "wgu", "wd")}

    W = {"embed": f(model.embed), "final_norm": f(model.final_norm), "lm_head": f(model.lm_head),
         "prelude": [blk(b) for b in model.prelude], "core": [blk(b) for b in model.core],
         "coda": [blk(b) for b in model.coda]}
    c = model.cfg
    cfg = {k: getattr(c, k) for k in ("n_heads", "n_kv_heads", "head_dim", "d_ff", "T_total", "norm_eps",
                                      "rope_theta", "rope_style")}
    return W, cfg
