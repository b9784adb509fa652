"""Numpy restatement of the reference's SDPA reference twins (test oracle).

Reference: src/decoding/fa4_attention.py
  _attn_dense_sdpa          :218-232   bottom-right causal when Tq != Tk
  _attn_cutoff_multi_sdpa   :281-291   per-query key cutoff  key j <= qpos[m]
  _attn_varlen_sdpa         :369-381   loop over cu_seqlens segments
  attn_varlen_q1_padded     :320-342   == q_len 1, causal=False
SDPA semantics: scale 1/sqrt(Dh), softmax over keys, GQA query head h reads kv
head h // (H / Hkv) (enable_gqa).  Arithmetic in float64 on the given inputs
(bf16 inputs are widened exactly).  Rows that see no key return zeros.
"""
from __future__ import annotations

import numpy as np


def _f64(x) -> np.ndarray:
    try:
        import torch
        if isinstance(x, torch.Tensor):
            return x.detach().to("cpu", dtype=torch.float64).numpy()
    except ImportError:  # pragma: no cover
        pass
    return np.asarray(x, dtype=np.float64)


def _segment(q: np.ndarray, k: np.ndarray, v: np.ndarray, limits: np.ndarray, scale: float) -> np.ndarray:
    """q (sq, H, Dh), k/v (sk, Hkv, Dh), limits (sq,): row r sees keys j <= limits[r]."""
    sq, H, Dh = q.shape
    sk, Hkv, _ = k.shape
    G = H // Hkv
    if sq == 0:
        return np.zeros((0, H, Dh))
    qg = q.reshape(sq, Hkv, G, Dh).transpose(1, 2, 0, 3)            # (Hkv, G, sq, Dh)
    kt = k.transpose(1, 0, 2)                                        # (Hkv, sk, Dh)
    vt = v.transpose(1, 0, 2)
    # batched matrix products per kv head (BLAS), float64
    s = np.matmul(qg.reshape(Hkv, G * sq, Dh), kt.transpose(0, 2, 1)).reshape(Hkv, G, sq, sk) * scale
    mask = np.arange(sk)[None, :] <= limits[:, None]                 # (sq, sk)
    s = np.where(mask[None, None], s, -np.inf)
    m = s.max(axis=-1, keepdims=True)
    m = np.where(np.isfinite(m), m, 0.0)
    p = np.exp(s - m)
    p = np.where(mask[None, None], p, 0.0)
    l = p.sum(axis=-1, keepdims=True)
    o = np.matmul(p.reshape(Hkv, G * sq, sk), vt).reshape(Hkv, G, sq, Dh) / np.where(l > 0, l, 1.0)
    return o.transpose(2, 0, 1, 3).reshape(sq, H, Dh)                # (sq, H, Dh)


def attn_varlen(q, k, v, cu_q, cu_k, causal: bool = False, scale: float | None = None) -> np.ndarray:
    """fa4_attention._attn_varlen_sdpa (:369-381) -> _attn_dense_sdpa (:218-232).
    q (total_q, H, Dh), k/v (total_k, Hkv, Dh); segment i = rows cu[i]:cu[i+1]."""
    q, k, v = _f64(q), _f64(k), _f64(v)
    cu_q = [int(x) for x in np.asarray(cu_q).tolist()]
    cu_k = [int(x) for x in np.asarray(cu_k).tolist()]
    scale = 1.0 / np.sqrt(q.shape[-1]) if scale is None else scale
    out = np.zeros(q.shape, dtype=np.float64)
    for i in range(len(cu_q) - 1):
        q0, q1, k0, k1 = cu_q[i], cu_q[i + 1], cu_k[i], cu_k[i + 1]
        sq, sk = q1 - q0, k1 - k0
        if sq == 0:
            continue
        r = np.arange(sq)
        # _attn_dense_sdpa: causal and Tq != Tk -> key j <= r + (Tk - Tq);
        # causal and Tq == Tk -> is_causal (the same rule); else every key.
        limits = r + (sk - sq) if causal else np.full(sq, sk - 1)
        out[q0:q1] = _segment(q[q0:q1], k[k0:k1], v[k0:k1], limits, scale)
    return out


def attn_dense(q, k, v, *, causal: bool, scale: float | None = None) -> np.ndarray:
    """fa4_attention._attn_dense_sdpa (:218-232): q (B, Tq, H, Dh), k/v (B, Tk, Hkv, Dh)."""
    q, k, v = _f64(q), _f64(k), _f64(v)
    B, Tq, H, Dh = q.shape
    Tk = k.shape[1]
    scale = 1.0 / np.sqrt(Dh) if scale is None else scale
    r = np.arange(Tq)
    limits = r + (Tk - Tq) if (causal and Tq > 1) else np.full(Tq, Tk - 1)
    return np.stack([_segment(q[b], k[b], v[b], limits, scale) for b in range(B)])


def attn_cutoff_multi(q, k, v, qpos, scale: float | None = None) -> np.ndarray:
    """fa4_attention._attn_cutoff_multi_sdpa (:281-291): query m sees keys j <= qpos[m]."""
    q, k, v = _f64(q), _f64(k), _f64(v)
    scale = 1.0 / np.sqrt(q.shape[-1]) if scale is None else scale
    limits = np.asarray([int(p) for p in qpos])
    return _segment(q[0], k[0], v[0], limits, scale)[None]
