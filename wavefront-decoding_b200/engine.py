"""GPU wavefront engine: the union P / R / C blocks over the wavefront kernels,
with CUDA-graph replay.

Implements the batch-blocks interface the reference's schedulers drive
(`prefill`, `prelude_union`, `advance_union`, `coda_argmax_union`,
ouro_blocks_batch.py:123-248, huginn_blocks_batch.py:207-346), B200-first:

* Token state (hidden, injected input) lives in a device pool; the `hidden`
  of a token in flight is its pool row, so a union call gathers rows instead of stacking
  per-token tensors, and writes them back in place.
* One R tick is one attention launch per core layer for the whole union
  (`wfd_wave_attn`: window append + attention in one call, one item table shared by all
  layers through `slot_offset`), replacing the reference's per-layer
  write_tokens + gather_pack + attn_varlen (ouro_blocks_batch.py:207-231) and the
  graph engine's per-row `_fa_varlen` loop (graph_blocks.py:187-194).
* Prelude and coda tokens of one sequence may share a slot inside one call, so
  those layers append first (`wfd_append`) and then attend with explicit
  segments over the cache (`wfd_attn_segments`).
* Per call the host builds one small int32 table, uploads it with a single
  pinned copy, and replays the CUDA graph captured for the union-size bucket
  (the reference captures per WFD phase, graph_blocks.py:82-95, 362-386; here
  per bucket, so the dynamic scheduler replays graphs every tick).  Rows past
  the union point at a scratch pool row and a scratch sequence of the cache, so
  a bucket's graph is valid for any union size up to its capacity.  The only
  host sync per tick is the greedy-id read-back of the C union, as in the
  reference (scheduler_batch.py:312).
"""
from __future__ import annotations

import numpy as np
import torch

from . import attention as wa
from . import fused
from . import runtime as rt
from .kv_cache import SlotKVCache
from .looped_lm import LoopedLM

_BUCKETS = (8, 16, 32, 64, 128, 256, 512, 1024, 2048)


def _bucket(n: int) -> int:
    for b in _BUCKETS:
        if n <= b:
            return b
    raise ValueError(f"union of {n} rows exceeds the largest bucket {_BUCKETS[-1]}")


def r_windows(seq_ids: list, slot_bases: list, positions: list, gaps: bool = False):
    """Attention windows of an R union (ouro_blocks_batch.py:184-205).

    Rows of one sequence on one depth slot (KV sharing, or the sources of a
    draft-then-verify round) are reordered by (sequence, slot, position), and a
    run of consecutive positions becomes one bottom-right-causal window; with
    `gaps`, all of a sequence's rows on one slot form one window whatever the
    gaps between their positions (attended with per-row positions, the way the
    reference pads them into one span).  Returns (order, runs): order is None
    when no sequence has two rows on one slot (rows keep their order), else the
    row permutation; runs[i] is the window's row count on its first row and 0 on
    the others."""
    n = len(seq_ids)
    key = list(zip(seq_ids, slot_bases))
    order = None
    if len(set(key)) < n:
        order = sorted(range(n), key=lambda i: (key[i], positions[i]))
        key = [key[i] for i in order]
        positions = [positions[i] for i in order]
    runs = [0] * n
    i = 0
    while i < n:
        e = i + 1
        while e < n and key[e] == key[i] and (gaps or positions[e] == positions[e - 1] + 1):
            e += 1
        runs[i] = e - i
        i = e
    return order, runs


class _Tables:
    """Device tables of one (kind, bucket) and their pinned staging copy.
    int32 columns: 0 pool row, 1 position, 2 token id, 3 cache sequence,
    4 R: slot base (depth slot * n_core), P / C: 0, 5 live (q_len 1; R: the
    window's row count on its first row, 0 on the others) / padding (0),
    6.. prelude / coda layers: first cache row of the row's (slot, sequence) (the
    device scheduler's table layout; the bodies address slots by item tables)."""

    def __init__(self, kind: str, cap: int, n_cols: int, device):
        self.kind = kind
        self.cap = cap
        self.n_cols = n_cols
        self.host = torch.zeros((cap, n_cols), dtype=torch.int32).pin_memory()
        self.dev = torch.zeros((cap, n_cols), dtype=torch.int32, device=device)
        self.items = torch.zeros((cap, 5), dtype=torch.int32, device=device)
        self.out = torch.zeros(cap, dtype=torch.int32, device=device)
        self.graph = None
        self.uploaded = torch.cuda.Event()   # the staging copy may be rewritten once this fired
        self.pending = False


class WaveEngine:
    def __init__(self, model: LoopedLM, batch_size: int, max_seq_len: int, use_graphs: bool = True):
        cfg = model.cfg
        self.model = model
        self.cfg = cfg
        self.T_total = cfg.T_total
        self.B = batch_size
        self.S = max_seq_len
        self.device = model.device
        self.use_graphs = use_graphs
        # one extra sequence row: the target of padding rows
        self.cache = SlotKVCache(cfg.n_slots, batch_size + 1, cfg.n_kv_heads, cfg.head_dim, max_seq_len, model.dtype,
                                 model.device)
        self.scratch_seq = batch_size
        # state pool: live tokens are at most B * (T_total / T_draft + 2) per tick;
        # round-robin reuse over this many rows never recycles a live row
        self.pool_cap = batch_size * 2 * (cfg.T_total + 8)
        self.scratch_row = self.pool_cap
        d = cfg.d_model
        self.pool_h = torch.zeros((self.pool_cap + 1, d), dtype=model.dtype, device=self.device)
        self.pool_e = torch.zeros((self.pool_cap + 1, d), dtype=model.dtype, device=self.device)
        self._next_row = 0
        model.rope_tables(max_seq_len)
        self._tables: dict[tuple[str, int], _Tables] = {}
        rt.reserve_workspace(self.device, _BUCKETS[-1], cfg.head_dim)
        rt.error_word(self.device)
        self.n_graph_replays = 0
        self.n_launch_calls = 0
        # accounting (host side, exact): K/V bytes the attention of live rows
        # reads, libwfd kernel launches, bytes read back per C union
        self._row_bytes = cfg.n_kv_heads * cfg.head_dim * torch.finfo(model.dtype).bits // 8
        # every libwfd kernel a body launches.  Per layer: 2 RMSNorm, RoPE split,
        # plan (with the window append), attention (tcgen05 or CUDA-core), SwiGLU
        # gate.  Per body: P gather + item table + scatter, R gather + item table +
        # scatter, C gather + item table + final RMSNorm + greedy argmax.
        # With the norms folded into the next layer (bf16) the two RMSNorm launches of
        # a layer and the final RMSNorm of the C body are gone.
        per_layer = 4 if model.fold_norms else 6
        self._launches = {"P": 3 + per_layer * cfg.n_prelude, "R": 3 + per_layer * cfg.n_core,
                          "C": (3 if model.fold_norms else 4) + per_layer * cfg.n_coda}
        self._layers = {"P": cfg.n_prelude, "R": cfg.n_core, "C": cfg.n_coda}
        # rows per R attention window: 1 without KV sharing; with sharing a run of
        # one sequence's tokens on one depth slot (at most T_total + 2 tokens live)
        self.r_max_q = 1 if cfg.n_depth_slots == cfg.T_total else cfg.T_total + 2
        # KV sharing: a sequence's tokens on one depth slot attend as one window,
        # gaps included, on the tensor-core kernel (per-row positions); the fp32
        # CUDA-core kernel keeps one window per run of consecutive positions
        self.gap_windows = cfg.n_depth_slots < cfg.T_total and self.model.dtype == torch.bfloat16
        self.kv_read_bytes = 0
        self.wfd_launches = 0
        self.d2h_bytes = 0

    # ------------------------------------------------------------------
    def synchronize(self) -> None:
        torch.cuda.synchronize(self.device)

    def ensure_window_rows(self, n: int) -> None:
        """Let an R window (a run of one sequence's tokens on one depth slot)
        hold up to n rows, e.g. the K + 1 sources of a draft-then-verify round.
        Captured R graphs bake the bound in and are dropped when it grows."""
        if n > self.r_max_q:
            self.r_max_q = n
            for (kind, _), t in self._tables.items():
                if kind == "R":
                    t.graph = None

    def drop_positions_at_and_after(self, b: int, position: int) -> None:
        self.cache.drop_positions_at_and_after(b, position)

    def _alloc_rows(self, n: int) -> list[int]:
        rows = [(self._next_row + i) % self.pool_cap for i in range(n)]
        self._next_row = (self._next_row + n) % self.pool_cap
        return rows

    def _seg_layers(self, kind: str) -> list[int]:
        cfg = self.cfg
        if kind == "P":
            return [cfg.slot_prelude(i) for i in range(cfg.n_prelude)]
        if kind == "C":
            return [cfg.slot_coda(i) for i in range(cfg.n_coda)]
        return []

    def _fill(self, kind: str, toks, seq_ids, rows) -> _Tables:
        cfg = self.cfg
        n = len(toks)
        runs = None
        if kind == "R":
            order, runs = r_windows([int(x) for x in seq_ids], [cfg.core_slot_base(tk.step) for tk in toks],
                                    [tk.position for tk in toks], gaps=self.gap_windows)
            if order is not None:
                toks = [toks[i] for i in order]
                seq_ids = [seq_ids[i] for i in order]
                rows = [rows[i] for i in order]
            if max(runs, default=0) > self.r_max_q:
                raise ValueError(f"R window of {max(runs)} rows exceeds {self.r_max_q}")
        cap = _bucket(n)
        t = self._tables.get((kind, cap))
        seg_slots = self._seg_layers(kind)
        if t is None:
            t = _Tables(kind, cap, 6 + len(seg_slots), self.device)
            self._tables[(kind, cap)] = t
        if t.pending:
            t.uploaded.synchronize()
        a = t.host.numpy()
        a[:] = 0
        a[:, 0] = self.scratch_row
        a[:, 3] = self.scratch_seq
        a[:n, 0] = rows
        a[:n, 1] = [tk.position for tk in toks]
        a[:n, 2] = [tk.token_id for tk in toks]
        a[:n, 3] = seq_ids
        if kind == "R":
            a[:n, 4] = [cfg.core_slot_base(tk.step) for tk in toks]
            a[:n, 5] = runs
        else:
            a[:n, 5] = 1
        for j, slot in enumerate(seg_slots):
            a[:, 6 + j] = (slot * (self.B + 1) + a[:, 3].astype(np.int64)) * self.S
        t.dev.copy_(t.host, non_blocking=True)
        t.uploaded.record()
        t.pending = True
        # K/V read: k_len = position + 1 of each window's last row (once per run)
        if runs is None:
            keys = int(a[:n, 1].sum()) + n
        else:
            keys = sum(int(a[i + runs[i] - 1, 1]) + 1 for i in range(n) if runs[i] > 0)
        self.kv_read_bytes += keys * self._layers[kind] * 2 * self._row_bytes
        self.wfd_launches += self._launches[kind]
        return t

    def reset_counters(self) -> None:
        self.kv_read_bytes = 0
        self.wfd_launches = 0
        self.d2h_bytes = 0

    def _padding_rows(self, t: _Tables) -> torch.Tensor:
        """A table of t's shape whose rows are all padding."""
        pad = torch.zeros_like(t.dev)
        pad[:, 0] = self.scratch_row
        pad[:, 3] = self.scratch_seq
        for j, slot in enumerate(self._seg_layers(t.kind)):
            pad[:, 6 + j] = (slot * (self.B + 1) + self.scratch_seq) * self.S
        return pad

    # ------------------------------------------------------------------
    # device-side bodies (captured into graphs)
    def _segment_block(self, blk, x, t: _Tables, slot: int):
        """Prelude / coda layer: one wave_attn over the body's item table with the
        layer's slot as the offset.  Several rows of a sequence may share the
        slot (the C union's commit and draft rows): every row's K / V is appended
        before any row attends."""
        m = self.model
        q, k, v = m.qkv(blk, x, pos=t.dev[:, 1])
        o = wa.wave_attn(q, k, v, self.cache.K, self.cache.V, t.items, 1, lens=self.cache.lens, slot_offset=slot)
        return m.finish_block(blk, x, o)

    def _body(self, kind: str, t: _Tables) -> None:
        m, cfg = self.model, self.cfg
        tab = t.dev
        rows = tab[:, 0]
        if kind == "P":
            x = fused.gather_rows(m.embed, tab[:, 2])
            fused.items_from_table(tab, 4, 3, 1, 5, t.items)   # (0, seq, position, live, row)
            for j, blk in enumerate(m.prelude):
                x = self._segment_block(blk, x, t, cfg.slot_prelude(j))
            fused.scatter_rows(x, rows, self.pool_e, zero=self.pool_h)
        elif kind == "R":
            x = fused.gather_rows(self.pool_h, rows, b=self.pool_e)
            fused.items_from_table(tab, 4, 3, 1, 5, t.items)   # (slot base, seq, position, live, row)
            for l, blk in enumerate(m.core):
                q, k, v = m.qkv(blk, x, pos=tab[:, 1])
                o = wa.wave_attn(q, k, v, self.cache.K, self.cache.V, t.items, self.r_max_q, lens=self.cache.lens,
                                 slot_offset=cfg.n_prelude + l, row_pos=tab[:, 1] if self.gap_windows else None)
                x = m.finish_block(blk, x, o)
            fused.scatter_rows(x, rows, self.pool_h)
        else:
            x = fused.gather_rows(self.pool_h, rows)
            fused.items_from_table(tab, 4, 3, 1, 5, t.items)
            for j, blk in enumerate(m.coda):
                x = self._segment_block(blk, x, t, cfg.slot_coda(j))
            m.greedy_ids(x, t.out)

    def _run(self, kind: str, t: _Tables) -> None:
        self.n_launch_calls += 1
        if not self.use_graphs:
            self._body(kind, t)
            return
        if t.graph is None:
            # The R body advances pool rows in place (not idempotent), so the
            # warm-up runs see a table of padding rows only (scratch pool row,
            # scratch sequence, q_len 0); the real table goes back before the
            # first replay.
            cur = torch.cuda.current_stream(self.device)
            real = t.dev.clone()
            t.dev.copy_(self._padding_rows(t))
            side = torch.cuda.Stream(self.device)
            side.wait_stream(cur)
            with torch.cuda.stream(side):
                for _ in range(2):
                    self._body(kind, t)
            cur.wait_stream(side)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self._body(kind, t)
            t.graph = g
            t.dev.copy_(real)
        t.graph.replay()
        self.n_graph_replays += 1

    # ------------------------------------------------------------------
    # reference blocks interface
    @torch.no_grad()
    def prefill(self, prompt_ids: torch.Tensor):
        B, L = prompt_ids.shape
        assert B == self.B, f"prefill expects (B={self.B}, L) prompt ids"
        self.cache.lens.zero_()
        ids = prompt_ids.to(self.device)
        pad = torch.zeros((1, L), dtype=ids.dtype, device=self.device)
        last_logits = self.model.prefill_dense(torch.cat([ids, pad]), self.cache)[:B]
        return self, last_logits

    @torch.no_grad()
    def prelude_union(self, seq_ids, toks, cache) -> None:
        rows = self._alloc_rows(len(toks))
        t = self._fill("P", toks, seq_ids, rows)
        self._run("P", t)
        for tk, r in zip(toks, rows):
            tk.hidden = r
            tk.static_state = r
            tk.step = 0

    @torch.no_grad()
    def advance_union(self, seq_ids, toks, cache) -> None:
        t = self._fill("R", toks, seq_ids, [tk.hidden for tk in toks])
        self._run("R", t)
        for tk in toks:
            tk.step += 1

    @torch.no_grad()
    def coda_argmax_union(self, seq_ids, toks, cache) -> list[int]:
        t = self._fill("C", toks, seq_ids, [tk.hidden for tk in toks])
        self._run("C", t)
        self.d2h_bytes += 4 * len(toks)
        return t.out[:len(toks)].tolist()

    # reporting
    @property
    def nbytes(self) -> int:
        return self.cache.nbytes
