"""Wavefront decoding with the route / settle on the GPU: one CUDA graph per tick.

`generate_wavefront_device(engine, prompt_ids, max_new_tokens, policy, emus)`
has the signature and result (a scheduler.BatchTrace) of
scheduler.generate_wavefront_batch, which mirrors the reference's host
scheduler (scheduler_batch.py:228-362).  The decisions are the same, field by
field; what moves is where they run: the P / R / C unions, the routing of
commit and draft points, the accept-or-reject cascade, rollbacks (KV lengths
truncated on the device) and the queueing of the next tokens are all device
work captured in one graph, replayed tick after tick.  The host reads nothing
per tick; between chunks of ticks it reads the committed counts, and replays
at least as many ticks as the slowest sequence still needs (each tick commits
at most one token per sequence), so no tick runs after the last commit.

Emulated acceptance draws (EmulatedAcceptance) are taken on the host in the
same order the host scheduler consumes them and uploaded once.

batch_invariant=True gives bit-exact greedy equality of wavefront and
sequential decoding (T_draft = T_total) in bf16: every union runs at a fixed
row capacity that does not depend on T_draft (so each GEMM sees the same shape
in every run, and a row's result does not depend on its neighbours), and the
attention runs in the library's batch-invariant mode (no split, no merge).
"""
from __future__ import annotations

import copy
import ctypes
import time

import torch

from . import _abi
from . import runtime as rt
from .engine import WaveEngine, _Tables
from .scheduler import BatchTrace, GenerationTrace, SsdPolicy

_CT = ("n_p_calls", "n_r_calls", "n_c_calls", "n_drafts_proposed", "n_drafts_accepted", "n_drafts_rejected",
       "n_rollback_events")


class DeviceWave:
    """Device scheduling state and the tick graph for one engine / length budget."""

    def __init__(self, engine: WaveEngine, max_new_tokens: int, policy: SsdPolicy, batch_invariant: bool = False):
        eng = engine
        cfg = eng.cfg
        if policy.T_total != cfg.T_total:
            raise ValueError(f"policy T_total {policy.T_total} != model loop depth {cfg.T_total}")
        self.eng = eng
        self.policy = policy
        self.max_new = max_new_tokens
        self.batch_invariant = batch_invariant
        B = eng.B
        self.B = B
        self.W = cfg.T_total + 2
        if B * self.W > eng.pool_cap:
            raise ValueError("engine state pool too small for the device token slots")
        if B > 1024 or self.W > 32:
            raise ValueError("device scheduling supports B <= 1024 sequences and loop depth <= 30")
        dev = eng.device
        self.device = dev
        i32 = dict(dtype=torch.int32, device=dev)
        n = B * self.W
        self.alive = torch.zeros(n, **i32)
        self.state = torch.zeros(n, **i32)
        self.tok = torch.zeros(n, **i32)
        self.pos = torch.zeros(n, **i32)
        self.step = torch.zeros(n, **i32)
        self.n_commit = torch.zeros(B, **i32)
        self.done = torch.zeros(B, **i32)
        self.committed = torch.zeros((B, max_new_tokens), **i32)
        self.seq_ct = torch.zeros((B, 8), **i32)
        self.emu_len = max_new_tokens * (cfg.T_total + 4) + 100
        self.emu = torch.zeros((B, self.emu_len), dtype=torch.uint8, device=dev)
        self.emu_ctr = torch.zeros(B, **i32)
        self.batch_ct = torch.zeros(8, **i32)
        self.keys = torch.zeros(3, dtype=torch.int64, device=dev)
        self.c_slot = torch.full((2 * B,), -1, **i32)
        # union tables: P one row per sequence, C two, R the live tokens (a
        # capacity independent of T_draft in batch-invariant mode)
        self.r_cap = B * ((cfg.T_total if batch_invariant else cfg.T_total // policy.T_draft) + 2)
        self.tp = _Tables("P", B, 6 + cfg.n_prelude, dev)
        self.tr = _Tables("R", self.r_cap, 6, dev)
        self.tc = _Tables("C", 2 * B, 6 + cfg.n_coda, dev)
        self._params = {}
        self._graphs: dict[bool, torch.cuda.CUDAGraph] = {}
        self.ticks_replayed = 0
        self.kv_read_bytes = 0
        self.d2h_bytes = 0      # device -> host bytes of the last generate

    # ------------------------------------------------------------------
    def _p(self, use_emu: bool) -> "_abi.wfd_sched_params":
        key = bool(use_emu)
        if key in self._params:
            return self._params[key]
        e, cfg = self.eng, self.eng.cfg
        p = _abi.wfd_sched_params()
        for name in ("alive", "state", "tok", "pos", "step", "n_commit", "done", "committed", "seq_ct", "emu_ctr",
                     "batch_ct", "keys", "c_slot"):
            setattr(p, name, getattr(self, name).data_ptr())
        p.emu = self.emu.data_ptr() if use_emu else None
        p.lens = e.cache.lens.data_ptr()
        p.err = rt.error_word(self.device).data_ptr()
        p.p_tab, p.r_tab, p.c_tab = self.tp.dev.data_ptr(), self.tr.dev.data_ptr(), self.tc.dev.data_ptr()
        p.c_out = self.tc.out.data_ptr()
        p.B, p.W, p.T_total, p.T_draft = self.B, self.W, cfg.T_total, self.policy.T_draft
        p.max_new, p.emu_len = self.max_new, self.emu_len
        p.n_core, p.n_kv_slots, p.lens_stride, p.max_seq = cfg.n_core, cfg.n_slots, e.B + 1, e.S
        p.p_cols, p.c_cols, p.r_cap = self.tp.n_cols, self.tc.n_cols, self.r_cap
        p.scratch_row, p.scratch_seq = e.scratch_row, e.scratch_seq
        p.p_slot0, p.n_prelude = cfg.slot_prelude(0), cfg.n_prelude
        p.c_slot0, p.n_coda = cfg.slot_coda(0), cfg.n_coda
        p.depth_slots = cfg.n_depth_slots
        p.gap_windows = 1 if self.eng.gap_windows else 0
        self._params[key] = p
        return p

    def _launch(self, name: str, p) -> None:
        st = getattr(_abi.load(), name)(ctypes.addressof(p), rt.stream_ptr(self.device))
        _abi.check(st, name)

    def _tick(self, p) -> None:
        e = self.eng
        self._launch("wfd_sched_pre_tick", p)
        e._body("P", self.tp)
        e._body("R", self.tr)
        self._launch("wfd_sched_route", p)
        e._body("C", self.tc)
        self._launch("wfd_sched_settle", p)

    def _capture(self, p) -> torch.cuda.CUDAGraph:
        # warm up on an all-finished state (every row padding, nothing changes),
        # then capture; the real state is loaded afterwards (pointers are fixed)
        with rt.batch_invariant(self.batch_invariant):
            return self._capture_graph(p)

    def _capture_graph(self, p) -> torch.cuda.CUDAGraph:
        self.done.fill_(1)
        cur = torch.cuda.current_stream(self.device)
        side = torch.cuda.Stream(self.device)
        side.wait_stream(cur)
        with torch.cuda.stream(side):
            for _ in range(2):
                self._tick(p)
        cur.wait_stream(side)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self._tick(p)
        return g

    # ------------------------------------------------------------------
    @torch.no_grad()
    def generate(self, prompt_ids: torch.Tensor, emus=None, use_graph: bool = True) -> BatchTrace:
        e, B = self.eng, self.B
        bt = BatchTrace()
        t0 = time.perf_counter()
        _, last_logits = e.prefill(prompt_ids)
        first = [int(x) for x in last_logits.argmax(dim=-1).tolist()]
        torch.cuda.synchronize(self.device)
        bt.prefill_s = time.perf_counter() - t0
        L = int(prompt_ids.shape[1])
        use_emu = emus is not None
        p = self._p(use_emu)
        if use_graph and use_emu not in self._graphs:
            self._graphs[use_emu] = self._capture(p)
        # initial state: first token committed, queued for the prelude at position L
        W = self.W
        alive = torch.zeros(B * W, dtype=torch.int32)
        state = torch.zeros(B * W, dtype=torch.int32)
        tok = torch.zeros(B * W, dtype=torch.int32)
        pos = torch.zeros(B * W, dtype=torch.int32)
        n_commit = torch.ones(B, dtype=torch.int32)
        done = torch.zeros(B, dtype=torch.int32)
        committed = torch.zeros((B, self.max_new), dtype=torch.int32)
        seq_ct = torch.zeros((B, 8), dtype=torch.int32)
        for b in range(B):
            committed[b, 0] = first[b]
            if self.max_new <= 1:
                done[b] = 1
                continue
            alive[b * W], state[b * W], tok[b * W], pos[b * W] = 1, 1, first[b], L
            seq_ct[b, 0] = 1
        for name, t in (("alive", alive), ("state", state), ("tok", tok), ("pos", pos), ("n_commit", n_commit),
                        ("done", done), ("committed", committed), ("seq_ct", seq_ct)):
            getattr(self, name).copy_(t)
        self.step.zero_()
        self.emu_ctr.zero_()
        self.batch_ct.zero_()
        self.keys.zero_()
        if use_emu:
            draws = torch.zeros((B, self.emu_len), dtype=torch.uint8)
            for b, em in enumerate(emus):
                em = copy.deepcopy(em)
                draws[b] = torch.tensor([1 if em.draw() else 0 for _ in range(self.emu_len)], dtype=torch.uint8)
            self.emu.copy_(draws)
        graph = self._graphs[use_emu] if use_graph else None

        guard = self.max_new * (e.cfg.T_total + 4) + 100
        ticks = 0
        d2h = 8 * B                       # first-token ids
        while True:
            nc = self.n_commit.tolist()
            dn = self.done.tolist()
            d2h += 8 * B
            remaining = [self.max_new - c for c, d in zip(nc, dn) if not d]
            if not remaining:
                break
            k = max(1, min(max(remaining), guard - ticks))
            if ticks >= guard:
                raise RuntimeError(f"device wavefront exceeded the tick guard ({guard})")
            with rt.batch_invariant(self.batch_invariant):
                for _ in range(k):
                    if graph is not None:
                        graph.replay()
                    else:
                        self._tick(p)
            ticks += k
        torch.cuda.synchronize(self.device)
        rt.read_device_error(self.device)
        bt.walltime_s = time.perf_counter() - t0
        self.ticks_replayed = ticks

        committed = self.committed.cpu()
        seq_ct = self.seq_ct.cpu()
        n_commit = self.n_commit.cpu()
        bc = self.batch_ct.tolist()
        bt.n_r_calls, bt.n_p_calls, bt.n_c_calls = bc[0], bc[1], bc[2]
        bt.r_union_total, bt.r_union_max = bc[3], bc[4]
        for b in range(B):
            tr = GenerationTrace()
            tr.tokens = committed[b, :min(int(n_commit[b]), self.max_new)].tolist()
            for i, name in enumerate(_CT):
                setattr(tr, name, int(seq_ct[b, i]))
            tr.walltime_s = bt.walltime_s
            bt.per_seq.append(tr)
        keys = self.keys.tolist()
        d2h += 4 * (B * self.max_new + 8 * B + B + 8) + 8 * 3 + 4
        self.d2h_bytes = d2h
        cfg = e.cfg
        self.kv_read_bytes = 2 * e._row_bytes * (keys[0] * cfg.n_prelude + keys[1] * cfg.n_core + keys[2] * cfg.n_coda)
        return bt


def generate_wavefront_device(engine: WaveEngine, prompt_ids: torch.Tensor, max_new_tokens: int, policy: SsdPolicy,
                              emus=None, *, use_graph: bool = True, batch_invariant: bool = False) -> BatchTrace:
    """scheduler.generate_wavefront_batch with route / settle on the device."""
    return DeviceWave(engine, max_new_tokens, policy, batch_invariant).generate(prompt_ids, emus, use_graph=use_graph)

