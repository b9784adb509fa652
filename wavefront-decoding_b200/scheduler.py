"""Fixed-batch wavefront (WFD) and autoregressive schedulers over union P/R/C calls.

Mirrors the reference's `src/decoding/scheduler_batch.py` (`generate_wavefront_batch`
:228-362, `ar_generate_batch` :185-222), `batch_state.SeqState` (:272-323),
`emu.EmulatedAcceptance` (:19-43) and `policy.SsdPolicy` (:16-59): same names,
arguments, decisions and counters, so a trace from either implementation can be
compared field by field.  The decision logic stays on the host (one token-id
read-back per tick, as in the reference, `scheduler_batch.py:312`); every tensor
operation runs in the `blocks` object (the GPU engine, engine.WaveEngine).

Per tick: P union (tokens queued for the prelude) -> R union (one loop step for
every live wave token) -> route (commit point: step == T_total -> verify; draft
point: step == T_draft -> copy for a draft C) -> C union (greedy ids) -> settle
(accept / reject cascade / rollback per sequence, new leading-edge draft).

`generate_dtv_batch` is the reference's draft-then-verify scheduler
(scheduler_batch.py:365-501): per sequence, rounds of K drafts at depth T_draft
followed by one verify of all K + 1 sources at full depth.
"""
from __future__ import annotations

import copy
import random
import time
import warnings
from dataclasses import dataclass, field
from typing import Optional


# ---------------------------------------------------------------------------
# policy / emulated acceptance (policy.py:16-59, emu.py:19-43)
# ---------------------------------------------------------------------------
@dataclass
class SsdPolicy:
    T_total: int = 8
    T_draft: int = 2
    mode: str = "greedy"

    def __post_init__(self) -> None:
        if self.T_draft < 1 or self.T_total < self.T_draft:
            raise ValueError(f"Invalid policy: T_total={self.T_total}, T_draft={self.T_draft}. "
                             "Require 1 <= T_draft <= T_total.")
        if self.mode != "greedy":
            raise ValueError(f"Unknown sampling mode: {self.mode!r} (this engine decodes greedily).")
        if self.T_total % self.T_draft != 0:
            warnings.warn(f"T_total ({self.T_total}) is not a multiple of T_draft ({self.T_draft}); "
                          "active wave size will fluctuate.", stacklevel=2)

    @property
    def steady_state_active_size(self) -> int:
        return self.T_total // self.T_draft


class EmulatedAcceptance:
    """Bernoulli(rate) accept stream, one per sequence (seed = base + index)."""

    def __init__(self, rate: float, seed: int = 0):
        assert 0.0 <= rate <= 1.0, f"acceptance rate must be in [0,1], got {rate}"
        self.rate = float(rate)
        self.seed = seed
        self.rng = random.Random(seed)
        self.n_draws = 0
        self.n_accepts = 0

    def draw(self) -> bool:
        self.n_draws += 1
        ok = self.rng.random() < self.rate
        self.n_accepts += int(ok)
        return ok

    @property
    def empirical_rate(self) -> float:
        return self.n_accepts / self.n_draws if self.n_draws else float("nan")


# ---------------------------------------------------------------------------
# state (state.py:20-65, batch_state.py:272-323)
# ---------------------------------------------------------------------------
@dataclass
class ActiveToken:
    """One token in flight.  `hidden` is an opaque handle the blocks own (a
    row of a device-resident state pool in the GPU engine)."""
    token_id: int
    position: int
    role: str
    step: int = 0
    hidden: object = None
    static_state: object = None
    is_alive: bool = True


@dataclass
class GenerationTrace:
    tokens: list = field(default_factory=list)
    walltime_s: float = 0.0
    n_r_calls: int = 0
    n_p_calls: int = 0
    n_c_calls: int = 0
    n_drafts_proposed: int = 0
    n_drafts_accepted: int = 0
    n_drafts_rejected: int = 0
    n_rollback_events: int = 0

    @property
    def acceptance_rate(self) -> float:
        return self.n_drafts_accepted / self.n_drafts_proposed if self.n_drafts_proposed else float("nan")


@dataclass
class SeqState:
    idx: int
    prefix_len: int
    emu: Optional[EmulatedAcceptance] = None
    trace: GenerationTrace = field(default_factory=GenerationTrace)
    committed: list = field(default_factory=list)
    done: bool = False
    active_p: list = field(default_factory=list)
    active_r: list = field(default_factory=list)
    active_c: list = field(default_factory=list)
    # DtV round state (batch_state.py:38-49): phase "need_p" (the next source needs
    # its prelude), "draft" (the current source runs steps 0..T_draft), "verify"
    # (all K + 1 sources run T_draft..T_total), "idle" once done
    phase: str = "need_p"
    K: int = 0                 # drafts this round
    j: int = 0                 # index of the current source (0..K)
    sources: list = field(default_factory=list)
    drafts: list = field(default_factory=list)
    cur_tok: int = 0           # token forwarded as source j, and its position
    cur_pos: int = 0
    last_token: int = 0        # last committed token (the round's seed), and its position
    p: int = 0

    def commit(self, token_id: int) -> None:
        self.committed.append(token_id)
        self.trace.tokens.append(token_id)

    def find_active(self, position: int) -> Optional[ActiveToken]:
        for lst in (self.active_r, self.active_p, self.active_c):
            for t in lst:
                if t.is_alive and t.position == position:
                    return t
        return None

    def rollback(self, position: int, cache) -> None:
        self.active_p = [t for t in self.active_p if t.position < position]
        self.active_r = [t for t in self.active_r if t.position < position]
        self.active_c = [t for t in self.active_c if t.position < position]
        cache.drop_positions_at_and_after(self.idx, position)

    def clear_working_state(self) -> None:
        self.active_p, self.active_r, self.active_c = [], [], []
        self.sources, self.drafts = [], []
        self.phase = "idle"


@dataclass
class BatchTrace:
    walltime_s: float = 0.0
    prefill_s: float = 0.0
    n_r_calls: int = 0
    n_p_calls: int = 0
    n_c_calls: int = 0
    r_union_total: int = 0
    r_union_max: int = 0
    per_seq: list = field(default_factory=list)

    @property
    def n_tokens(self) -> int:
        return sum(len(t.tokens) for t in self.per_seq)

    @property
    def tokens_per_s(self) -> float:
        return self.n_tokens / self.walltime_s if self.walltime_s > 0 else float("nan")

    @property
    def walltime_decode_s(self) -> float:
        return max(self.walltime_s - self.prefill_s, 0.0)

    @property
    def r_union_mean(self) -> float:
        return self.r_union_total / self.n_r_calls if self.n_r_calls else 0.0

    @property
    def acceptance_rate(self) -> float:
        prop = sum(t.n_drafts_proposed for t in self.per_seq)
        acc = sum(t.n_drafts_accepted for t in self.per_seq)
        return acc / prop if prop else float("nan")


def _record_r(bt: BatchTrace, n_union: int) -> None:
    bt.n_r_calls += 1
    bt.r_union_total += n_union
    bt.r_union_max = max(bt.r_union_max, n_union)


def _sync(blocks) -> None:
    fn = getattr(blocks, "synchronize", None)
    if fn is not None:
        fn()


def _prefill_and_first(blocks, prompt_ids, emus, max_new_tokens, bt: BatchTrace, t0: float):
    """scheduler_batch.py:123-159: prefill, commit the greedy first token."""
    cache, last_logits = blocks.prefill(prompt_ids)
    first = [int(x) for x in last_logits.argmax(dim=-1).tolist()]
    _sync(blocks)
    bt.prefill_s = time.perf_counter() - t0
    L = int(prompt_ids.shape[1])
    seqs = []
    for b in range(int(prompt_ids.shape[0])):
        s = SeqState(idx=b, prefix_len=L, emu=(emus[b] if emus is not None else None))
        s.commit(first[b])
        if len(s.committed) >= max_new_tokens:
            s.done = True
        seqs.append(s)
    return cache, seqs


def _finalize(bt: BatchTrace, seqs, t0: float, blocks) -> BatchTrace:
    _sync(blocks)
    bt.walltime_s = time.perf_counter() - t0
    for s in seqs:
        s.trace.walltime_s = bt.walltime_s
    bt.per_seq = [s.trace for s in seqs]
    return bt


def ar_generate_batch(blocks, prompt_ids, max_new_tokens: int) -> BatchTrace:
    """Lockstep batched sequential loop decoding (scheduler_batch.py:185-222):
    every live sequence runs P, T_total R steps and C per committed token."""
    bt = BatchTrace()
    t0 = time.perf_counter()
    cache, seqs = _prefill_and_first(blocks, prompt_ids, None, max_new_tokens, bt, t0)
    T_total = blocks.T_total
    while True:
        act = [s for s in seqs if not s.done]
        if not act:
            break
        toks = []
        for s in act:
            pos = s.prefix_len + len(s.committed) - 1
            toks.append(ActiveToken(token_id=s.committed[-1], position=pos, role="verify"))
            s.trace.n_p_calls += 1
        seq_ids = [s.idx for s in act]
        blocks.prelude_union(seq_ids, toks, cache)
        bt.n_p_calls += 1
        for _ in range(T_total):
            blocks.advance_union(seq_ids, toks, cache)
            _record_r(bt, len(toks))
            for s in act:
                s.trace.n_r_calls += 1
        out_ids = blocks.coda_argmax_union(seq_ids, toks, cache)
        bt.n_c_calls += 1
        for s, nid in zip(act, out_ids):
            s.trace.n_c_calls += 1
            s.commit(int(nid))
            if len(s.committed) >= max_new_tokens:
                s.done = True
    return _finalize(bt, seqs, t0, blocks)


def generate_wavefront_batch(blocks, prompt_ids, max_new_tokens: int, policy: SsdPolicy,
                             emus: list | None = None) -> BatchTrace:
    """One independent wave per sequence, union P/R/C per tick
    (scheduler_batch.py:228-362).  emus[b] = EmulatedAcceptance replaces the
    gold == draft comparison of sequence b (None: real comparison)."""
    bt = BatchTrace()
    t0 = time.perf_counter()
    cache, seqs = _prefill_and_first(blocks, prompt_ids, emus, max_new_tokens, bt, t0)
    T_total, T_draft = policy.T_total, policy.T_draft
    if emus is None:
        emus = [None] * len(seqs)

    for s in seqs:
        if s.done:
            continue
        s.active_p.append(ActiveToken(token_id=s.committed[-1], position=s.prefix_len, role="draft"))
        s.trace.n_p_calls += 1

    ticks, max_ticks = 0, max_new_tokens * (T_total + 4) + 100
    while True:
        alive = [s for s in seqs if not s.done]
        if not alive:
            break
        ticks += 1
        if ticks > max_ticks:
            raise RuntimeError(f"wfd batch exceeded tick guard ({max_ticks}) — scheduler bug?")

        # ---- P: union of queued tokens
        p_pairs = [(s, t) for s in alive for t in s.active_p]
        if p_pairs:
            blocks.prelude_union([s.idx for s, _ in p_pairs], [t for _, t in p_pairs], cache)
            for s, t in p_pairs:
                s.active_r.append(t)
            for s in alive:
                s.active_p = []
            bt.n_p_calls += 1

        # ---- R: one loop step for every live wave token
        r_pairs = [(s, t) for s in alive for t in s.active_r if t.is_alive]
        if r_pairs:
            blocks.advance_union([s.idx for s, _ in r_pairs], [t for _, t in r_pairs], cache)
            _record_r(bt, len(r_pairs))
            for s in alive:
                if any(t.is_alive for t in s.active_r):
                    s.trace.n_r_calls += 1

        # ---- route commit / draft points
        for s in alive:
            survivors = []
            for t in s.active_r:
                if not t.is_alive:
                    continue
                if t.step == T_total:
                    t.role = "verify"
                    s.active_c.append(t)
                else:
                    survivors.append(t)
                    if t.step == T_draft:
                        c = copy.copy(t)
                        c.role = "draft"
                        s.active_c.append(c)
            s.active_r = survivors

        # ---- C: one head pass over the union of active_c
        c_meta, c_toks, c_seq_ids = [], [], []
        for s in alive:
            if not s.active_c:
                continue
            vs = sorted((t for t in s.active_c if t.role == "verify"), key=lambda t: t.position)
            ds = [t for t in s.active_c if t.role == "draft"]
            c_meta.append((s, vs, ds))
            c_toks += vs + ds
            c_seq_ids += [s.idx] * (len(vs) + len(ds))
        gold_of = {}
        if c_toks:
            out_ids = blocks.coda_argmax_union(c_seq_ids, c_toks, cache)
            bt.n_c_calls += 1
            gold_of = {id(t): int(nid) for t, nid in zip(c_toks, out_ids)}
            for s, _, _ in c_meta:
                s.trace.n_c_calls += 1

        # ---- settle per sequence + new leading-edge draft
        for s, vs, ds in c_meta:
            rejected = False
            boundary = False
            for i, vtok in enumerate(vs):
                gold = gold_of[id(vtok)]
                vtok.is_alive = False
                next_pos = vtok.position + 1
                nxt = vs[i + 1] if i + 1 < len(vs) else s.find_active(next_pos)
                if nxt is None:
                    s.commit(gold)
                    s.active_p.append(ActiveToken(gold, next_pos, "draft"))
                    s.trace.n_p_calls += 1
                    boundary = True
                else:
                    accept = s.emu.draw() if s.emu is not None else (gold == nxt.token_id)
                    s.trace.n_drafts_proposed += 1
                    if accept:
                        s.trace.n_drafts_accepted += 1
                        s.commit(nxt.token_id)
                    else:
                        s.trace.n_drafts_rejected += 1
                        s.trace.n_rollback_events += 1
                        rejected = True
                        s.commit(gold)
                        s.rollback(next_pos, cache)
                        s.active_p.append(ActiveToken(gold, next_pos, "draft"))
                        s.trace.n_p_calls += 1
                if len(s.committed) >= max_new_tokens:
                    s.done = True
                if s.done or rejected or boundary:
                    break
            if s.done:
                s.clear_working_state()
                continue
            if not rejected and ds:
                dsrc = ds[0]
                s.active_p.append(ActiveToken(gold_of[id(dsrc)], dsrc.position + 1, "draft"))
                s.trace.n_p_calls += 1
            s.active_c = []

    return _finalize(bt, seqs, t0, blocks)


# ---------------------------------------------------------------------------
# draft-then-verify (scheduler_batch.py:365-501)
# ---------------------------------------------------------------------------
def _dtv_new_round(s: SeqState, max_new_tokens: int, draft_length: int) -> None:
    """scheduler_batch.py:368-376: K = min(draft_length, tokens still to commit)
    drafts, seeded by the last committed token."""
    s.K = min(draft_length, max_new_tokens - len(s.committed))
    s.j = 0
    s.sources, s.drafts = [], []
    s.cur_tok, s.cur_pos = s.last_token, s.p
    s.phase = "need_p"


def generate_dtv_batch(blocks, prompt_ids, max_new_tokens: int, policy: SsdPolicy, draft_length: int,
                       emus: list | None = None) -> BatchTrace:
    """Draft-then-verify over union P / R / C calls (scheduler_batch.py:378-501).

    Each sequence runs rounds: source 0 is the last committed token; each source
    goes through the prelude and T_draft loop steps, and its draft-depth greedy id
    is the next source (draft d_{j+1}), K drafts per round.  Then all K + 1
    sources advance together from T_draft to T_total (one window per sequence:
    consecutive positions on one depth slot) and the full-depth ids verify the
    drafts: accept while equal (emus[b] replaces the comparison), commit the
    first gold on a reject and drop the cache from there, or commit the bonus
    token when all K are accepted."""
    bt = BatchTrace()
    t0 = time.perf_counter()
    cache, seqs = _prefill_and_first(blocks, prompt_ids, emus, max_new_tokens, bt, t0)
    T_total, T_draft = policy.T_total, policy.T_draft
    rows = getattr(blocks, "ensure_window_rows", None)
    if rows is not None:
        rows(draft_length + 1)   # the verify union attends K + 1 sources of a sequence as one window
    for s in seqs:
        if not s.done:
            s.last_token, s.p = s.committed[-1], s.prefix_len
            _dtv_new_round(s, max_new_tokens, draft_length)

    ticks, max_ticks = 0, max_new_tokens * ((draft_length + 1) * max(T_draft, 1) + T_total + 4) + 100
    while True:
        alive = [s for s in seqs if not s.done]
        if not alive:
            break
        ticks += 1
        if ticks > max_ticks:
            raise RuntimeError(f"dtv batch exceeded the tick guard ({max_ticks})")

        # P: sequences whose next source needs its prelude
        need = [s for s in alive if s.phase == "need_p"]
        if need:
            toks = []
            for s in need:
                t = ActiveToken(token_id=s.cur_tok, position=s.cur_pos, role="verify")
                s.sources.append(t)
                s.trace.n_p_calls += 1
                s.phase = "draft"
                toks.append(t)
            blocks.prelude_union([s.idx for s in need], toks, cache)
            bt.n_p_calls += 1

        # R: a drafting sequence advances its current source, a verifying one all
        # of its sources (until they reach full depth)
        pairs, took = [], []
        for s in alive:
            if s.phase == "draft":
                pairs.append((s, s.sources[-1]))
                took.append(s)
            elif s.phase == "verify" and s.sources[0].step < T_total:
                pairs += [(s, t) for t in s.sources]
                took.append(s)
        if pairs:
            blocks.advance_union([s.idx for s, _ in pairs], [t for _, t in pairs], cache)
            _record_r(bt, len(pairs))
            for s in took:
                s.trace.n_r_calls += 1

        # C: a draft (the current source reached T_draft) or the verify (all
        # sources reached T_total)
        entries = []
        for s in alive:
            if s.phase == "draft" and s.sources[-1].step == T_draft:
                entries.append((s, "draft", [s.sources[-1]]))
            elif s.phase == "verify" and s.sources[0].step == T_total:
                entries.append((s, "verify", list(s.sources)))
        if not entries:
            continue
        flat = [t for _, _, ts in entries for t in ts]
        ids = blocks.coda_argmax_union([s.idx for s, _, ts in entries for _ in ts], flat, cache)
        bt.n_c_calls += 1
        k = 0
        for s, kind, ts in entries:
            out = [int(x) for x in ids[k:k + len(ts)]]
            k += len(ts)
            s.trace.n_c_calls += 1
            if kind == "draft":
                if s.j < s.K:
                    s.drafts.append(out[0])          # d_{j+1}, at cur_pos + 1
                s.cur_tok, s.cur_pos = out[0], s.cur_pos + 1
                s.j += 1
                s.phase = "need_p" if s.j <= s.K else "verify"
                continue
            # verify: source p + i predicts position p + i + 1
            rejected = False
            for i in range(s.K):
                s.trace.n_drafts_proposed += 1
                accept = s.emu.draw() if s.emu is not None else out[i] == s.drafts[i]
                if accept:
                    s.trace.n_drafts_accepted += 1
                    s.commit(s.drafts[i])
                    if len(s.committed) >= max_new_tokens:
                        s.done = True
                        break
                else:
                    s.trace.n_drafts_rejected += 1
                    s.trace.n_rollback_events += 1
                    rejected = True
                    s.commit(out[i])
                    cache.drop_positions_at_and_after(s.idx, s.p + i + 1)
                    s.last_token, s.p = out[i], s.p + i + 1
                    if len(s.committed) >= max_new_tokens:
                        s.done = True
                    break
            if not rejected and not s.done:
                s.commit(out[s.K])                   # every draft accepted: the bonus token
                s.last_token, s.p = out[s.K], s.p + s.K + 1
                if len(s.committed) >= max_new_tokens:
                    s.done = True
            if s.done:
                s.clear_working_state()
            else:
                _dtv_new_round(s, max_new_tokens, draft_length)
    return _finalize(bt, seqs, t0, blocks)

