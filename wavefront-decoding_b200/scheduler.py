"""Host-side batch schedulers over the engine's union P / R / C calls.

A *lane* is one sequence of the batch.  Its *wave* holds the tokens that are in
the recurrent block, keyed by absolute position; a token that enters the wave
at step 0 advances one loop step per tick and is read out by the coda twice:
at depth T_draft (its greedy id drafts the next position, which then enters
the wave right behind it) and at depth T_total (its greedy id is the gold for
the next position, which confirms or refutes the draft in flight there).  This
is the state the device scheduler keeps in fixed token slots
(csrc/wfd_sched.cuh); here it is a dict per lane, and a tick is

    prelude  the lane's queued tokens enter the wave        (one P union)
    advance  every token in flight takes one loop step      (one R union)
    read     tokens at full depth leave the wave; tokens at
             draft depth are read as drafts                 (one C union)
    settle   per lane, in position order: confirm the next draft or commit
             the gold and cut the wave there (the KV slots of the sequence
             drop the positions from the cut on); queue the next token

Behaviour follows the reference's batch schedulers
(src/decoding/scheduler_batch.py: ar_generate_batch :185-222,
generate_wavefront_batch :228-362, generate_dtv_batch :365-501): the same
decisions in the same order, the same counters, the same union sizes, the same
rollback calls and, under emulated acceptance, the same order of draws from
each sequence's random.Random stream (emu.py:19-43), so the reference's own
traces pin this module (tests/golden/reference_scheduler.json).  The engine
(engine.WaveEngine) does every tensor operation; the host reads back one
vector of greedy ids per tick.
"""
from __future__ import annotations

import random
import time
import warnings
from dataclasses import dataclass, field
from typing import Optional


# ---------------------------------------------------------------------------
# depths and emulated acceptance
# ---------------------------------------------------------------------------
@dataclass(frozen=True)
class SsdPolicy:
    """Wave depths (reference policy.py:16-59): a token is read as a draft at
    loop step T_draft and verified at step T_total.  Greedy decoding only."""
    T_total: int = 8
    T_draft: int = 2
    mode: str = "greedy"

    def __post_init__(self) -> None:
        if not 1 <= self.T_draft <= self.T_total:
            raise ValueError(f"SsdPolicy needs 1 <= T_draft <= T_total; got T_draft={self.T_draft}, "
                             f"T_total={self.T_total}")
        if self.mode != "greedy":
            raise ValueError(f"SsdPolicy: only greedy decoding is built (mode={self.mode!r})")
        if self.T_total % self.T_draft:
            warnings.warn(f"T_draft={self.T_draft} does not divide T_total={self.T_total}: the number of tokens "
                          "in flight per sequence will vary from tick to tick", stacklevel=2)

    @property
    def steady_state_active_size(self) -> int:
        """Tokens in flight per sequence once the wave is full."""
        return self.T_total // self.T_draft


class EmulatedAcceptance:
    """Draft outcomes drawn instead of compared (reference emu.py:19-43): each
    draw accepts with probability `rate`, from a random.Random(seed) stream of
    its own per sequence; one draw per verified draft, in commit order."""

    def __init__(self, rate: float, seed: int = 0):
        if not 0.0 <= rate <= 1.0:
            raise ValueError(f"EmulatedAcceptance: rate {rate} is not a probability")
        self.rate = float(rate)
        self.seed = seed
        self._stream = random.Random(seed)
        self.n_draws = 0
        self.n_accepts = 0

    def draw(self) -> bool:
        ok = self._stream.random() < self.rate
        self.n_draws += 1
        self.n_accepts += ok
        return ok

    @property
    def empirical_rate(self) -> float:
        return self.n_accepts / self.n_draws if self.n_draws else float("nan")


# ---------------------------------------------------------------------------
# traces (the reference's counter names: they are compared field by field)
# ---------------------------------------------------------------------------
@dataclass
class GenerationTrace:
    """Per-sequence record: committed tokens and the counters of the reference's
    state.GenerationTrace."""
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
class BatchTrace:
    """Batch record: union-call counts, R-union sizes and the per-sequence traces."""
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
        return sum(t.n_drafts_accepted for t in self.per_seq) / prop if prop else float("nan")

    def count_union(self, kind: str, rows: int = 0) -> None:
        if kind == "P":
            self.n_p_calls += 1
        elif kind == "C":
            self.n_c_calls += 1
        else:
            self.n_r_calls += 1
            self.r_union_total += rows
            self.r_union_max = max(self.r_union_max, rows)


# ---------------------------------------------------------------------------
# lanes
# ---------------------------------------------------------------------------
class Flight:
    """One token in flight: what the engine's union calls read and update
    (`hidden` / `static_state`: the engine's handle of its state rows; `step`:
    loop steps taken)."""
    __slots__ = ("token_id", "position", "step", "hidden", "static_state")

    def __init__(self, token_id: int, position: int):
        self.token_id = int(token_id)
        self.position = int(position)
        self.step = 0
        self.hidden = None
        self.static_state = None


class _Lane:
    def __init__(self, idx: int, prompt_len: int, acceptance: Optional[EmulatedAcceptance]):
        self.idx = idx
        self.prompt_len = prompt_len
        self.acceptance = acceptance
        self.trace = GenerationTrace()
        self.finished = False
        self.wave: dict[int, Flight] = {}   # position -> token in the recurrent block (ascending positions)
        self.queue: list[Flight] = []       # tokens waiting for the prelude
        # draft-then-verify round (generate_dtv_batch)
        self.anchor_tok = 0                 # last committed token and its position: the next round's seed
        self.anchor_pos = 0
        self.round: Optional[_DtvRound] = None

    @property
    def n_committed(self) -> int:
        return len(self.trace.tokens)

    def emit(self, token_id: int, limit: int) -> None:
        self.trace.tokens.append(int(token_id))
        if self.n_committed >= limit:
            self.finished = True

    def enqueue(self, token_id: int, position: int) -> None:
        self.queue.append(Flight(token_id, position))
        self.trace.n_p_calls += 1

    def cut(self, position: int, cache) -> None:
        """Forget every token at or after `position` and drop those positions
        from the sequence's KV slots (BatchStaticKVCache.drop_positions_at_and_after)."""
        self.wave = {p: f for p, f in self.wave.items() if p < position}
        self.queue = [f for f in self.queue if f.position < position]
        cache.drop_positions_at_and_after(self.idx, position)

    def retire(self) -> None:
        self.wave, self.queue, self.round = {}, [], None


def _start(blocks, prompt_ids, emus, max_new_tokens: int, bt: BatchTrace, t0: float):
    """Prefill every prompt and commit each sequence's first greedy token
    (scheduler_batch.py:123-159)."""
    cache, logits = blocks.prefill(prompt_ids)
    first = logits.argmax(dim=-1).tolist()
    _synchronize(blocks)
    bt.prefill_s = time.perf_counter() - t0
    L = int(prompt_ids.shape[1])
    lanes = [_Lane(b, L, emus[b] if emus is not None else None) for b in range(int(prompt_ids.shape[0]))]
    for lane, tok in zip(lanes, first):
        lane.emit(tok, max_new_tokens)
    return cache, lanes


def _synchronize(blocks) -> None:
    sync = getattr(blocks, "synchronize", None)
    if sync is not None:
        sync()


def _close(bt: BatchTrace, lanes, t0: float, blocks) -> BatchTrace:
    _synchronize(blocks)
    bt.walltime_s = time.perf_counter() - t0
    for lane in lanes:
        lane.trace.walltime_s = bt.walltime_s
    bt.per_seq = [lane.trace for lane in lanes]
    return bt


def _tick_bound(max_new_tokens: int, per_token: int) -> int:
    """Ticks after which a run that has not finished is a scheduler fault: every
    tick commits a token of some live sequence within `per_token` ticks."""
    return (max_new_tokens + 2) * (per_token + 4) + 128


def _advance(blocks, cache, bt: BatchTrace, entries) -> None:
    """One R union over (lane, token) entries; counts the call per lane once."""
    blocks.advance_union([lane.idx for lane, _ in entries], [f for _, f in entries], cache)
    bt.count_union("R", len(entries))
    seen = set()
    for lane, _ in entries:
        if lane.idx not in seen:
            seen.add(lane.idx)
            lane.trace.n_r_calls += 1


# ---------------------------------------------------------------------------
# sequential loop decoding
# ---------------------------------------------------------------------------
def ar_generate_batch(blocks, prompt_ids, max_new_tokens: int) -> BatchTrace:
    """Batched sequential loop decoding (scheduler_batch.py:185-222): per
    committed token, every live sequence runs the prelude, T_total loop steps
    and the coda in lockstep."""
    bt = BatchTrace()
    t0 = time.perf_counter()
    cache, lanes = _start(blocks, prompt_ids, None, max_new_tokens, bt, t0)
    depth = blocks.T_total
    while True:
        live = [lane for lane in lanes if not lane.finished]
        if not live:
            break
        batch = []
        for lane in live:
            lane.trace.n_p_calls += 1
            batch.append((lane, Flight(lane.trace.tokens[-1], lane.prompt_len + lane.n_committed - 1)))
        ids = [lane.idx for lane, _ in batch]
        toks = [f for _, f in batch]
        blocks.prelude_union(ids, toks, cache)
        bt.count_union("P")
        for _ in range(depth):
            _advance(blocks, cache, bt, batch)
        heads = blocks.coda_argmax_union(ids, toks, cache)
        bt.count_union("C")
        for (lane, _), tok in zip(batch, heads):
            lane.trace.n_c_calls += 1
            lane.emit(tok, max_new_tokens)
    return _close(bt, lanes, t0, blocks)


# ---------------------------------------------------------------------------
# wavefront decoding
# ---------------------------------------------------------------------------
def _wave_settle(lane: _Lane, full, gold, drafts, draft_ids, cache, limit: int) -> None:
    """Resolve one lane's read-outs of a tick.  `full`: tokens that reached
    T_total (ascending positions) with their gold ids; `drafts`: tokens read at
    T_draft with their greedy ids."""
    trace = lane.trace
    cut = False
    for k, (tok, g) in enumerate(zip(full, gold)):
        nxt = tok.position + 1
        following = full[k + 1] if k + 1 < len(full) else lane.wave.get(nxt)
        if following is None:
            # nothing in flight behind it: the gold is committed and starts the wave again
            lane.emit(g, limit)
            lane.enqueue(g, nxt)
            stop = True
        else:
            trace.n_drafts_proposed += 1
            agree = lane.acceptance.draw() if lane.acceptance is not None else g == following.token_id
            if agree:
                trace.n_drafts_accepted += 1
                lane.emit(following.token_id, limit)
                stop = False
            else:
                trace.n_drafts_rejected += 1
                trace.n_rollback_events += 1
                lane.emit(g, limit)
                lane.cut(nxt, cache)
                lane.enqueue(g, nxt)
                cut = stop = True
        if lane.finished or stop:
            break
    if lane.finished:
        lane.retire()
        return
    if not cut and drafts:
        lane.enqueue(draft_ids[0], drafts[0].position + 1)


def generate_wavefront_batch(blocks, prompt_ids, max_new_tokens: int, policy: SsdPolicy,
                             emus: list | None = None) -> BatchTrace:
    """Wavefront decoding, one independent wave per sequence, union P / R / C
    calls per tick (scheduler_batch.py:228-362).  emus[b] (an
    EmulatedAcceptance) replaces the gold == draft comparison of sequence b."""
    bt = BatchTrace()
    t0 = time.perf_counter()
    cache, lanes = _start(blocks, prompt_ids, emus, max_new_tokens, bt, t0)
    deep, shallow = policy.T_total, policy.T_draft
    for lane in lanes:
        if not lane.finished:
            lane.enqueue(lane.trace.tokens[-1], lane.prompt_len)
    bound = _tick_bound(max_new_tokens, deep)
    for _tick in range(bound + 1):
        live = [lane for lane in lanes if not lane.finished]
        if not live:
            return _close(bt, lanes, t0, blocks)
        if _tick == bound:
            break
        # prelude: queued tokens enter their lane's wave
        entering = [(lane, f) for lane in live for f in lane.queue]
        if entering:
            blocks.prelude_union([lane.idx for lane, _ in entering], [f for _, f in entering], cache)
            bt.count_union("P")
            for lane, f in entering:
                lane.wave[f.position] = f
            for lane in live:
                lane.queue = []
        # one loop step for every token in flight
        moving = [(lane, f) for lane in live for f in lane.wave.values()]
        if moving:
            _advance(blocks, cache, bt, moving)
        # read-outs: full depth leaves the wave, draft depth is read in place
        reads = []
        for lane in live:
            full = [f for f in lane.wave.values() if f.step == deep]
            drafts = [f for f in lane.wave.values() if f.step == shallow and f.step != deep]
            for f in full:
                del lane.wave[f.position]
            if full or drafts:
                reads.append((lane, sorted(full, key=lambda f: f.position), drafts))
        if not reads:
            continue
        rows = [(lane, f) for lane, full, drafts in reads for f in full + drafts]
        heads = [int(x) for x in blocks.coda_argmax_union([lane.idx for lane, _ in rows], [f for _, f in rows],
                                                          cache)]
        bt.count_union("C")
        at = 0
        for lane, full, drafts in reads:
            lane.trace.n_c_calls += 1
            n_full = len(full)
            _wave_settle(lane, full, heads[at:at + n_full], drafts, heads[at + n_full:at + n_full + len(drafts)],
                         cache, max_new_tokens)
            at += n_full + len(drafts)
    raise RuntimeError(f"wavefront scheduler: no progress after {bound} ticks")


# ---------------------------------------------------------------------------
# draft-then-verify
# ---------------------------------------------------------------------------
class _DtvRound:
    """One round of a lane: a chain of up to K + 1 sources, each run to draft
    depth in turn (its read-out is the next source), then all verified together
    at full depth."""
    __slots__ = ("budget", "chain", "guesses", "stage", "next_tok", "next_pos")

    def __init__(self, budget: int, seed_tok: int, seed_pos: int):
        self.budget = budget        # drafts K of this round
        self.chain: list[Flight] = []
        self.guesses: list[int] = []
        self.stage = "prelude"      # prelude -> draft (-> prelude -> draft ...) -> verify
        self.next_tok, self.next_pos = seed_tok, seed_pos


def _dtv_open(lane: _Lane, limit: int, draft_length: int) -> None:
    lane.round = _DtvRound(min(draft_length, limit - lane.n_committed), lane.anchor_tok, lane.anchor_pos)


def _dtv_verify(lane: _Lane, heads, cache, limit: int, draft_length: int) -> None:
    """Source i's full-depth id checks guess i; the first mismatch is committed
    in its place and the sequence's KV is dropped from there; a fully accepted
    round also commits the last source's id."""
    rnd, trace = lane.round, lane.trace
    base = lane.anchor_pos
    refuted = False
    for i, guess in enumerate(rnd.guesses):
        trace.n_drafts_proposed += 1
        agree = lane.acceptance.draw() if lane.acceptance is not None else heads[i] == guess
        if agree:
            trace.n_drafts_accepted += 1
            lane.emit(guess, limit)
            if lane.finished:
                break
        else:
            trace.n_drafts_rejected += 1
            trace.n_rollback_events += 1
            refuted = True
            lane.emit(heads[i], limit)
            cache.drop_positions_at_and_after(lane.idx, base + i + 1)
            lane.anchor_tok, lane.anchor_pos = heads[i], base + i + 1
            break
    if not refuted and not lane.finished:
        k = len(rnd.guesses)
        lane.emit(heads[k], limit)
        lane.anchor_tok, lane.anchor_pos = heads[k], base + k + 1
    if lane.finished:
        lane.retire()
    else:
        _dtv_open(lane, limit, draft_length)


def generate_dtv_batch(blocks, prompt_ids, max_new_tokens: int, policy: SsdPolicy, draft_length: int,
                       emus: list | None = None) -> BatchTrace:
    """Draft-then-verify over union P / R / C calls (scheduler_batch.py:365-501).

    A round of a sequence: K = min(draft_length, tokens still to commit)
    drafts.  Source 0 is the last committed token; each source runs the prelude
    and T_draft loop steps, and its greedy id there is the next source (a
    draft).  Then the K + 1 sources advance together from T_draft to T_total
    (one window per sequence: consecutive positions on one depth slot) and their
    full-depth ids verify the drafts.  emus[b] replaces the comparison."""
    bt = BatchTrace()
    t0 = time.perf_counter()
    cache, lanes = _start(blocks, prompt_ids, emus, max_new_tokens, bt, t0)
    deep, shallow = policy.T_total, policy.T_draft
    widen = getattr(blocks, "ensure_window_rows", None)
    if widen is not None:
        widen(draft_length + 1)   # the verify union attends a sequence's K + 1 sources as one window
    for lane in lanes:
        if not lane.finished:
            lane.anchor_tok, lane.anchor_pos = lane.trace.tokens[-1], lane.prompt_len
            _dtv_open(lane, max_new_tokens, draft_length)
    bound = _tick_bound(max_new_tokens, (draft_length + 1) * shallow + deep)
    for _tick in range(bound + 1):
        live = [lane for lane in lanes if not lane.finished]
        if not live:
            return _close(bt, lanes, t0, blocks)
        if _tick == bound:
            break
        # prelude: the next source of every round that needs one
        starting = [lane for lane in live if lane.round.stage == "prelude"]
        if starting:
            toks = []
            for lane in starting:
                rnd = lane.round
                src = Flight(rnd.next_tok, rnd.next_pos)
                rnd.chain.append(src)
                rnd.stage = "draft"
                lane.trace.n_p_calls += 1
                toks.append(src)
            blocks.prelude_union([lane.idx for lane in starting], toks, cache)
            bt.count_union("P")
        # loop step: the current source of a drafting round, or every source of
        # a verifying round that has not reached full depth
        moving = []
        for lane in live:
            rnd = lane.round
            if rnd.stage == "draft":
                moving.append((lane, rnd.chain[-1]))
            elif rnd.stage == "verify" and rnd.chain[0].step < deep:
                moving += [(lane, f) for f in rnd.chain]
        if moving:
            _advance(blocks, cache, bt, moving)
        # read-outs: a source at draft depth, or a whole chain at full depth
        reads = []
        for lane in live:
            rnd = lane.round
            if rnd.stage == "draft" and rnd.chain[-1].step == shallow:
                reads.append((lane, [rnd.chain[-1]]))
            elif rnd.stage == "verify" and rnd.chain[0].step == deep:
                reads.append((lane, list(rnd.chain)))
        if not reads:
            continue
        heads = [int(x) for x in blocks.coda_argmax_union([lane.idx for lane, ts in reads for _ in ts],
                                                          [f for _, ts in reads for f in ts], cache)]
        bt.count_union("C")
        at = 0
        for lane, ts in reads:
            mine = heads[at:at + len(ts)]
            at += len(ts)
            lane.trace.n_c_calls += 1
            rnd = lane.round
            if rnd.stage == "draft":
                if len(rnd.chain) - 1 < rnd.budget:
                    rnd.guesses.append(mine[0])     # the draft for the position after this source
                rnd.next_tok, rnd.next_pos = mine[0], rnd.chain[-1].position + 1
                rnd.stage = "prelude" if len(rnd.chain) <= rnd.budget else "verify"
            else:
                _dtv_verify(lane, mine, cache, max_new_tokens, draft_length)
    raise RuntimeError(f"draft-then-verify scheduler: no progress after {bound} ticks")
