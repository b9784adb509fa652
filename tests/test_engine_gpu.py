"""End-to-end: the GPU wavefront engine (union P/R/C over the wavefront kernels,
CUDA graphs) driven by the batch schedulers.

* sequential loop decoding on the engine == the float64 full-recompute oracle;
* greedy wavefront decoding == sequential loop decoding, token for token, for
  every T_draft (the lossless claim, README of the reference, scheduler.py:14-17);
* graph replay == eager launches;
* emulated acceptance (rollbacks every few ticks) keeps every sequence's
  commits consistent (alpha = 1: no rejects, exactly N commits).
fp32 model: no reduced-precision GEMMs, so token equality is a fair test.
"""
from __future__ import annotations

import pytest
import torch

import golden_inputs as gi

pytestmark = pytest.mark.gpu


def _small_cfg(**kw):
    from wavefront_decoding_b200.looped_lm import LoopedLMConfig
    base = dict(vocab=512, d_model=256, n_heads=4, n_kv_heads=2, head_dim=64, d_ff=512, n_prelude=1, n_core=2,
                n_coda=1, T_total=4)
    base.update(kw)
    return LoopedLMConfig(**base)


def _engine(cfg, B, S, dtype=torch.float32, graphs=True, seed=0):
    from wavefront_decoding_b200.engine import WaveEngine
    from wavefront_decoding_b200.looped_lm import LoopedLM
    torch.backends.cuda.matmul.allow_tf32 = False
    model = LoopedLM(cfg, seed=seed, dtype=dtype, device="cuda")
    return model, WaveEngine(model, B, S, use_graphs=graphs)


def _prompts(B, L, vocab, seed=5):
    return torch.randint(0, vocab, (B, L), generator=gi.gen(seed))


def test_engine_ar_matches_full_recompute_oracle(cuda_dev):
    from oracle import looped_lm as olm
    from wavefront_decoding_b200 import scheduler as sch
    cfg = _small_cfg()
    B, L, N = 2, 12, 10
    model, eng = _engine(cfg, B, L + N + 16)
    prompts = _prompts(B, L, cfg.vocab)
    bt = sch.ar_generate_batch(eng, prompts, N)
    W, c = olm.weights_from(model)
    for b in range(B):
        ids = prompts[b].tolist()
        for i, tok in enumerate(bt.per_seq[b].tokens):
            lg = olm.last_logits(W, c, torch.tensor(ids))
            want = int(lg.argmax())
            if tok != want:
                # fp32 vs fp64 may only disagree on a near-tie; the streams diverge after it
                assert float(lg[want] - lg[tok]) < 1e-4, (b, i, tok, want)
                break
            ids.append(tok)


@pytest.mark.parametrize("T_draft", [1, 2, 4])
def test_engine_wfd_equals_sequential(cuda_dev, T_draft):
    from wavefront_decoding_b200 import scheduler as sch
    cfg = _small_cfg()
    B, L, N = 3, 10, 24
    prompts = _prompts(B, L, cfg.vocab, seed=6)
    _, eng = _engine(cfg, B, L + N + 16)
    ar = sch.ar_generate_batch(eng, prompts, N)
    _, eng2 = _engine(cfg, B, L + N + 16)
    wfd = sch.generate_wavefront_batch(eng2, prompts, N, sch.SsdPolicy(T_total=4, T_draft=T_draft), None)
    assert [t.tokens for t in wfd.per_seq] == [t.tokens for t in ar.per_seq]
    if T_draft < 4:
        assert sum(t.n_drafts_proposed for t in wfd.per_seq) > 0
    assert eng2.n_graph_replays > 0
    from wavefront_decoding_b200 import runtime as rt
    assert rt.read_device_error(cuda_dev) == 0


def test_engine_graphs_equal_eager(cuda_dev):
    from wavefront_decoding_b200 import scheduler as sch
    cfg = _small_cfg(n_kv_heads=4)
    B, L, N = 2, 9, 16
    prompts = _prompts(B, L, cfg.vocab, seed=8)
    outs = []
    for graphs in (True, False):
        _, eng = _engine(cfg, B, L + N + 16, graphs=graphs)
        emus = [sch.EmulatedAcceptance(0.6, seed=3 + b) for b in range(B)]
        bt = sch.generate_wavefront_batch(eng, prompts, N, sch.SsdPolicy(4, 1), emus)
        outs.append(([t.tokens for t in bt.per_seq], [t.n_rollback_events for t in bt.per_seq]))
    assert outs[0] == outs[1]


def test_engine_emulated_acceptance(cuda_dev):
    from wavefront_decoding_b200 import scheduler as sch
    cfg = _small_cfg()
    B, L, N = 4, 8, 20
    prompts = _prompts(B, L, cfg.vocab, seed=9)
    _, eng = _engine(cfg, B, L + N + 16, dtype=torch.bfloat16)
    emus = [sch.EmulatedAcceptance(1.0, seed=b) for b in range(B)]
    bt = sch.generate_wavefront_batch(eng, prompts, N, sch.SsdPolicy(4, 2), emus)
    for t in bt.per_seq:
        assert len(t.tokens) == N and t.n_drafts_rejected == 0
    _, eng = _engine(cfg, B, L + N + 16, dtype=torch.bfloat16)
    emus = [sch.EmulatedAcceptance(0.5, seed=20 + b) for b in range(B)]
    bt = sch.generate_wavefront_batch(eng, prompts, N, sch.SsdPolicy(4, 1), emus)
    assert sum(t.n_rollback_events for t in bt.per_seq) > 0
    for t in bt.per_seq:
        assert len(t.tokens) == N
    # after the run every slot length of a sequence stays within its committed span
    lens = eng.cache.seqlen
    for b in range(B):
        assert max(lens[s][b] for s in range(cfg.n_slots)) <= L + N + 2 * cfg.T_total
    from wavefront_decoding_b200 import runtime as rt
    assert rt.read_device_error(cuda_dev) == 0


# ---------------------------------------------------------------------------
# config 1: the reference's ParcaeBlocks tokens / counters / KV lengths
# ---------------------------------------------------------------------------
def _config1_engine(kv_budget_s: int = 0):
    import parcae_fixture as pf
    from wavefront_decoding_b200.engine import WaveEngine
    from wavefront_decoding_b200.looped_lm import LoopedLM
    from test_config1 import GOLD
    torch.backends.cuda.matmul.allow_tf32 = False
    m = pf.ParcaeFixture(seed=0)
    model = LoopedLM(pf.looped_config(m, GOLD["T_total"], kv_budget_s), dtype=torch.float32, device="cuda")
    model.load_weights(pf.to_looped_weights(m))
    return WaveEngine(model, 1, 256), pf.config1_prompt()[None], GOLD


def test_config1_ar_matches_reference(cuda_dev):
    from wavefront_decoding_b200 import scheduler as sch
    eng, prompt, gold = _config1_engine()
    bt = sch.ar_generate_batch(eng, prompt, gold["n_new"])
    assert bt.per_seq[0].tokens == gold["ar"]["tokens"]
    lens = eng.cache.seqlen
    assert {str(s): lens[s][0] for s in range(len(lens))} == gold["ar"]["seqlen"]


@pytest.mark.parametrize("T_draft", [1, 2, 4])
def test_config1_wfd_matches_reference(cuda_dev, T_draft):
    from wavefront_decoding_b200 import scheduler as sch
    eng, prompt, gold = _config1_engine()
    g = gold[f"wfd_d{T_draft}"]
    bt = sch.generate_wavefront_batch(eng, prompt, gold["n_new"], sch.SsdPolicy(gold["T_total"], T_draft), None)
    t = bt.per_seq[0]
    assert t.tokens == g["tokens"] == gold["ar"]["tokens"]
    for k in ("n_drafts_proposed", "n_drafts_accepted", "n_drafts_rejected", "n_rollback_events"):
        assert getattr(t, k) == g[k], k
    lens = eng.cache.seqlen
    assert {str(s): lens[s][0] for s in range(len(lens))} == g["seqlen"]


@pytest.mark.parametrize("T_draft,K", [(1, 3), (2, 4), (2, 1)])
def test_config1_dtv_is_lossless(cuda_dev, T_draft, K):
    """Draft-then-verify on the engine (the verify union attends each sequence's
    K + 1 sources as one window on their depth slot): greedy DtV commits the
    reference's AR tokens, and the cache holds every depth's K / V of the
    committed positions as sequential decoding would."""
    from wavefront_decoding_b200 import scheduler as sch
    eng, prompt, gold = _config1_engine()
    bt = sch.generate_dtv_batch(eng, prompt, gold["n_new"], sch.SsdPolicy(gold["T_total"], T_draft), K)
    t = bt.per_seq[0]
    assert t.tokens == gold["ar"]["tokens"]
    assert t.n_drafts_proposed > 0 and bt.r_union_max >= min(K + 1, 2)
    if K == 3:
        _check_cache_vs_oracle(eng, eng.model, prompt, bt.per_seq, 2e-4)


def _seqlen_as_reference(eng):
    """The engine's slot lengths keyed like the reference's cache: with KV sharing
    ParcaeBlocks keeps its coda slots at n_prelude + T_total * n_core
    (parcae_blocks.py:76), while the engine allocates only the depth slots in use."""
    cfg = eng.cfg
    shift = (cfg.T_total - cfg.n_depth_slots) * cfg.n_core
    lens = eng.cache.seqlen
    return {str(s if s < cfg.slot_coda(0) else s + shift): lens[s][0] for s in range(len(lens))}


@pytest.mark.parametrize("s", [1, 2])
def test_config1_ar_kv_sharing_matches_reference(cuda_dev, s):
    """KV-sharing budget s (core depth r keeps its K/V in slot r % s): the
    reference's AR tokens and slot lengths."""
    from wavefront_decoding_b200 import scheduler as sch
    eng, prompt, gold = _config1_engine(kv_budget_s=s)
    assert eng.cfg.n_slots == 1 + 2 * s + 1
    bt = sch.ar_generate_batch(eng, prompt, gold["n_new"])
    assert bt.per_seq[0].tokens == gold[f"ar_s{s}"]["tokens"]
    assert _seqlen_as_reference(eng) == gold[f"ar_s{s}"]["seqlen"]


@pytest.mark.parametrize("s", [1, 2])
@pytest.mark.parametrize("T_draft", [1, 2])
def test_config1_wfd_kv_sharing_matches_reference(cuda_dev, T_draft, s):
    """KV sharing with the host scheduler: tokens, draft counters (they differ
    from the unshared run's) and slot lengths of the reference.  With s = 1 the
    tokens of a sequence share one depth slot and each run of them is one
    attention window."""
    from wavefront_decoding_b200 import scheduler as sch
    eng, prompt, gold = _config1_engine(kv_budget_s=s)
    g = gold[f"wfd_d{T_draft}_s{s}"]
    bt = sch.generate_wavefront_batch(eng, prompt, gold["n_new"], sch.SsdPolicy(gold["T_total"], T_draft), None)
    t = bt.per_seq[0]
    assert t.tokens == g["tokens"]
    for k in ("n_drafts_proposed", "n_drafts_accepted", "n_drafts_rejected", "n_rollback_events"):
        assert getattr(t, k) == g[k], k
    assert _seqlen_as_reference(eng) == g["seqlen"]


def _check_cache_vs_oracle(eng, model, prompts, per_seq, tol):
    """Every K / V the engine cached for the committed positions equals the
    full-recompute oracle's: each depth's hidden state was computed exactly once
    and at the right depth."""
    from oracle import looped_lm as olm
    W, c = olm.weights_from(model)
    K, V = eng.cache.K, eng.cache.V
    for b, tr in enumerate(per_seq):
        ids = torch.cat([prompts[b], torch.tensor(tr.tokens[:-1], dtype=prompts.dtype)])
        ref = olm.slot_kv(W, c, ids)
        n = ids.numel()
        assert len(ref) == model.cfg.n_slots
        for s, (k, v) in enumerate(ref):
            dk = (K[s, b, :n].double().cpu() - k).abs().max().item()
            dv = (V[s, b, :n].double().cpu() - v).abs().max().item()
            assert dk < tol and dv < tol, (b, s, dk, dv)


@pytest.mark.parametrize("T_draft", [1, 2, 4])
def test_engine_cache_matches_oracle(cuda_dev, T_draft):
    """Stronger than token equality (a looped model that converges in depth hides
    depth mistakes from argmax): the cached K / V at every slot and committed
    position, after sequential and after wavefront decoding."""
    from wavefront_decoding_b200 import scheduler as sch
    cfg = _small_cfg()
    B, L, N = 2, 10, 14
    prompts = _prompts(B, L, cfg.vocab, seed=12)
    model, eng = _engine(cfg, B, L + N + 16)
    if T_draft == 4:
        bt = sch.ar_generate_batch(eng, prompts, N)
    else:
        bt = sch.generate_wavefront_batch(eng, prompts, N, sch.SsdPolicy(4, T_draft), None)
    _check_cache_vs_oracle(eng, model, prompts, bt.per_seq, 2e-4)
