"""Device-side wavefront scheduling (route / settle kernels, one CUDA graph per
tick) against the host scheduler that mirrors the reference
(scheduler.generate_wavefront_batch): same tokens, every per-sequence and batch
counter, and the same final KV slot lengths; plus config 1 against the
reference's own ParcaeBlocks golden and the cached K/V against the oracle."""
from __future__ import annotations

import pytest
import torch

from test_engine_gpu import _check_cache_vs_oracle, _config1_engine, _engine, _prompts, _seqlen_as_reference, _small_cfg

pytestmark = pytest.mark.gpu

_CT = ("n_p_calls", "n_r_calls", "n_c_calls", "n_drafts_proposed", "n_drafts_accepted", "n_drafts_rejected",
       "n_rollback_events")


def _summary(bt, eng, B):
    lens = eng.cache.lens[:, :B].cpu().tolist()
    return ([t.tokens for t in bt.per_seq], [[getattr(t, k) for k in _CT] for t in bt.per_seq],
            [bt.n_r_calls, bt.n_p_calls, bt.n_c_calls, bt.r_union_total, bt.r_union_max], lens)


def _both(cfg, B, L, N, T_draft, alpha=None, seed=0, pseed=21, dtype=torch.float32):
    from wavefront_decoding_b200 import scheduler as sch
    from wavefront_decoding_b200.device_scheduler import generate_wavefront_device
    prompts = _prompts(B, L, cfg.vocab, seed=pseed)
    pol = sch.SsdPolicy(cfg.T_total, T_draft)

    def emus():
        return None if alpha is None else [sch.EmulatedAcceptance(alpha, seed=50 + b) for b in range(B)]

    _, eh = _engine(cfg, B, L + N + 2 * cfg.T_total + 8, dtype=dtype, seed=seed)
    host = sch.generate_wavefront_batch(eh, prompts, N, pol, emus())
    model, ed = _engine(cfg, B, L + N + 2 * cfg.T_total + 8, dtype=dtype, seed=seed)
    dev = generate_wavefront_device(ed, prompts, N, pol, emus())
    return _summary(host, eh, B), _summary(dev, ed, B), (model, ed, prompts, dev)


@pytest.mark.parametrize("T_draft", [1, 2, 4])
def test_device_matches_host_greedy(cuda_dev, T_draft):
    cfg = _small_cfg()
    h, d, _ = _both(cfg, 3, 10, 24, T_draft)
    assert d == h


@pytest.mark.parametrize("alpha,T_draft", [(0.5, 1), (0.8, 2), (0.3, 2)])
def test_device_matches_host_emulated(cuda_dev, alpha, T_draft):
    cfg = _small_cfg(n_kv_heads=4)
    h, d, _ = _both(cfg, 5, 9, 30, T_draft, alpha=alpha)
    assert d == h
    assert sum(x[6] for x in d[1]) > 0          # rollbacks exercised


@pytest.mark.parametrize("s,alpha,T_draft", [(1, 0.6, 1), (1, 0.8, 2), (2, 0.5, 1)])
def test_device_matches_host_kv_sharing(cuda_dev, s, alpha, T_draft):
    """KV sharing under emulated acceptance (many rollbacks): the pre-tick kernel's
    ordering of each sequence's rows and its shared-slot windows reproduce the host
    scheduler's tables exactly (tokens, counters, union sizes, KV lengths)."""
    cfg = _small_cfg(n_kv_heads=4, kv_budget_s=s)
    h, d, _ = _both(cfg, 5, 9, 30, T_draft, alpha=alpha)
    assert d == h
    assert sum(x[6] for x in d[1]) > 0          # rollbacks exercised


def test_device_cache_matches_oracle(cuda_dev):
    cfg = _small_cfg()
    _, _, (model, eng, prompts, bt) = _both(cfg, 2, 10, 14, 2)
    _check_cache_vs_oracle(eng, model, prompts, bt.per_seq, 2e-4)


def test_device_graph_equals_eager(cuda_dev):
    from wavefront_decoding_b200 import scheduler as sch
    from wavefront_decoding_b200.device_scheduler import generate_wavefront_device
    cfg = _small_cfg()
    B, L, N = 4, 8, 20
    prompts = _prompts(B, L, cfg.vocab, seed=23)
    outs = []
    for graph in (True, False):
        _, eng = _engine(cfg, B, L + N + 16)
        emus = [sch.EmulatedAcceptance(0.6, seed=3 + b) for b in range(B)]
        bt = generate_wavefront_device(eng, prompts, N, sch.SsdPolicy(4, 1), emus, use_graph=graph)
        outs.append(_summary(bt, eng, B))
    assert outs[0] == outs[1]


@pytest.mark.parametrize("T_draft", [1, 2, 4])
def test_device_config1_matches_reference(cuda_dev, T_draft):
    from wavefront_decoding_b200 import scheduler as sch
    from wavefront_decoding_b200.device_scheduler import generate_wavefront_device
    eng, prompt, gold = _config1_engine()
    g = gold[f"wfd_d{T_draft}"]
    bt = generate_wavefront_device(eng, prompt, gold["n_new"], sch.SsdPolicy(gold["T_total"], T_draft))
    t = bt.per_seq[0]
    assert t.tokens == g["tokens"] == gold["ar"]["tokens"]
    for k in ("n_drafts_proposed", "n_drafts_accepted", "n_drafts_rejected", "n_rollback_events"):
        assert getattr(t, k) == g[k], k
    lens = eng.cache.seqlen
    assert {str(s): lens[s][0] for s in range(len(lens))} == g["seqlen"]


@pytest.mark.parametrize("s", [1, 2])
@pytest.mark.parametrize("T_draft", [1, 2])
def test_device_config1_kv_sharing_matches_reference(cuda_dev, T_draft, s):
    """KV sharing with route / settle on the device (the pre-tick kernel orders
    each sequence's rows and forms the shared-slot windows): the reference's
    tokens, counters and slot lengths."""
    from wavefront_decoding_b200 import scheduler as sch
    from wavefront_decoding_b200.device_scheduler import generate_wavefront_device
    eng, prompt, gold = _config1_engine(kv_budget_s=s)
    g = gold[f"wfd_d{T_draft}_s{s}"]
    bt = generate_wavefront_device(eng, prompt, gold["n_new"], sch.SsdPolicy(gold["T_total"], T_draft))
    t = bt.per_seq[0]
    assert t.tokens == g["tokens"]
    for k in ("n_drafts_proposed", "n_drafts_accepted", "n_drafts_rejected", "n_rollback_events"):
        assert getattr(t, k) == g[k], k
    assert _seqlen_as_reference(eng) == g["seqlen"]


def test_device_repeat_generation_reuses_graph(cuda_dev):
    """A DeviceWave generates twice with one captured graph; same result."""
    from wavefront_decoding_b200 import scheduler as sch
    from wavefront_decoding_b200.device_scheduler import DeviceWave
    cfg = _small_cfg()
    B, L, N = 3, 7, 12
    prompts = _prompts(B, L, cfg.vocab, seed=24)
    _, eng = _engine(cfg, B, L + N + 16)
    dw = DeviceWave(eng, N, sch.SsdPolicy(4, 2))
    a = _summary(dw.generate(prompts), eng, B)
    b = _summary(dw.generate(prompts), eng, B)
    assert a == b and len(dw._graphs) == 1


@pytest.mark.parametrize("cfg_name", ["small", "config1"])
def test_bf16_wavefront_bit_exact_with_batch_invariance(cuda_dev, cfg_name):
    """bf16: with fixed union capacities and batch-invariant attention, greedy
    wavefront decoding (T_draft 1, 2) commits exactly the tokens of sequential
    decoding (T_draft = T_total) for every sequence."""
    from wavefront_decoding_b200 import scheduler as sch
    from wavefront_decoding_b200.device_scheduler import generate_wavefront_device
    from wavefront_decoding_b200.looped_lm import CONFIG1
    cfg = _small_cfg() if cfg_name == "small" else CONFIG1
    B, L, N = (8, 16, 40) if cfg_name == "small" else (4, 128, 48)
    prompts = _prompts(B, L, cfg.vocab, seed=31)
    runs = {}
    for d in (cfg.T_total, 1, 2):
        _, eng = _engine(cfg, B, L + N + 2 * cfg.T_total + 8, dtype=torch.bfloat16)
        bt = generate_wavefront_device(eng, prompts, N, sch.SsdPolicy(cfg.T_total, d), batch_invariant=True)
        runs[d] = [t.tokens for t in bt.per_seq]
    assert runs[1] == runs[cfg.T_total]
    assert runs[2] == runs[cfg.T_total]


def test_gapped_windows_bf16_kv_sharing(cuda_dev):
    """bf16 with KV sharing s = 2: a sequence's tokens on one depth slot attend as
    one gapped window (per-row positions) in both schedulers.  Under emulated
    acceptance the schedule does not depend on token values, so host and device
    give identical counters, union sizes and KV lengths; the committed tokens
    agree as well, apart from rare bf16 rounding differences between the two
    schedulers' union shapes."""
    from wavefront_decoding_b200 import runtime as rt
    cfg = _small_cfg(n_kv_heads=4, kv_budget_s=2)
    h, d, (model, ed, prompts, _) = _both(cfg, 5, 9, 30, 1, alpha=0.7, dtype=torch.bfloat16)
    assert ed.gap_windows
    assert d[1] == h[1] and d[2] == h[2] and d[3] == h[3]
    assert sum(x[6] for x in d[1]) > 0          # rollbacks exercised (irregular gaps)
    same = sum(a == b for ta, tb in zip(d[0], h[0]) for a, b in zip(ta, tb))
    assert same >= 0.8 * sum(len(t) for t in h[0])
    assert rt.read_device_error(cuda_dev) == 0
