"""The host restatement of the reference's decode loop (oracle/cpu_path.py
LoopedBlocksCPU), which bench.py times as the config-4 CPU baseline, checked
against the float64 full-recompute oracle (oracle/looped_lm.py): its prompt
logits, and the tokens that the package's host schedulers commit through it
(sequential, wavefront, draft-then-verify), which for greedy decoding are the
tokens of sequential decoding."""
from __future__ import annotations

import pytest
import torch

from oracle import cpu_path
from oracle import looped_lm as olm

DIMS = dict(vocab=97, d_model=48, n_heads=4, n_kv_heads=2, head_dim=12, d_ff=64, n_prelude=1, n_core=2,
            n_coda=1, T_total=4, norm_eps=1e-6, rope_theta=10000.0, rope_style="half")


def _setup(seed=0, B=3, L=7, style="half"):
    dims = dict(DIMS, rope_style=style)
    W = cpu_path.random_weights(dims, seed, dtype=torch.float64, std=0.25)
    prompts = torch.randint(0, dims["vocab"], (B, L), generator=torch.Generator().manual_seed(seed + 1))
    return dims, W, prompts


def _sched():
    from wavefront_decoding_b200 import scheduler
    return scheduler


@pytest.mark.parametrize("style", ["half", "interleaved"])
def test_prefill_logits_match_recompute(style):
    dims, W, prompts = _setup(style=style)
    blocks = cpu_path.LoopedBlocksCPU(W, dims, prompts.shape[0], 32, dtype=torch.float64)
    _, logits = blocks.prefill(prompts)
    for b in range(prompts.shape[0]):
        ref = olm.last_logits(W, dims, prompts[b])
        assert float((logits[b].double() - ref).abs().max()) < 1e-5   # logits come back as float32
    # the cached K / V are the recompute's (slot ids as in the package)
    kv = olm.slot_kv(W, dims, prompts[1])
    for slot, (k, v) in enumerate(kv):
        assert float((blocks.K[slot, 1, :prompts.shape[1]] - k).abs().max()) < 1e-9
        assert float((blocks.V[slot, 1, :prompts.shape[1]] - v).abs().max()) < 1e-9


@pytest.mark.parametrize("gen", ["ar", "wavefront_d1", "wavefront_d2", "dtv"])
def test_generation_commits_sequential_tokens(gen):
    sch = _sched()
    dims, W, prompts = _setup(seed=3)
    n_new = 6
    blocks = cpu_path.LoopedBlocksCPU(W, dims, prompts.shape[0], 64, dtype=torch.float64)
    if gen == "ar":
        bt = sch.ar_generate_batch(blocks, prompts, n_new)
    elif gen == "dtv":
        bt = sch.generate_dtv_batch(blocks, prompts, n_new, sch.SsdPolicy(dims["T_total"], 2), 3)
    else:
        bt = sch.generate_wavefront_batch(blocks, prompts, n_new,
                                          sch.SsdPolicy(dims["T_total"], int(gen[-1])))
    for b, tr in enumerate(bt.per_seq):
        assert tr.tokens == olm.greedy_generate(W, dims, prompts[b].tolist(), n_new), (gen, b)


def test_synthetic_prompt_decodes_bf16():
    """The timing mode: random prompt K / V, bf16, the wavefront scheduler runs to
    the end and every slot's length covers the committed tokens."""
    sch = _sched()
    dims = dict(DIMS, T_total=4)
    W = cpu_path.random_weights(dims, 5, dtype=torch.bfloat16)
    prompts = torch.randint(0, dims["vocab"], (2, 16), generator=torch.Generator().manual_seed(2))
    blocks = cpu_path.LoopedBlocksCPU(W, dims, 2, 64, dtype=torch.bfloat16, synthetic_prompt=True)
    bt = sch.generate_wavefront_batch(blocks, prompts, 5, sch.SsdPolicy(4, 2))
    assert [len(t.tokens) for t in bt.per_seq] == [5, 5]
    assert [t.tokens[0] for t in bt.per_seq] == prompts[:, -1].tolist()
    assert min(blocks.seqlen[blocks.slot_coda(0)]) >= 16 + 4
