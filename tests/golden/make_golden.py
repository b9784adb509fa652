"""Generate the golden vectors that pin the CPU oracle to the reference.

Run in a checkout that has the reference tree available (it is NOT needed at
test time; only the .npz / .json outputs are committed):

    python tests/golden/make_golden.py --reference <path-to-wavefront-decoding>

It imports the reference's own `src/decoding/fa4_attention.py` (SDPA backend,
`set_backend("sdpa")`) and `src/decoding/batch_kv_cache.py` on CPU.  The
reference imports two helpers from its empty `external/parcae` submodule
(fa4_attention.py:55-56); the fixture model's own functions
(tests/parcae_fixture.py) stand in for them.

Config 1 (end-to-end greedy decoding) runs the reference's own `ParcaeBlocks`
with `ar_generate_parcae_blocks` and `generate_wavefront_dynamic` over the
fixture model (seed 0, initial recurrent state "zero"), and stores the tokens,
counters and final KV slot lengths.

Inputs are drawn from torch CPU generators with fixed seeds and are NOT stored
(except tiny index tables); the tests regenerate them with the same calls and
check the stored input checksums first, so an RNG change fails loudly instead
of silently comparing different data.
"""
from __future__ import annotations

import argparse
import json
import pathlib
import sys
import types

import numpy as np
import torch

HERE = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))
import golden_inputs as gi  # noqa: E402  (shared input recipes, tests/golden_inputs.py)


def import_reference(ref_root: str):
    for name in ("parcae_lm", "parcae_lm.modules", "parcae_lm.modules.mixer", "parcae_lm.modules.utils"):
        sys.modules.setdefault(name, types.ModuleType(name))

    # the fixture model's own RoPE / qk-norm stand in for parcae_lm's (qk-norm is
    # off in the fixture and raises if called)
    import parcae_fixture as pf
    sys.modules["parcae_lm.modules.mixer"].norm = pf.qk_norm
    sys.modules["parcae_lm.modules.utils"].apply_rotary_emb_complex_like = pf.apply_rotary_emb_complex_like
    sys.path.insert(0, ref_root)
    import src.decoding.fa4_attention as fa  # noqa: E402
    from src.decoding.batch_kv_cache import BatchStaticKVCache  # noqa: E402
    fa.set_backend("sdpa")
    return fa, BatchStaticKVCache


def f32(t: torch.Tensor) -> np.ndarray:
    return t.detach().to(torch.float32).numpy()


def gen_attention(fa) -> dict:
    out = {}
    # ---- varlen cases (fp32 and bf16 inputs) ----
    for case in gi.VARLEN_CASES:
        q, k, v, cu_q, cu_k = gi.varlen_inputs(case)
        o = fa.attn_varlen(q, k, v, cu_q, cu_k, int((cu_q[1:] - cu_q[:-1]).max()),
                           int((cu_k[1:] - cu_k[:-1]).max()), causal=case["causal"])
        out[f"varlen/{case['name']}/out"] = f32(o)
        out[f"varlen/{case['name']}/checksum"] = np.asarray(gi.checksum(q, k, v))
    # ---- q1 padded ----
    q, k, v, cu_q, cu_k = gi.varlen_inputs(gi.Q1_PADDED_CASE)
    o = fa.attn_varlen_q1_padded(q, k, v, cu_k, int((cu_k[1:] - cu_k[:-1]).max()))
    out["q1_padded/out"] = f32(o)
    out["q1_padded/checksum"] = np.asarray(gi.checksum(q, k, v))
    # ---- dense ----
    for case in gi.DENSE_CASES:
        q, k, v = gi.dense_inputs(case)
        o = fa.attn_dense(q, k, v, causal=case["causal"])
        out[f"dense/{case['name']}/out"] = f32(o)
        out[f"dense/{case['name']}/checksum"] = np.asarray(gi.checksum(q, k, v))
    # ---- cutoff multi ----
    q, k, v, qpos = gi.cutoff_inputs()
    o = fa.attn_cutoff_multi(q, k, v, qpos)
    out["cutoff/out"] = f32(o)
    out["cutoff/checksum"] = np.asarray(gi.checksum(q, k, v))
    # ---- exp5 gate 1 shapes (verify_graph.py:45-147): lengths as data ----
    K, V, q1, q8 = gi.gate1_inputs()
    out["gate1/checksum"] = np.asarray(gi.checksum(K, V, q1, q8))
    for n in gi.GATE1_LENGTHS:
        cu1 = torch.tensor([0, 1], dtype=torch.int32)
        cuk = torch.tensor([0, n], dtype=torch.int32)
        oa = fa.attn_varlen(q1, K[:n], V[:n], cu1, cuk, 1, n, causal=False)
        cu8 = torch.tensor([0, 8], dtype=torch.int32)
        ob = fa.attn_varlen(q8, K[:n], V[:n], cu8, cuk, 8, n, causal=True)
        out[f"gate1/a/{n}"] = f32(oa)
        out[f"gate1/b/{n}"] = f32(ob)
    return out


def gen_kv_cache(BatchStaticKVCache) -> dict:
    """Scripted BatchStaticKVCache session: prefill, token writes, per-sequence
    rollbacks, gather_pack — the final seqlen table and packed K/V."""
    n_slots, B, S, Hkv, Dh = gi.KV_SCRIPT_GEOM
    c = BatchStaticKVCache(n_slots, B, Hkv, Dh, S, torch.float32, torch.device("cpu"))
    log = {"seqlen": []}
    tensors = {}
    for step, op in enumerate(gi.kv_script()):
        kind = op[0]
        if kind == "prefill":
            _, slot, k, v = op
            c.write_prefill(slot, k, v)
        elif kind == "tokens":
            _, slots, seqs, pos, k, v = op
            c.write_tokens(slots, seqs, pos, k, v)
        elif kind == "drop":
            _, b, p = op
            c.drop_positions_at_and_after(b, p)
        elif kind == "pack":
            _, slots, seqs, uptos = op
            kp, vp, cu_k, max_k = c.gather_pack(slots, seqs, uptos)
            tensors[f"kv/pack{step}/k"] = f32(kp)
            tensors[f"kv/pack{step}/v"] = f32(vp)
            tensors[f"kv/pack{step}/cu_k"] = cu_k.numpy()
            tensors[f"kv/pack{step}/max_k"] = np.asarray(max_k)
        log["seqlen"].append([row[:] for row in c.seqlen])
    tensors["kv/seqlen_final"] = np.asarray(c.seqlen, dtype=np.int64)
    return tensors, log


def gen_cfg3_commit(BatchStaticKVCache) -> dict:
    """Config 3 commit: window of 8 rows at positions [8192-r, 8200-r) of slot r;
    sequence b accepts a_b ~ U{0..8} (seed 3).  Each slot's rollback is the
    reference's drop_positions_at_and_after(b, 8192 - r + a_b) on that slot."""
    R, B, L0, W = 8, 32, 8192, 8
    a = gi.cfg3_accept()
    seqlen = np.zeros((R, B), dtype=np.int64)
    for r in range(R):
        c = BatchStaticKVCache(1, B, 1, 1, L0 + W, torch.float32, torch.device("cpu"))
        c.seqlen = [[L0 - r + W] * B]
        for b in range(B):
            c.drop_positions_at_and_after(b, L0 - r + int(a[b]))
        seqlen[r] = np.asarray(c.seqlen[0])
    return {"cfg3/accept": a.numpy().astype(np.int64), "cfg3/seqlen": seqlen}


def gen_scheduler() -> dict:
    """The reference's own batch schedulers (scheduler_batch.py:185-362) driven
    by the deterministic FakeBlocks: committed tokens, every per-sequence and
    batch counter, and the rollback calls, per case."""
    from src.decoding import scheduler_batch as sb
    from src.decoding.emu import EmulatedAcceptance
    from src.decoding.policy import SsdPolicy
    out = {}
    for case in gi.SCHED_CASES:
        blocks = gi.FakeBlocks(case["T_total"])
        prompts = gi.sched_prompts(case)
        emus = None
        if case["alpha"] is not None:
            emus = [EmulatedAcceptance(case["alpha"], seed=100 + b) for b in range(case["B"])]
        bt = sb.generate_wavefront_batch(blocks, prompts, case["new"],
                                         SsdPolicy(T_total=case["T_total"], T_draft=case["T_draft"]), emus)
        out[case["name"]] = gi.trace_summary(bt, blocks.last_cache)
    blocks = gi.FakeBlocks(4)
    prompts = gi.sched_prompts(gi.SCHED_CASES[0])
    bt = sb.ar_generate_batch(blocks, prompts, 12)
    out["ar_T4"] = gi.trace_summary(bt, blocks.last_cache)
    for case in gi.DTV_CASES:
        blocks = gi.FakeBlocks(case["T_total"])
        prompts = gi.sched_prompts(case)
        emus = None
        if case["alpha"] is not None:
            emus = [EmulatedAcceptance(case["alpha"], seed=200 + b) for b in range(case["B"])]
        bt = sb.generate_dtv_batch(blocks, prompts, case["new"],
                                   SsdPolicy(T_total=case["T_total"], T_draft=case["T_draft"]), case["K"], emus)
        out[case["name"]] = gi.trace_summary(bt, blocks.last_cache)
    return out


def gen_config1(n_new: int = 64, T_total: int = 4, drafts=(1, 2, 4), budgets=(2, 1), budget_drafts=(1, 2)) -> dict:
    """Config 1: the reference's ParcaeBlocks on the fixture model, greedy, fp32,
    SDPA backend; AR (ar_baseline.py:132-193) and WFD (scheduler.py:89-225).
    With KV sharing (`kv_budget_s` = s < T_total, parcae_blocks.py:77-81,114-120:
    core depth r uses recurrence slot r % s, last write wins) for AR and WFD at
    the given draft depths; keys ar_s{s} / wfd_d{d}_s{s}."""
    import parcae_fixture as pf
    from src.decoding.ar_baseline import ar_generate_parcae_blocks
    from src.decoding.parcae_blocks import ParcaeBlocks
    from src.decoding.policy import SsdPolicy
    from src.decoding.scheduler import generate_wavefront_dynamic

    model = pf.ParcaeFixture(seed=0).eval()
    prompt = pf.config1_prompt()

    def blocks(budget=None):
        b = ParcaeBlocks(model, T_total, max_seq_len=pf.MAX_SEQ)
        b.state_init = "zero"
        b.kv_budget_s = budget
        caches = []
        orig = b.prefill

        def prefill(*a, **k):
            st, lg = orig(*a, **k)
            caches.append(st.kv_cache)
            return st, lg

        b.prefill = prefill
        return b, caches

    def lens(cache):
        return {str(k): int(v) for k, v in sorted(cache.seqlen.items())}

    out = {"prompt_head": prompt[:8].tolist(), "n_new": n_new, "T_total": T_total,
           "weight_sums": pf.weight_sums(model)}
    b, caches = blocks()
    toks, _ = ar_generate_parcae_blocks(b, prompt[None], n_new)
    out["ar"] = {"tokens": [int(t) for t in toks], "seqlen": lens(caches[-1])}
    for d in drafts:
        b, caches = blocks()
        toks, tr = generate_wavefront_dynamic(b, prompt, n_new, SsdPolicy(T_total=T_total, T_draft=d))
        out[f"wfd_d{d}"] = {"tokens": [int(t) for t in toks], "seqlen": lens(caches[-1]),
                            **{k: getattr(tr, k) for k in ("n_r_calls", "n_p_calls", "n_c_calls", "n_drafts_proposed",
                                                           "n_drafts_accepted", "n_drafts_rejected",
                                                           "n_rollback_events")}}
        print(f"config1 T_draft={d}: {out[f'wfd_d{d}']['n_drafts_accepted']}/"
              f"{out[f'wfd_d{d}']['n_drafts_proposed']} drafts accepted")
    counters = ("n_r_calls", "n_p_calls", "n_c_calls", "n_drafts_proposed", "n_drafts_accepted",
                "n_drafts_rejected", "n_rollback_events")
    for sb in budgets:
        b, caches = blocks(sb)
        toks, _ = ar_generate_parcae_blocks(b, prompt[None], n_new)
        out[f"ar_s{sb}"] = {"tokens": [int(t) for t in toks], "seqlen": lens(caches[-1])}
        for d in budget_drafts:
            b, caches = blocks(sb)
            toks, tr = generate_wavefront_dynamic(b, prompt, n_new, SsdPolicy(T_total=T_total, T_draft=d))
            key = f"wfd_d{d}_s{sb}"
            out[key] = {"tokens": [int(t) for t in toks], "seqlen": lens(caches[-1]),
                        **{k: getattr(tr, k) for k in counters}}
            print(f"config1 kv_budget_s={sb} T_draft={d}: {out[key]['n_drafts_accepted']}/"
                  f"{out[key]['n_drafts_proposed']} drafts accepted, "
                  f"{sum(a != c for a, c in zip(out[key]['tokens'], out[f'ar_s{sb}']['tokens']))} tokens differ from AR")
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    ap.add_argument("--only", choices=["all", "config1", "scheduler"], default="all")
    args = ap.parse_args()
    fa, BSK = import_reference(args.reference)
    if args.only in ("all", "config1"):
        (HERE / "reference_config1.json").write_text(json.dumps(gen_config1(), indent=0) + "\n")
    if args.only == "config1":
        return
    if args.only == "scheduler":
        (HERE / "reference_scheduler.json").write_text(json.dumps(gen_scheduler(), indent=0) + "\n")
        return
    data = {}
    data.update(gen_attention(fa))
    kv, log = gen_kv_cache(BSK)
    data.update(kv)
    data.update(gen_cfg3_commit(BSK))
    np.savez_compressed(HERE / "reference_golden.npz", **data)
    (HERE / "reference_kv_log.json").write_text(json.dumps(log) + "\n")
    (HERE / "reference_scheduler.json").write_text(json.dumps(gen_scheduler(), indent=0) + "\n")
    total = sum(v.nbytes for v in data.values())
    print(f"wrote {len(data)} arrays ({total / 1e6:.2f} MB raw) to {HERE / 'reference_golden.npz'}")


if __name__ == "__main__":
    main()
