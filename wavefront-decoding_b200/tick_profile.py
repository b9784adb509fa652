"""Per-tick kernel breakdown of greedy wavefront decoding on the device scheduler.

    python wavefront-decoding_b200/tick_profile.py [--batch 8 64] [--new-tokens 32] [--t-draft 2]

Runs the config-4 looped LM (random init, bf16, 1024-token prompts) once to
capture the tick graph, then once more under torch.profiler (CUPTI kernel
records, no replay) and prints, for the decode ticks only: span and busy time
per tick, every kernel's launches and device time per tick, and each attention
launch's K/V bytes and read rate.  Device times come from CUPTI kernel records
of the graph replays; the kernels run at their normal clocks and overlap (PDL)
as in a plain run, so the busy time per tick is close to a plain run's tick.
"""
from __future__ import annotations

import argparse
import collections
import pathlib
import sys

import torch
from torch.profiler import ProfilerActivity, profile

sys.path.insert(0, str(pathlib.Path(__file__).resolve().parent.parent))
import __graft_entry__  # noqa: E402

__graft_entry__.load_package()
from wavefront_decoding_b200 import scheduler as sch  # noqa: E402
from wavefront_decoding_b200.device_scheduler import DeviceWave  # noqa: E402
from wavefront_decoding_b200.engine import WaveEngine  # noqa: E402
from wavefront_decoding_b200.looped_lm import CONFIG4, LoopedLM  # noqa: E402


def profile_batch(B: int, new: int, t_draft: int, prompt_len: int = 1024) -> None:
    dev = torch.device("cuda", torch.cuda.current_device())
    cfg = CONFIG4
    prompts = torch.randint(0, cfg.vocab, (B, prompt_len), generator=torch.Generator().manual_seed(4)).pin_memory()
    model = LoopedLM(cfg, seed=0, dtype=torch.bfloat16, device=dev)
    eng = WaveEngine(model, B, prompt_len + new + 2 * cfg.T_total + 8)
    dw = DeviceWave(eng, new, sch.SsdPolicy(cfg.T_total, t_draft))
    dw.generate(prompts, None)  # captures the tick graph
    torch.cuda.synchronize()

    # a marker kernel between the prompt pass and the first tick
    orig = eng.prefill

    def prefill(ids):
        out = orig(ids)
        torch.cuda._sleep(1000)
        return out

    eng.prefill = prefill
    try:
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            bt = dw.generate(prompts, None)
            torch.cuda.synchronize()
    finally:
        del eng.prefill
    ks = sorted((e.time_range.start, e.time_range.end, e.name) for e in prof.events()
                if e.device_type == torch.autograd.DeviceType.CUDA)
    marks = [i for i, k in enumerate(ks) if "spin" in k[2].lower()]
    if marks:
        ks = ks[marks[-1] + 1:]
    ticks = max(dw.ticks_replayed, 1)
    busy, cur_s, cur_e = 0.0, None, None
    for s, e, _ in ks:
        if cur_e is None or s > cur_e:
            if cur_e is not None:
                busy += cur_e - cur_s
            cur_s, cur_e = s, e
        else:
            cur_e = max(cur_e, e)
    if cur_e is not None:
        busy += cur_e - cur_s
    span = ks[-1][1] - ks[0][0] if ks else 0.0
    agg = collections.defaultdict(lambda: [0, 0.0])
    for s, e, nm in ks:
        agg[nm[:100]][0] += 1
        agg[nm[:100]][1] += e - s
    total = sum(a[1] for a in agg.values()) or 1.0
    print(f"batch {B}: {ticks} ticks, {bt.n_tokens} tokens; per tick: span {span / ticks:.1f} us, "
          f"busy {busy / ticks:.1f} us, {len(ks) / ticks:.1f} kernels")
    print(f"  {'launches':>8} {'us/tick':>9} {'share':>6} {'us/launch':>10}  kernel")
    for nm, (c, t) in sorted(agg.items(), key=lambda x: -x[1][1]):
        print(f"  {c:8d} {t / ticks:9.2f} {100 * t / total:5.1f}% {t / c:10.2f}  {nm}")
    # the eight attention launches of a tick: prelude x2, core x4, coda x2
    keys = dw.keys.tolist()
    rb = 2 * eng._row_bytes
    per_layer = [keys[0]] * cfg.n_prelude + [keys[1]] * cfg.n_core + [keys[2]] * cfg.n_coda
    tc = [e - s for s, e, nm in ks if "wave_tc_kernel" in nm or "wave_decode_kernel" in nm]
    n_att = len(per_layer)
    if tc and len(tc) % n_att == 0:
        print("  attention launch (position in the tick): mean us, K/V MB, GB/s")
        for i in range(n_att):
            m = sum(tc[i::n_att]) / len(tc[i::n_att])
            mb = per_layer[i] / ticks * rb / 1e6
            print(f"    {i}: {m:8.2f} us {mb:8.1f} MB {mb / 1e3 / (m * 1e-6):7.0f}")


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--batch", type=int, nargs="+", default=[8, 64])
    ap.add_argument("--new-tokens", type=int, default=32)
    ap.add_argument("--t-draft", type=int, default=2)
    args = ap.parse_args()
    if not torch.cuda.is_available():
        raise SystemExit("tick_profile needs a CUDA device")
    for B in args.batch:
        profile_batch(B, args.new_tokens, args.t_draft)
        torch.cuda.empty_cache()


if __name__ == "__main__":
    main()
