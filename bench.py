#!/usr/bin/env python
"""Benchmark: wavefront decode / verify attention on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl wfd|reference]
                    [--workload cfg2|cfg3|cfg4] [--kernel -1|0|1] [--batch B]
                    [--t-draft D] [--scheduler device|host] [--alpha A] [--new-tokens T]

Default workload: one step = one wavefront decode tick of
the isolated attention op: B=8 sequences x R=8 loop-depth slots, Hq=16 / Hkv=4
(GQA 4:1), Dh=128, bf16; slot r holds L_r = 4096 - r positions and gets one
query (the new row is appended and attended in the same step).  Q, K, V ~
N(0,1) from torch CPU seed 1 (draw order q, K, V), synthetic.  The KV working
set (537 MB) is larger than L2 (126 MB), so no L2 flush is needed.

--workload cfg3: verify + commit.  B=32 (or --batch),
R=8, Hq=32 / Hkv=8, Dh=128, bf16; slot r holds 8192 - r positions and gets an
8-row causal draft window; a step is the fused append + verify attention and
the accept commit (per-sequence accepted lengths U{0..8}, seed 3).  Q, K, V
~ N(0,1) drawn on the device from seed 2 (8.6 GB of KV does not fit a CPU draw).

--workload cfg4: end-to-end greedy wavefront decoding of
the random-init looped LM (vocab 50304, d 1536, 24 x 64 heads, SwiGLU 4096,
prelude 2 / core 4 x R=8 / coda 2, bf16) through the engine and the device
scheduler; 64 prompts of 1024 uniform token ids (seed 4) split over the ranks
(strong scaling; --batch sets the total), 256 new tokens, T_draft 2 (--t-draft).
One step = one generation; value = committed tokens / decode time (CUDA events,
max over ranks), e2e includes the prefill and the host copies.

value : algorithmic KV-read GB/s with every input resident in HBM (one CUDA
        graph per step), max time over ranks.
e2e   : the same metric through the public Python / C-ABI call with host
        buffers: every step copies q, the new K/V rows and the item table from
        pinned host memory and reads the output back; the uploads of step i + 1
        run on a copy stream while step i computes (double-buffered inputs).
Multi-GPU (torchrun): every rank runs its own independent batch (weak scaling);
the only collectives are the timing max and a final counter gather.
cfg4_e2e (default line only, --no-cfg4-e2e skips it): a short config-4
generation (64 new tokens, T_draft 2, the 64 sequences sharded over the ranks)
timed after the cfg2 measurement, so a 1 -> N GPU series of default runs also
records end-to-end strong scaling.
--impl reference: the reference's CPU path (write_tokens + gather_pack + SDPA
varlen loop, restated in oracle/cpu_path.py) on all host cores (whatever
OMP_NUM_THREADS says), rank 0 only, with the repo arm's config.
"""
from __future__ import annotations

import argparse
import dataclasses
import datetime
import json
import os
import pathlib
import statistics
import subprocess
import sys
import time

ROOT = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "WFD decode tokens/s/GPU; wavefront-attn KV read GB/s vs HBM peak"
UNIT = "GB/s"
FALLBACK_HBM_GBS = 6650.0

CFG2 = dict(B=8, R=8, H=16, Hkv=4, Dh=128, S=4096, seed=1)
GRAPH_STEPS = 50  # attention workloads: consecutive steps captured per CUDA graph
CFG3 = dict(B=32, R=8, H=32, Hkv=8, Dh=128, L0=8192, W=8, seed=2, accept_seed=3)
CFG4 = dict(B=64, L=1024, new=256, seed=4, model_seed=0, emu_seed=5)
# the attention op of one config-4 R tick: 64 sequences x 8 loop depths, MHA 24 x 64,
# slot r holding 1100 - r positions (1024-token prompts plus ~76 generated tokens)
CFG4A = dict(B=64, R=8, H=24, Hkv=24, Dh=64, S=1100, seed=4)
# config 5 as stated needs 9.1 GB of KV per sequence (128 / GPU: 1.17 TB); the stated
# reduction measured here: one layer's 16 loop-depth slots, 64 sequences per GPU (137 GB)
CFG5 = dict(B=64, R=16, H=32, Hkv=8, Dh=128, L0=32768, W=8, seed=5, alpha=0.8)
# config 5 with the reference's KV sharing kv_budget_s = 1 (parcae_blocks.py:77-81): every
# loop depth of a layer shares one slot, so a sequence holds 8 slots (2 prelude + 4 core +
# 2 coda) of 32768 positions, 1.07 GB, and 128 sequences per GPU fit (137 GB); the
# tokens a sequence has in flight on a layer form one 8-row window on that slot
CFG5S1 = dict(CFG5, B=128, R=1, kv_budget=1)

# DRAM traffic per launch (dram__bytes_read.sum + dram__bytes_write.sum) of the
# timed attention kernel, from one ncu capture of that kernel on the same
# workload.  cfg3 was captured at batch 8, cfg4attn at batch 16 and cfg5 at batch
# 2, scaled by the units processed (x4 to batch 32, x4 to batch 64, x32 to batch 64).
NCU_TRAFFIC_BYTES = {("cfg2", "cuda_core"): 537_539_072 + 5_969_920,
                     ("cfg2", "tc"): 538_102_272 + 4_250_368,
                     ("cfg3", "tc"): (2_158_536_192 + 9_401_600) * 4,
                     ("cfg4attn", "tc"): (866_308_864 + 4_023_040) * 4,
                     ("cfg5", "tc"): (4_314_130_176 + 6_834_176) * 32}


def ncu_traffic(workload: str, tc: bool, c: dict):
    """Captured DRAM bytes per launch, scaled to this run's batch (every sequence
    reads the same bytes), or None when no capture covers the kernel."""
    t = NCU_TRAFFIC_BYTES.get((workload, "tc" if tc else "cuda_core"))
    if t is None:
        return None
    base = {"cfg2": CFG2, "cfg3": CFG3, "cfg4attn": CFG4A, "cfg5": CFG5}[workload]
    if workload == "cfg5" and c.get("kv_budget") == 1:
        return None  # captured for the 16-slot layout only
    return int(t * c["B"] / base["B"])


def init_dist(dev, timeout_s: int):
    """NCCL process group for this rank; NCCL's start-up banner (printed on fd 1
    when the environment enables it) goes to stderr so rank 0's stdout stays
    the one JSON line."""
    import torch.distributed as dist
    sys.stdout.flush()
    saved = os.dup(1)
    os.dup2(2, 1)
    try:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=timeout_s), device_id=dev)
        dist.barrier(device_ids=[dev.index])
    finally:
        sys.stdout.flush()
        os.dup2(saved, 1)
        os.close(saved)


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["wfd", "reference"], default="wfd")
    ap.add_argument("--workload", choices=["cfg2", "cfg3", "cfg4", "cfg4attn", "cfg5", "cfg4tick", "prefill",
                                           "linear"],
                    default="cfg2",
                    help="cfg4tick: per-tick kernel breakdown of config 4 (diagnostic table, no JSON line); "
                         "prefill: the prompt kernel on one config-4 layer")
    ap.add_argument("--batch", type=int, default=None,
                    help="sequences per GPU (cfg2 / cfg3) or in total over all GPUs (cfg4); default: the config's")
    ap.add_argument("--t-draft", type=int, default=2, help="cfg4: draft depth T_draft")
    ap.add_argument("--new-tokens", type=int, default=None, help="cfg4: generated tokens per sequence")
    ap.add_argument("--alpha", type=float, default=None,
                    help="cfg4: emulated draft acceptance rate (default: greedy gold == draft); "
                         "cfg5: Bernoulli draft acceptance (default 0.8)")
    ap.add_argument("--scheduler", choices=["device", "host", "dtv"], default="device",
                    help="cfg4: wavefront with route / settle on the GPU (one graph per tick) or on the host, "
                         "or draft-then-verify (host)")
    ap.add_argument("--draft-length", type=int, default=8, help="cfg4 with --scheduler dtv: drafts per round")
    ap.add_argument("--kv-budget", type=int, default=0,
                    help="cfg4: KV-sharing budget s (core depth r keeps its K/V in slot r %% s); 0 = off; "
                         "cfg5: 1 = the kv_budget_s=1 layout (128 sequences per GPU, one slot per layer)")
    ap.add_argument("--batch-invariant", action="store_true",
                    help="cfg4 (device scheduler): fixed union capacities + batch-invariant attention "
                         "(bit-exact greedy equality with sequential decoding)")
    ap.add_argument("--cpu-seconds", type=float, default=15.0, help="CPU baseline sample budget")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-cfg4-e2e", action="store_true",
                    help="cfg2: skip the short config-4 end-to-end generation recorded beside the line")
    ap.add_argument("--kernel", type=int, default=-1, choices=[-1, 0, 1],
                    help="-1 library default, 0 CUDA-core decode kernel, 1 tcgen05 kernel")
    return ap.parse_args()


def measured_peak():
    p = ROOT / "MEASURED_PEAKS.json"
    try:
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def algorithmic_bytes(items, H, Hkv, Dh, elem=2):
    kv = sum((p0 + ql) for _, _, p0, ql, _ in items) * Hkv * Dh * elem * 2   # every key row read once per kv head
    rows = sum(it[3] for it in items)
    qo = 2 * rows * H * Dh * elem                                             # q in, out
    app = rows * Hkv * Dh * elem * 2                                          # appended K/V rows written
    return kv + qo + app, rows


# ---------------------------------------------------------------------------
# workloads
# ---------------------------------------------------------------------------
def cfg2_cpu_inputs(seed: int, batch: int | None = None):
    import torch
    c = dict(CFG2)
    if batch:
        c["B"] = batch
    g = torch.Generator().manual_seed(seed)
    q = torch.randn((c["B"], c["R"], c["H"], c["Dh"]), generator=g).to(torch.bfloat16)
    K = torch.randn((c["R"], c["B"], c["S"], c["Hkv"], c["Dh"]), generator=g).to(torch.bfloat16)
    V = torch.randn((c["R"], c["B"], c["S"], c["Hkv"], c["Dh"]), generator=g).to(torch.bfloat16)
    items = [[r, b, c["S"] - r - 1, 1, b * c["R"] + r] for b in range(c["B"]) for r in range(c["R"])]
    q = q.reshape(c["B"] * c["R"], c["H"], c["Dh"])
    kn = torch.stack([K[r, b, p] for r, b, p, _, _ in items])
    vn = torch.stack([V[r, b, p] for r, b, p, _, _ in items])
    return c, q, K, V, kn, vn, items


def cfg3_device_inputs(dev, seed: int, batch: int | None = None, base: dict | None = None,
                       alpha: float | None = None):
    """Verify-window workload (config 3; config 5 with base=CFG5): q, K, V ~ N(0,1)
    drawn on the device, per-sequence accepted lengths for the commit."""
    import torch
    c = dict(base or CFG3)
    if batch:
        c["B"] = batch
    if alpha is not None:
        c["alpha"] = alpha
    B, R, H, Hkv, Dh, L0, W = c["B"], c["R"], c["H"], c["Hkv"], c["Dh"], c["L0"], c["W"]
    g = torch.Generator(device=dev).manual_seed(seed)
    q = torch.randn((B, R, W, H, Dh), generator=g, device=dev, dtype=torch.bfloat16)
    K = torch.randn((R, B, L0 + W, Hkv, Dh), generator=g, device=dev, dtype=torch.bfloat16)
    V = torch.randn((R, B, L0 + W, Hkv, Dh), generator=g, device=dev, dtype=torch.bfloat16)
    items = [[r, b, L0 - r, W, (b * R + r) * W] for b in range(B) for r in range(R)]
    q = q.reshape(B * R * W, H, Dh)
    # the window rows are the rows already drawn at those positions, so every
    # repetition of the step appends identical data
    idx_r = torch.tensor([r for r, b, p, w, _ in items for j in range(w)], device=dev)
    idx_b = torch.tensor([b for r, b, p, w, _ in items for j in range(w)], device=dev)
    idx_p = torch.tensor([p + j for r, b, p, w, _ in items for j in range(w)], device=dev)
    kn = K[idx_r, idx_b, idx_p].contiguous()
    vn = V[idx_r, idx_b, idx_p].contiguous()
    if "alpha" in c:
        # config 5: Bernoulli(alpha) draft outcomes, seed 5; a sequence keeps the
        # drafts before its first rejection, in every depth slot
        ok = torch.rand((B, W), generator=torch.Generator().manual_seed(c["seed"])) < c["alpha"]
        lead = torch.cumprod(ok.int(), dim=1).sum(dim=1)
        acc_seq = [int(x) for x in lead]
    else:
        accept = torch.randint(0, 9, (32,), generator=torch.Generator().manual_seed(c["accept_seed"]))
        acc_seq = [int(accept[b % 32]) for b in range(B)]
    c["accepted"] = acc_seq
    acc_items = torch.tensor([acc_seq[b] for r, b, p, w, _ in items], dtype=torch.int32, device=dev)
    return c, q, K, V, kn, vn, items, acc_items


def decode_device_inputs(dev, c: dict, seed: int):
    """Single-row wavefront decode inputs drawn on the device: q (B*R, H, Dh), K / V
    (R, B, S + 8, Hkv, Dh) ~ N(0,1); slot r of each sequence appends its row at
    S - r - 1 (the row already drawn there, so repeated steps append identical
    data) and attends S - r keys."""
    import torch
    B, R, H, Hkv, Dh, S = c["B"], c["R"], c["H"], c["Hkv"], c["Dh"], c["S"]
    g = torch.Generator(device=dev).manual_seed(seed)
    q = torch.randn((B * R, H, Dh), generator=g, device=dev, dtype=torch.bfloat16)
    K = torch.randn((R, B, S + 8, Hkv, Dh), generator=g, device=dev, dtype=torch.bfloat16)
    V = torch.randn((R, B, S + 8, Hkv, Dh), generator=g, device=dev, dtype=torch.bfloat16)
    items = [[r, b, S - r - 1, 1, b * R + r] for b in range(B) for r in range(R)]
    ir = torch.tensor([it[0] for it in items], device=dev)
    ib = torch.tensor([it[1] for it in items], device=dev)
    ip = torch.tensor([it[2] for it in items], device=dev)
    return c, q, K, V, K[ir, ib, ip].contiguous(), V[ir, ib, ip].contiguous(), items


class ClockSampler:
    """Clocks / throttle reasons sampled during the timed region: the nvidia-smi
    clocks line (every 20 ms) and, in-process, NVML every ~1 ms (a timed region of
    a few ms would otherwise hold one sample or none)."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None

    def _poll(self):
        import pynvml
        try:
            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByIndex(self.gpu)
            mx = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
            get_reasons = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                pynvml.nvmlDeviceGetCurrentClocksThrottleReasons
        except Exception:
            self._ready.set()
            return
        self._ready.set()
        self._go.wait()  # NVML is up; samples only from the start of the timed region
        try:
            while not self._stop.is_set():
                try:
                    self.nvml_rows.append(dict(sm=float(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)),
                                               max=mx, power=pynvml.nvmlDeviceGetPowerUsage(h) / 1000.0,
                                               bits=int(get_reasons(h))))
                except Exception:
                    break
                self._stop.wait(0.001)
        finally:
            try:
                pynvml.nvmlShutdown()
            except Exception:
                pass

    def __enter__(self):
        import threading
        self.first = []
        self.nvml_rows = []
        self._stop, self._ready, self._go = threading.Event(), threading.Event(), threading.Event()
        self._thread = threading.Thread(target=self._poll, daemon=True)
        self._thread.start()
        self._ready.wait(timeout=10.0)
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "20", "-i", str(self.gpu)], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
            self._go.set()
            return self
        # the timed region starts once sampling is live (nvidia-smi takes a
        # moment to print its first line)
        import select
        r, _, _ = select.select([self.proc.stdout], [], [], 10.0)
        if r:
            self.first = [self.proc.stdout.readline()]
        self._go.set()  # NVML samples from here on: the timed region starts next
        return self

    def __exit__(self, *exc):
        self._stop.set()
        self._go.set()
        self._thread.join(timeout=5)
        self.lines = []
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()
                out = ""
            self.lines = [ln for ln in self.first + (out or "").splitlines() if ln.strip()]

    def summary(self):
        rows = []
        for ln in getattr(self, "lines", []):
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                rows.append(dict(sm=float(f[1]), max=float(f[2]), power=float(f[3]), hw=f[5], hwt=f[6], swt=f[7],
                                 pcap=f[8]))
            except ValueError:
                continue
        reasons = set()
        for r in rows:
            for key, name in (("hw", "hw_slowdown"), ("hwt", "hw_thermal_slowdown"), ("swt", "sw_thermal_slowdown"),
                              ("pcap", "sw_power_cap")):
                if r[key].lower().startswith("active"):
                    reasons.add(name)
        # NVML reason bits: sw power cap 0x4, hw slowdown 0x8, sw thermal 0x20, hw thermal 0x40
        nv = getattr(self, "nvml_rows", [])
        for r in nv:
            for bit, name in ((0x4, "sw_power_cap"), (0x8, "hw_slowdown"), (0x20, "sw_thermal_slowdown"),
                              (0x40, "hw_thermal_slowdown")):
                if r["bits"] & bit:
                    reasons.add(name)
        allr = rows + nv
        if not allr:
            return None
        return {"sm_mhz": statistics.median(r["sm"] for r in allr), "sm_max_mhz": max(r["max"] for r in allr),
                "reasons": sorted(reasons), "samples": len(allr), "samples_nvidia_smi": len(rows),
                "samples_nvml": len(nv), "power_w_max": max(r["power"] for r in allr)}


def cpu_baseline(q, K, V, kn, vn, items, budget_s: float, warmup: int = 1, steps: int | None = None,
                 label: str = "cfg2 decode"):
    """Time the reference's CPU path (oracle/cpu_path.py) on a bounded sample."""
    import torch
    from oracle import cpu_path
    H, Dh = q.shape[1], q.shape[2]
    Hkv = K.shape[3]
    t0 = time.perf_counter()
    cpu_path.wave_step(K, V, q, kn, vn, items)
    first = time.perf_counter() - t0
    sample = items
    if steps is None:
        if first > 2.0:  # slow host: time a proportional subset of the rows
            sample = items[:max(1, int(len(items) * 2.0 / first))]
        n = max(1, int(budget_s / max(first * len(sample) / len(items), 1e-3)))
    else:
        # fixed step count (reference arm): shrink the rows per step so that
        # warm-up + timed steps stay within the budget
        per_step = budget_s / max(1, steps + warmup)
        if first > per_step:
            sample = items[:max(1, int(len(items) * per_step / first))]
        n = steps
    for _ in range(max(0, warmup - 1)):
        cpu_path.wave_step(K, V, q, kn, vn, sample)
    t0 = time.perf_counter()
    for _ in range(n):
        cpu_path.wave_step(K, V, q, kn, vn, sample)
    dt = (time.perf_counter() - t0) / n
    nbytes, rows = algorithmic_bytes(sample, H, Hkv, Dh)
    return {"value": nbytes / dt / 1e9, "unit": UNIT, "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{len(sample)} of {len(items)} {label} items per step (write_tokens + gather_pack + "
                      f"SDPA varlen loop, bf16, torch CPU), {n} steps, {dt * 1e3:.1f} ms/step",
            "ms_per_step": dt * 1e3, "host_cpu_count": os.cpu_count()}, n, dt


def cfg3_cpu_sample(K, V, q, kn, vn, items, n_items: int = 4):
    """A few cfg3 items copied to host memory for the CPU baseline."""
    import torch
    sel = items[:n_items]
    Hkv, Dh = K.shape[3], K.shape[4]
    S = K.shape[2]
    Kc = torch.empty((1, len(sel), S, Hkv, Dh), dtype=K.dtype)
    Vc = torch.empty_like(Kc)
    qs, ks, vs, its = [], [], [], []
    row = 0
    for i, (r, b, p0, ql, r0) in enumerate(sel):
        Kc[0, i] = K[r, b].cpu()
        Vc[0, i] = V[r, b].cpu()
        qs.append(q[r0:r0 + ql].cpu())
        ks.append(kn[r0:r0 + ql].cpu())
        vs.append(vn[r0:r0 + ql].cpu())
        its.append([0, i, p0, ql, row])
        row += ql
    return Kc, Vc, torch.cat(qs), torch.cat(ks), torch.cat(vs), its


# bounded CPU sample of config 4: the first B of the 64 sequences (prompt K / V drawn,
# not computed), decode rate = the tokens of a `long` generation minus those of a
# `short` one over the difference of their decode times (pipeline fill cancels)
CFG4_CPU = dict(B=16, short=2, long=6)


def cfg4_cpu_baseline(t_draft: int, kv_budget: int, alpha, steps: int = 1, budget_s: float = 150.0):
    """The reference's decode loop on the host cores: oracle/cpu_path.LoopedBlocksCPU
    (write_tokens + gather_pack + SDPA varlen loop per layer, bf16 torch CPU)
    driven by the package's host wavefront scheduler, on CFG4_CPU's sample of the
    config-4 workload.  One step = one (short, long) pair of generations."""
    import torch

    import __graft_entry__
    __graft_entry__.load_package()
    from oracle import cpu_path
    from wavefront_decoding_b200 import scheduler as sch
    from wavefront_decoding_b200.looped_lm import CONFIG4

    cfg = CONFIG4
    dims = {k: getattr(cfg, k) for k in ("vocab", "d_model", "n_heads", "n_kv_heads", "head_dim", "d_ff",
                                         "n_prelude", "n_core", "n_coda", "T_total", "norm_eps", "rope_theta",
                                         "rope_style")}
    dims["kv_budget_s"] = kv_budget
    B, L, short, long_ = CFG4_CPU["B"], CFG4["L"], CFG4_CPU["short"], CFG4_CPU["long"]
    prompts = torch.randint(0, cfg.vocab, (CFG4["B"], L),
                            generator=torch.Generator().manual_seed(CFG4["seed"]))[:B].contiguous()
    W = cpu_path.random_weights(dims, CFG4["model_seed"])
    blocks = cpu_path.LoopedBlocksCPU(W, dims, B, L + long_ + 2 * cfg.T_total + 8, synthetic_prompt=True,
                                      seed=CFG4["seed"])
    policy = sch.SsdPolicy(cfg.T_total, t_draft)

    def generate(n):
        emus = None
        if alpha is not None:
            emus = [sch.EmulatedAcceptance(alpha, seed=CFG4["emu_seed"] * 1_000_003 + b) for b in range(B)]
        bt = sch.generate_wavefront_batch(blocks, prompts, n, policy, emus)
        prop = sum(t.n_drafts_proposed for t in bt.per_seq)
        acc = sum(t.n_drafts_accepted for t in bt.per_seq)
        return bt.n_tokens, bt.walltime_s - bt.prefill_s, prop, acc

    generate(short)                                   # warm-up
    d_tok = d_s = prop = acc = 0
    n = 0
    t_start = time.perf_counter()
    while n < max(1, steps):
        a = generate(short)
        b = generate(long_)
        d_tok += b[0] - a[0]
        d_s += b[1] - a[1]
        prop += b[2]
        acc += b[3]
        n += 1
        if time.perf_counter() - t_start > budget_s:
            break
    rate = d_tok / d_s
    return {"value": rate, "unit": "tokens/s", "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{B} of the {CFG4['B']} config-4 sequences, prompt {L} (prompt K/V drawn at random, the "
                      f"prompt pass is outside the decode region), wavefront T_draft {t_draft}: decode tokens of "
                      f"a {long_}-token generation minus a {short}-token one over the decode-time difference, "
                      f"{n} pair(s); per layer write_tokens + gather_pack + SDPA varlen loop, bf16 torch CPU",
            "acceptance_rate": acc / prop if prop else None, "steps": n,
            "ms_per_token_step": 1e3 * d_s / max(1, d_tok) * B, "host_cpu_count": os.cpu_count()}


def host_threads() -> int:
    """Every core this process may run on, whatever OMP_NUM_THREADS says (torchrun
    sets it to 1 per rank): the CPU baseline gets the whole host."""
    import torch
    try:
        n = len(os.sched_getaffinity(0))
    except AttributeError:
        n = os.cpu_count() or 1
    torch.set_num_threads(max(1, n))
    return torch.get_num_threads()


def run_reference(args):
    """--impl reference: the reference's CPU path on all host cores, rank 0 only
    (the other ranks exit without work)."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    host_threads()
    if args.workload == "cfg4":
        base = cfg4_cpu_baseline(args.t_draft, args.kv_budget, args.alpha, steps=max(1, args.steps))
        line = {"impl": "reference", "metric": METRIC, "value": base["value"], "unit": "tokens/s",
                "n_gpus": args.gpus, "steps": base["steps"], "warmup": 1,
                "ms_per_step": base["ms_per_token_step"], "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None, "dtype": "bf16", "data": "synthetic (random-init weights, uniform random "
                "prompt ids)", "config": cfg4_config(args, world),
                "acceptance_rate": base["acceptance_rate"],
                "cpu_baseline": {k: base[k] for k in ("value", "unit", "cores", "kind", "sample")},
                "e2e": {"value": base["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return
    if args.workload == "cfg2":
        c, q, K, V, kn, vn, items = cfg2_cpu_inputs(CFG2["seed"], args.batch)
        full_items = items
        label = "cfg2 decode"
    else:
        import torch
        dev = torch.device("cuda", 0) if torch.cuda.is_available() else None
        if dev is None:
            print(json.dumps({"impl": "reference", "unavailable": "cfg3 inputs are drawn on the GPU"}))
            return
        if args.workload == "cfg4attn":
            c = dict(CFG4A, **({"B": args.batch} if args.batch else {}))
            c, q, K, V, kn, vn, items = decode_device_inputs(dev, c, c["seed"])
        else:
            base = CFG3 if args.workload == "cfg3" else (CFG5S1 if args.kv_budget == 1 else CFG5)
            c, q, K, V, kn, vn, items, _ = cfg3_device_inputs(dev, base["seed"], args.batch, base,
                                                              args.alpha if args.workload == "cfg5" else None)
        full_items = items
        K, V, q, kn, vn, items = cfg3_cpu_sample(K, V, q, kn, vn, items)
        label = f"{args.workload} verify"
    base, n, dt = cpu_baseline(q, K, V, kn, vn, items, 90.0, warmup=max(1, args.warmup), steps=max(1, args.steps),
                               label=label)
    _, rows = algorithmic_bytes(full_items, c["H"], c["Hkv"], c["Dh"])
    line = {"impl": "reference", "metric": METRIC, "value": base["value"], "unit": UNIT, "n_gpus": args.gpus,
            "steps": n, "warmup": args.warmup, "ms_per_step": base["ms_per_step"], "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": workload_config(args.workload, c, world, rows),
            "cpu_baseline": {k: base[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": base["value"], "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def workload_config(name, c, world, rows=None):
    if name == "cfg2":
        d = {"workload": "cfg2_wavefront_decode_attention", "batch_per_gpu": c["B"], "slots": c["R"],
             "n_heads": c["H"], "n_kv_heads": c["Hkv"], "head_dim": c["Dh"], "slot_len": "4096-r",
             "l2": "KV working set 537 MB > 126 MB L2, no flush"}
    elif name == "cfg4attn":
        d = {"workload": "cfg4_tick_attention (the wavefront decode attention of one config-4 R tick)",
             "batch_per_gpu": c["B"], "slots": c["R"], "n_heads": c["H"], "n_kv_heads": c["Hkv"],
             "head_dim": c["Dh"], "slot_len": f"{c['S']}-r", "l2": "KV working set 3.5 GB > L2, no flush"}
    elif name == "cfg3":
        d = {"workload": "cfg3_wavefront_verify_attention_plus_commit", "batch_per_gpu": c["B"], "slots": c["R"],
             "n_heads": c["H"], "n_kv_heads": c["Hkv"], "head_dim": c["Dh"], "slot_len": "8192-r + 8-row window",
             "window": c["W"], "l2": "KV working set > 126 MB L2, no flush"}
    elif c.get("kv_budget") == 1:
        d = {"workload": "cfg5_long_context_verify_plus_commit with KV sharing kv_budget_s=1 (every loop depth "
                         "of a layer on one slot: 8 slots of 32768 positions per sequence, 137 GB for 128 "
                         "sequences per GPU; the timed step is one layer: one 8-row window per sequence)",
             "batch_per_gpu": c["B"], "slots": c["R"], "n_heads": c["H"], "n_kv_heads": c["Hkv"],
             "head_dim": c["Dh"], "slot_len": "32768 + 8-row window", "window": c["W"],
             "acceptance": f"Bernoulli({c['alpha']}) seed {c['seed']}, accepted prefix per sequence",
             "l2": "KV working set 8.6 GB > L2, no flush"}
    else:
        d = {"workload": "cfg5_long_context_verify_plus_commit (stated reduction: one layer's 16 loop-depth "
                         "slots, 64 sequences per GPU; the full model needs 1.17 TB of KV per GPU)",
             "batch_per_gpu": c["B"], "slots": c["R"], "n_heads": c["H"], "n_kv_heads": c["Hkv"],
             "head_dim": c["Dh"], "slot_len": "32768-r + 8-row window", "window": c["W"],
             "acceptance": f"Bernoulli({c['alpha']}) seed {c['seed']}, accepted prefix per sequence",
             "l2": "KV working set 137 GB > L2, no flush"}
    d["parallelism"] = f"sequences sharded, {world} rank(s)"
    d["timing"] = f"CUDA graphs of up to {GRAPH_STEPS} consecutive steps"
    if rows is not None:
        d["rows_per_step_per_gpu"] = rows
    return d


def run_wfd(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        init_dist(dev, 300)

    import __graft_entry__
    __graft_entry__.load_package()
    from wavefront_decoding_b200 import attention as wa
    from wavefront_decoding_b200 import runtime as rt
    from wavefront_decoding_b200.kv_cache import SlotKVCache

    if args.workload == "cfg2":
        c, q, K, V, kn, vn, items = cfg2_cpu_inputs(CFG2["seed"] + rank, args.batch)
        qd, Kd, Vd, knd, vnd = q.to(dev), K.to(dev), V.to(dev), kn.to(dev), vn.to(dev)
        acc = None
        max_q = 1
    elif args.workload == "cfg4attn":
        c = dict(CFG4A)
        if args.batch:
            c["B"] = args.batch
        c, qd, Kd, Vd, knd, vnd, items = decode_device_inputs(dev, c, c["seed"] + rank)
        acc = None
        max_q = 1
        q = kn = vn = K = V = None
    else:
        base = CFG3 if args.workload == "cfg3" else (CFG5S1 if args.kv_budget == 1 else CFG5)
        c, qd, Kd, Vd, knd, vnd, items, acc = cfg3_device_inputs(dev, base["seed"] + rank, args.batch, base,
                                                                 args.alpha if args.workload == "cfg5" else None)
        max_q = c["W"]
        q = kn = vn = K = V = None
    H, Hkv, Dh = c["H"], c["Hkv"], c["Dh"]
    nbytes, rows = algorithmic_bytes(items, H, Hkv, Dh)
    items_t = torch.tensor(items, dtype=torch.int32)
    itd = items_t.to(dev)
    # the cache object owns the slot lengths; its K / V are the workload's tensors
    cache = SlotKVCache.wrap(Kd, Vd)
    out = torch.empty_like(qd)
    rt.reserve_workspace(dev, len(items), Dh)
    rt.error_word(dev)
    acc_rows = torch.empty((qd.shape[0],), dtype=torch.int32, device=dev)
    acc_cnt = torch.empty((len(items),), dtype=torch.int32, device=dev)

    def step():
        wa.wave_attn(qd, knd, vnd, Kd, Vd, itd, max_q, lens=cache.lens, out=out, kernel=args.kernel)
        if acc is not None:
            cache.commit_window(itd, accept_len=acc, n_rows=qd.shape[0], out=(acc_rows, acc_cnt))

    # warm up eagerly, then capture one step
    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()
    rt.read_device_error(dev)
    # the K timed steps run as replays of graphs of up to GRAPH_STEPS consecutive
    # steps (one replay per step would add a graph launch gap to every step)
    def capture(n):
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                for _ in range(n):
                    step()
        torch.cuda.current_stream().wait_stream(s)
        return g

    per = max(1, min(GRAPH_STEPS, args.steps))
    g_full = capture(per)
    g_rest = capture(args.steps % per) if args.steps % per else None
    plan = [g_full] * (args.steps // per) + ([g_rest] if g_rest is not None else [])
    g_full.replay()
    torch.cuda.synchronize()

    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier(device_ids=[local])
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        # the W warm-up steps run right before the timed ones, with no host wait in
        # between: the timed region starts on a busy GPU, not one idle since set-up
        for _ in range(max(1, -(-args.warmup // per))):
            g_full.replay()
        ev0.record()
        for g in plan:
            g.replay()
        ev1.record()
        torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1) / args.steps
    if world > 1:
        dist.barrier(device_ids=[local])
    rt.read_device_error(dev)

    # ---- e2e: the public API call with host buffers every step.  Each step's
    # inputs (q, the new K / V rows, the item table) sit packed in one pinned host
    # buffer and go up in one copy on a copy stream while the previous step
    # computes (two device copies of the packed inputs and of the output); the
    # output is read back to pinned host memory right after its step; every copy
    # of every step lies inside the timed region.
    parts = [qd, knd, vnd, items_t]
    offs, total_b = [], 0
    for t in parts:
        offs.append(total_b)
        total_b += (t.numel() * t.element_size() + 255) // 256 * 256
    stage_h = torch.empty(total_b, dtype=torch.uint8).pin_memory()
    for t, o in zip(parts, offs):
        nb = t.numel() * t.element_size()
        stage_h[o:o + nb].copy_(t.detach().cpu().contiguous().view(-1).view(torch.uint8))
    out_h = [torch.empty(out.shape, dtype=out.dtype).pin_memory() for _ in range(2)]
    h2d = sum(t.numel() * t.element_size() for t in parts)
    d2h = out_h[0].numel() * 2

    def device_views(buf):
        return tuple(buf[o:o + t.numel() * t.element_size()].view(t.dtype).view(t.shape) for t, o in zip(parts, offs))

    stage_d = [torch.empty(total_b, dtype=torch.uint8, device=dev) for _ in range(2)]
    bufs = [device_views(b) + (torch.empty_like(out),) for b in stage_d]
    comp = torch.cuda.current_stream(dev)
    copy = torch.cuda.Stream(dev)
    uploaded = [torch.cuda.Event(), torch.cuda.Event()]
    computed = [torch.cuda.Event(), torch.cuda.Event()]
    for e in computed:
        e.record(comp)

    def upload(i):
        with torch.cuda.stream(copy):
            copy.wait_event(computed[i % 2])          # the step that last used these buffers is done
            stage_d[i % 2].copy_(stage_h, non_blocking=True)
            uploaded[i % 2].record(copy)

    def compute(i):
        bq, bk, bv, bi, bo = bufs[i % 2]
        comp.wait_event(uploaded[i % 2])
        wa.wave_attn(bq, bk, bv, Kd, Vd, bi, max_q, lens=cache.lens, out=bo, kernel=args.kernel)
        if acc is not None:
            cache.commit_window(bi, accept_len=acc, n_rows=bq.shape[0], out=(acc_rows, acc_cnt))
        computed[i % 2].record(comp)
        with torch.cuda.stream(copy):
            copy.wait_event(computed[i % 2])
            out_h[i % 2].copy_(bo, non_blocking=True)

    def e2e_run(n):
        copy.wait_stream(comp)
        upload(0)
        for i in range(n):
            if i + 1 < n:
                upload(i + 1)
            compute(i)
        comp.wait_stream(copy)

    e2e_steps = args.steps if args.workload == "cfg2" else max(1, args.steps // 4)
    e2e_run(max(3, args.warmup))
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier(device_ids=[local])
    ev0.record()
    e2e_run(e2e_steps)
    ev1.record()
    torch.cuda.synchronize()
    ms_e2e = ev0.elapsed_time(ev1) / e2e_steps
    rt.read_device_error(dev)

    from wavefront_decoding_b200.parallel import reduce_over_ranks
    (ms, ms_e2e), (total_bytes, total_rows) = reduce_over_ranks([ms, ms_e2e], [nbytes, rows], dev)

    value = total_bytes / (ms * 1e-3) / 1e9
    value_e2e = total_bytes / (ms_e2e * 1e-3) / 1e9
    peak, peak_kind = measured_peak()
    achieved = nbytes / (ms * 1e-3) / 1e9    # per GPU, per launch of the step
    # bf16 / Dh=128 defaults to the tensor-core kernel: plan (with the window
    # append) + wave_tc_kernel per step; the CUDA-core kernel is plan + wave_decode_kernel
    tc = args.kernel != 0
    nqp = 16 if c["H"] // c["Hkv"] * max_q <= 16 else 32
    kernel_name = (f"wave_tc_kernel<{nqp}> (+ plan_kernel with the window append" if tc else
                   "wave_decode_kernel<bf16,128,4> (+ plan_kernel")
    kernel_name += (", commit_window_kernel" if acc is not None else "") + ", timed together)"
    launches_per_step = 2 + (1 if acc is not None else 0)
    line = None
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": workload_config(args.workload, c, world, rows),
            "wave_rows_per_s": total_rows / (ms * 1e-3),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_kind": peak_kind,
                         "traffic": ncu_traffic(args.workload, tc, c),
                         "algorithmic_bytes_per_launch": nbytes,
                         "kernel": kernel_name},
            "e2e": {"value": value_e2e, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "ms_per_step": ms_e2e},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clk.summary(),
        }
        if args.workload in ("cfg3", "cfg5"):
            flops = sum((p0 + ql) for _, _, p0, ql, _ in items) * Hkv * (H // Hkv) * max_q * Dh * 4
            line["tensor_tflops"] = flops / (ms * 1e-3) / 1e12
        if args.workload == "cfg5":
            # tokens one verify step commits per sequence: accepted drafts + the corrected / bonus token
            line["tokens_per_s"] = world * sum(a + 1 for a in c["accepted"]) / (ms * 1e-3)
            line["accepted_mean"] = sum(c["accepted"]) / len(c["accepted"])
    if args.workload == "cfg2" and not args.no_cfg4_e2e:
        del g
        torch.cuda.empty_cache()
        rec = cfg4_e2e_record(dev, world, rank)
        if rank == 0:
            line["cfg4_e2e"] = rec
    if world > 1:
        dist.barrier(device_ids=[local])
        g = None
        dist.destroy_process_group()
    if rank == 0:
        if world == 1 and not args.no_cpu_baseline:
            host_threads()
            if args.workload == "cfg2":
                base, _, _ = cpu_baseline(q, K, V, kn, vn, items, args.cpu_seconds)
            else:
                Kc, Vc, qc, knc, vnc, itc = cfg3_cpu_sample(Kd, Vd, qd, knd, vnd, items)
                base, _, _ = cpu_baseline(qc, Kc, Vc, knc, vnc, itc, args.cpu_seconds,
                                          label=f"{args.workload} verify")
            line["cpu_baseline"] = {k: base[k] for k in ("value", "unit", "cores", "kind", "sample")}
        else:
            line["cpu_baseline"] = None
        print(json.dumps(line), flush=True)


def cfg4_measure(dev, world: int, rank: int, *, batch: int, new: int, t_draft: int, scheduler: str = "device",
                 kv_budget: int = 0, batch_invariant: bool = False, alpha: float | None = None,
                 draft_length: int = 8, warmup: int = 1, steps: int = 1) -> dict:
    """Config 4 generation on this rank's shard of `batch` sequences: warm-up
    generations, then `steps` timed ones.  Device times are CUDA events; the
    results are reduced over ranks (max time, summed counts)."""
    import torch
    import torch.distributed as dist

    import __graft_entry__
    __graft_entry__.load_package()
    from wavefront_decoding_b200 import runtime as rt
    from wavefront_decoding_b200 import scheduler as sch
    from wavefront_decoding_b200.device_scheduler import DeviceWave
    from wavefront_decoding_b200.engine import WaveEngine
    from wavefront_decoding_b200.looped_lm import CONFIG4, LoopedLM
    from wavefront_decoding_b200.parallel import reduce_over_ranks, shard_range

    cfg = dataclasses.replace(CONFIG4, kv_budget_s=kv_budget)
    s0, s1 = shard_range(batch, world, rank)
    Bl = s1 - s0
    if Bl < 1:
        raise SystemExit(f"global batch {batch} leaves rank {rank} of {world} without sequences")
    L = CFG4["L"]
    prompts_all = torch.randint(0, cfg.vocab, (batch, L), generator=torch.Generator().manual_seed(CFG4["seed"]))
    prompts = prompts_all[s0:s1].contiguous().pin_memory()
    model = LoopedLM(cfg, seed=CFG4["model_seed"], dtype=torch.bfloat16, device=dev)
    eng = WaveEngine(model, Bl, L + new + 2 * cfg.T_total + 8)
    policy = sch.SsdPolicy(cfg.T_total, t_draft)
    dwave = DeviceWave(eng, new, policy, batch_invariant) if scheduler == "device" else None

    ev_all0, ev_dec0, ev_end = (torch.cuda.Event(enable_timing=True) for _ in range(3))

    def generate():
        emus = None
        if alpha is not None:
            emus = [sch.EmulatedAcceptance(alpha, seed=CFG4["emu_seed"] * 1_000_003 + s0 + b) for b in range(Bl)]
        orig = eng.prefill

        def prefill(ids):
            out = orig(ids)
            ev_dec0.record()
            return out

        eng.prefill = prefill
        try:
            ev_all0.record()
            if dwave is not None:
                bt = dwave.generate(prompts, emus)
            elif scheduler == "dtv":
                bt = sch.generate_dtv_batch(eng, prompts, new, policy, draft_length, emus)
            else:
                bt = sch.generate_wavefront_batch(eng, prompts, new, policy, emus)
            ev_end.record()
            torch.cuda.synchronize()
        finally:
            del eng.prefill
        return bt, ev_dec0.elapsed_time(ev_end), ev_all0.elapsed_time(ev_end)

    for _ in range(max(1, warmup)):
        generate()
    rt.read_device_error(dev)
    eng.reset_counters()
    if world > 1:
        dist.barrier(device_ids=[dev.index])
    torch.cuda.synchronize()
    dec_ms = all_ms = 0.0
    tokens = proposed = accepted = ticks = 0
    kv_dev = launches_dev = 0
    # libwfd kernels of one device tick: 3 scheduling kernels + the P / R / C bodies
    tick_launches = 3 + sum(eng._launches.values())
    with ClockSampler(dev.index) as clk:
        for _ in range(steps):
            bt, d_ms, a_ms = generate()
            dec_ms += d_ms
            all_ms += a_ms
            tokens += bt.n_tokens
            proposed += sum(t.n_drafts_proposed for t in bt.per_seq)
            accepted += sum(t.n_drafts_accepted for t in bt.per_seq)
            ticks += bt.n_r_calls
            if dwave is not None:
                kv_dev += dwave.kv_read_bytes
                launches_dev += tick_launches * dwave.ticks_replayed
    torch.cuda.synchronize()
    rt.read_device_error(dev)
    kv_bytes = eng.kv_read_bytes if dwave is None else kv_dev
    launches = eng.wfd_launches if dwave is None else launches_dev
    if world > 1:
        dist.barrier(device_ids=[dev.index])
    (dec_max, all_max), (tot_tokens, tot_prop, tot_acc, tot_kv) = reduce_over_ranks(
        [dec_ms, all_ms], [tokens, proposed, accepted, kv_bytes], dev)
    d2h = (eng.d2h_bytes // steps) if dwave is None else dwave.d2h_bytes
    return dict(cfg=cfg, Bl=Bl, dec_max=dec_max, all_max=all_max, tot_tokens=tot_tokens, tot_prop=tot_prop,
                tot_acc=tot_acc, kv_bytes=kv_bytes, dec_ms=dec_ms, ticks=ticks, launches=launches,
                h2d=prompts.numel() * prompts.element_size(), d2h=d2h, clocks=clk.summary())


# the short config-4 generation recorded next to the default (config-2) line, so
# the 1 -> N GPU runs also record end-to-end strong scaling
CFG4_E2E_NEW = 64


def cfg4_e2e_record(dev, world: int, rank: int) -> dict:
    r = cfg4_measure(dev, world, rank, batch=CFG4["B"], new=CFG4_E2E_NEW, t_draft=2, warmup=1, steps=1)
    return {"metric": "WFD decode tokens/s (config 4, end to end)", "unit": "tokens/s", "scaling": "strong",
            "value": r["tot_tokens"] / (r["dec_max"] * 1e-3),
            "e2e": r["tot_tokens"] / (r["all_max"] * 1e-3),
            "tokens_per_s_per_gpu": r["tot_tokens"] / (r["dec_max"] * 1e-3) / world,
            "ms_decode": r["dec_max"], "ms_with_prefill": r["all_max"],
            "acceptance_rate": (r["tot_acc"] / r["tot_prop"]) if r["tot_prop"] else None,
            "config": {"model": f"looped LM config 4 ({r['cfg'].n_params() / 1e6:.0f}M params), random init, "
                                "bf16", "global_batch": CFG4["B"],
                       "batch_per_gpu": r["Bl"], "prompt_len": CFG4["L"], "new_tokens": CFG4_E2E_NEW,
                       "T_draft": 2, "scheduler": "device", "parallelism": f"sequences sharded, {world} rank(s)"},
            "timing": "one timed generation after one warm-up, CUDA events, max over ranks; value = decode "
                      "region, e2e = with prompt upload and prefill"}


def cfg4_config(args, world: int) -> dict:
    from wavefront_decoding_b200.looped_lm import CONFIG4 as cfg
    Bg = args.batch or CFG4["B"]
    return {"workload": "cfg4_looped_lm_e2e_greedy_decode",
            "model": f"looped LM {cfg.n_params() / 1e6:.0f}M params: vocab {cfg.vocab}, d {cfg.d_model}, "
                     f"{cfg.n_heads}x{cfg.head_dim} heads (kv {cfg.n_kv_heads}), SwiGLU {cfg.d_ff}, "
                     f"prelude {cfg.n_prelude} / core {cfg.n_core} x R={cfg.T_total} / coda {cfg.n_coda}",
            "global_batch": Bg, "batch_per_gpu": Bg // world if Bg % world == 0 else f"{Bg // world}-{-(-Bg // world)}",
            "prompt_len": CFG4["L"], "new_tokens": args.new_tokens or CFG4["new"],
            "T_draft": args.t_draft, "scheduler": args.scheduler, "batch_invariant": args.batch_invariant,
            "draft_length": args.draft_length if args.scheduler == "dtv" else None,
            "kv_budget_s": args.kv_budget,
            "acceptance": "greedy gold == draft" if args.alpha is None else f"emulated Bernoulli({args.alpha})",
            "parallelism": f"sequences sharded, {world} rank(s), no collective on the hot path",
            "timing": "decode region per generation, CUDA events, max over ranks; KV working set > L2, no flush"}


def run_cfg4(args):
    """Config 4: end-to-end greedy wavefront decoding of the looped LM (random
    init, bf16) through the engine and scheduler; one step = one generation of
    `new` tokens for this rank's sequences (prefill included in e2e only)."""
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        init_dist(dev, 600)
    Bg = args.batch or CFG4["B"]
    new = args.new_tokens or CFG4["new"]
    r = cfg4_measure(dev, world, rank, batch=Bg, new=new, t_draft=args.t_draft, scheduler=args.scheduler,
                     kv_budget=args.kv_budget, batch_invariant=args.batch_invariant, alpha=args.alpha,
                     draft_length=args.draft_length, warmup=args.warmup, steps=args.steps)
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    if rank != 0:
        return
    cfg, Bl = r["cfg"], r["Bl"]
    peak, peak_kind = measured_peak()
    value = r["tot_tokens"] / (r["dec_max"] * 1e-3)
    kv_gbs = r["kv_bytes"] / (r["dec_ms"] * 1e-3) / 1e9      # rank 0's attention KV reads over its decode time
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": max(1, args.warmup), "ms_per_step": r["dec_max"] / args.steps, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic (random-init weights, "
        "uniform random prompt ids)",
        "config": cfg4_config(args, world),
        "tokens_per_s_per_gpu": value / world,
        "acceptance_rate": (r["tot_acc"] / r["tot_prop"]) if r["tot_prop"] else None,
        "ticks_per_generation": r["ticks"] / args.steps,
        "roofline": {"bound": "hbm", "achieved": kv_gbs, "peak": peak, "unit": "GB/s", "frac": kv_gbs / peak,
                     "peak_kind": peak_kind, "traffic": None,
                     "note": "attention K/V bytes read by live rows over the whole decode wall time "
                             "(GEMMs, host scheduling and launches included in the time)"},
        "e2e": {"value": r["tot_tokens"] / (r["all_max"] * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": r["h2d"],
                "d2h_bytes_per_step": r["d2h"], "ms_per_step": r["all_max"] / args.steps,
                "includes": "prefill, prompt upload from pinned host memory, per-tick greedy-id read-back"},
        "gpu_launches": r["launches"],
        "clocks": r["clocks"],
        "cpu_baseline": None,
    }
    if world == 1 and not args.no_cpu_baseline:
        host_threads()
        base = cfg4_cpu_baseline(args.t_draft, args.kv_budget, args.alpha)
        line["cpu_baseline"] = {k: base[k] for k in ("value", "unit", "cores", "kind", "sample")}
    print(json.dumps(line), flush=True)


def run_prefill(args):
    """--workload prefill: the prompt pass's causal attention of one config-4 layer
    (B = 64 (--batch), L = 1024, MHA 24 x 64, bf16) on the tcgen05 prompt kernel
    K7; value = causal TFLOP/s (4 * B * H * Dh * L^2 / 2 per launch), roofline
    against the measured bf16 tensor peak (burst)."""
    import torch

    import __graft_entry__
    __graft_entry__.load_package()
    from wavefront_decoding_b200 import attention as wa
    from wavefront_decoding_b200 import runtime as rt

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    B, L, H, Dh = args.batch or 64, CFG4["L"], 24, 64
    g = torch.Generator(device=dev).manual_seed(CFG4["seed"])
    q = torch.randn((B, L, H, Dh), generator=g, device=dev, dtype=torch.bfloat16)
    k = torch.randn((B, L, H, Dh), generator=g, device=dev, dtype=torch.bfloat16)
    v = torch.randn((B, L, H, Dh), generator=g, device=dev, dtype=torch.bfloat16)
    out = torch.empty_like(q)
    for _ in range(max(3, args.warmup)):
        wa.attn_prefill(q, k, v, causal=True, out=out)
    torch.cuda.synchronize()
    rt.read_device_error(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(0) as clk:
        ev0.record()
        for _ in range(args.steps):
            wa.attn_prefill(q, k, v, causal=True, out=out)
        ev1.record()
        torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1) / args.steps
    rt.read_device_error(dev)
    flops = 4.0 * B * H * Dh * L * L / 2
    tf = flops / (ms * 1e-3) / 1e12
    try:
        peak, kind = float(json.loads((ROOT / "MEASURED_PEAKS.json").read_text())["bf16_tflops"]), "measured"
    except Exception:
        peak, kind = 1590.0, "fallback"
    print(json.dumps({"metric": "prompt attention TFLOP/s (config-4 layer, causal)", "value": tf, "unit": "TFLOP/s",
                      "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
                      "higher_is_better": True, "dtype": "bf16", "data": "synthetic",
                      "config": {"workload": "prefill_causal_attention", "batch": B, "prompt_len": L, "n_heads": H,
                                 "head_dim": Dh},
                      "roofline": {"bound": "tensor", "achieved": tf, "peak": peak, "unit": "TFLOP/s",
                                   "frac": tf / peak, "peak_kind": kind},
                      "gpu_launches": args.steps, "clocks": clk.summary()}), flush=True)


def run_linear(args):
    """--workload linear: the four linear layers of config-4 blocks on the fused
    skinny-linear kernel K8 (wfd_linear: RMSNorm + QKV + RoPE, o_proj + residual,
    RMSNorm + gate/up + SwiGLU, down + residual), --batch rows (default 8), eight
    layers with their own weights per step (453 MB, larger than L2); value = weight
    bytes streamed per second (HBM roofline).  The same chain on RMSNorm + cuBLAS +
    the element-wise kernels is timed beside it (`unfused`), and the chain the bf16
    engine runs, cuBLAS with the RMSNorm folded into the weights and its row scale
    applied by the RoPE split / SwiGLU kernels (`folded`)."""
    import torch

    import __graft_entry__
    __graft_entry__.load_package()
    from wavefront_decoding_b200 import fused
    from wavefront_decoding_b200 import runtime as rt
    from wavefront_decoding_b200.looped_lm import CONFIG4 as cfg

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    n, d, dff, H, Dh, layers = args.batch or 8, cfg.d_model, cfg.d_ff, cfg.n_heads, cfg.head_dim, 8
    g = torch.Generator(device=dev).manual_seed(CFG4["model_seed"])

    def w(*shape):
        return (torch.randn(shape, generator=g, device=dev) * 0.02).to(torch.bfloat16)

    ones = torch.ones(d, dtype=torch.bfloat16, device=dev)
    W = [dict(qkv=w(d, 3 * H * Dh), o=w(H * Dh, d), gu=w(d, 2 * dff), dn=w(dff, d)) for _ in range(layers)]
    for blk in W:
        blk["qkv_f"] = fused.fold_norm(blk["qkv"], ones)
        blk["gu_n"] = fused.fold_norm(blk["gu"], ones)
        blk["gu_f"] = fused.interleave_gate_up(blk["gu_n"])
    S = 4096
    inv = 1.0 / (cfg.rope_theta ** (torch.arange(0, Dh, 2, dtype=torch.float64) / Dh))
    ang = torch.outer(torch.arange(S, dtype=torch.float64), inv)
    cos, sin = ang.cos().float().to(dev), ang.sin().float().to(dev)
    x = torch.randn((n, d), generator=g, device=dev).to(torch.bfloat16)
    attn = torch.randn((n, H * Dh), generator=g, device=dev).to(torch.bfloat16)
    pos = torch.randint(0, S, (n,), generator=g, device=dev, dtype=torch.int32)
    rt.error_word(dev)

    def fused_step():
        for blk in W:
            fused.linear_rope(x, blk["qkv_f"], cos, sin, H, H, Dh, pos=pos, norm_eps=cfg.norm_eps)
            fused.linear_residual(attn, blk["o"], x)
            a = fused.linear_swiglu(x, blk["gu_f"], norm_eps=cfg.norm_eps)
            fused.linear_residual(a, blk["dn"], x)

    def unfused_step():
        for blk in W:
            h = fused.rmsnorm(x, ones, cfg.norm_eps)
            fused.rope_split(h @ blk["qkv"], cos, sin, H, H, Dh, pos=pos)
            x.addmm_(attn, blk["o"])
            a = fused.silu_mul(fused.rmsnorm(x, ones, cfg.norm_eps) @ blk["gu"])
            x.addmm_(a, blk["dn"])

    def folded_step():
        for blk in W:
            fused.rope_split(x @ blk["qkv_f"], cos, sin, H, H, Dh, pos=pos, norm_x=x, norm_eps=cfg.norm_eps)
            x.addmm_(attn, blk["o"])
            a = fused.silu_mul(x @ blk["gu_n"], norm_x=x, norm_eps=cfg.norm_eps)
            x.addmm_(a, blk["dn"])

    def timed(step):
        for _ in range(max(3, args.warmup)):
            step()
        torch.cuda.synchronize()
        gr = torch.cuda.CUDAGraph()
        st = torch.cuda.Stream()
        st.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(st):
            with torch.cuda.graph(gr, stream=st):
                step()
        torch.cuda.current_stream().wait_stream(st)
        gr.replay()
        torch.cuda.synchronize()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(0) as clk:
            ev0.record()
            for _ in range(args.steps):
                gr.replay()
            ev1.record()
            torch.cuda.synchronize()
        return ev0.elapsed_time(ev1) / args.steps, clk.summary()

    ms, clocks = timed(fused_step)
    ms_unfused, _ = timed(unfused_step)
    ms_folded, _ = timed(folded_step)
    rt.read_device_error(dev)
    wbytes = sum(t.numel() * 2 for blk in W for t in (blk["qkv"], blk["o"], blk["gu"], blk["dn"]))
    gbs = wbytes / (ms * 1e-3) / 1e9
    peak, peak_kind = measured_peak()
    print(json.dumps({"metric": "fused linear layers: weight bytes streamed (config-4 blocks)", "value": gbs,
                      "unit": "GB/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
                      "higher_is_better": True, "dtype": "bf16", "data": "synthetic",
                      "config": {"workload": "linear_fused_cfg4_blocks", "rows": n, "layers": layers,
                                 "launches_per_layer": 4, "weights_mb": wbytes / 1e6},
                      "unfused": {"ms_per_step": ms_unfused, "launches_per_layer": 8,
                                  "what": "RMSNorm + cuBLAS GEMM + RoPE split / SwiGLU kernels"},
                      "folded": {"ms_per_step": ms_folded, "launches_per_layer": 6,
                                 "what": "cuBLAS GEMM on norm-folded weights + RoPE split / SwiGLU with the row scale "
                                         "(the bf16 engine's chain)"},
                      "roofline": {"bound": "hbm", "achieved": gbs, "peak": peak, "unit": "GB/s", "frac": gbs / peak,
                                   "peak_kind": peak_kind},
                      "gpu_launches": 4 * layers * args.steps, "clocks": clocks}), flush=True)


def run_tick_profile(args):
    """--workload cfg4tick: per-tick kernel breakdown of greedy wavefront decoding
    on the device scheduler (diagnostic; prints a table, no JSON line).  Runs
    the config-4 model (random init, bf16, 1024-token prompts, --batch
    sequences, --new-tokens, --t-draft) once to capture the tick graph, then once
    more under torch.profiler (CUPTI kernel records of the graph replays, no
    kernel replay) and prints, for the decode ticks only: span and busy time per
    tick, every kernel's launches and device time per tick, and each attention
    launch's K/V bytes and read rate."""
    import collections

    import torch
    from torch.profiler import ProfilerActivity, profile

    import __graft_entry__
    __graft_entry__.load_package()
    from wavefront_decoding_b200 import scheduler as sch
    from wavefront_decoding_b200.device_scheduler import DeviceWave
    from wavefront_decoding_b200.engine import WaveEngine
    from wavefront_decoding_b200.looped_lm import CONFIG4, LoopedLM

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    B, new, L = args.batch or 8, args.new_tokens or 32, CFG4["L"]
    cfg = CONFIG4
    prompts = torch.randint(0, cfg.vocab, (B, L), generator=torch.Generator().manual_seed(CFG4["seed"])).pin_memory()
    model = LoopedLM(cfg, seed=CFG4["model_seed"], dtype=torch.bfloat16, device=dev)
    eng = WaveEngine(model, B, L + new + 2 * cfg.T_total + 8)
    dw = DeviceWave(eng, new, sch.SsdPolicy(cfg.T_total, args.t_draft))
    dw.generate(prompts, None)  # captures the tick graph
    torch.cuda.synchronize()
    orig = eng.prefill

    def prefill(ids):  # a marker kernel between the prompt pass and the first tick
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
    for s0, e0, _ in ks:
        if cur_e is None or s0 > cur_e:
            if cur_e is not None:
                busy += cur_e - cur_s
            cur_s, cur_e = s0, e0
        else:
            cur_e = max(cur_e, e0)
    if cur_e is not None:
        busy += cur_e - cur_s
    span = ks[-1][1] - ks[0][0] if ks else 0.0
    agg = collections.defaultdict(lambda: [0, 0.0])
    for s0, e0, nm in ks:
        agg[nm[:100]][0] += 1
        agg[nm[:100]][1] += e0 - s0
    total = sum(a[1] for a in agg.values()) or 1.0
    print(f"batch {B}: {ticks} ticks, {bt.n_tokens} tokens; per tick: span {span / ticks:.1f} us, "
          f"busy {busy / ticks:.1f} us, {len(ks) / ticks:.1f} kernels")
    print(f"  {'launches':>8} {'us/tick':>9} {'share':>6} {'us/launch':>10}  kernel")
    for nm, (c, t) in sorted(agg.items(), key=lambda x: -x[1][1]):
        print(f"  {c:8d} {t / ticks:9.2f} {100 * t / total:5.1f}% {t / c:10.2f}  {nm}")
    # the attention launches of a tick: prelude layers, core layers, coda layers
    keys = dw.keys.tolist()
    rb = 2 * eng._row_bytes
    per_layer = [keys[0]] * cfg.n_prelude + [keys[1]] * cfg.n_core + [keys[2]] * cfg.n_coda
    tc = [e0 - s0 for s0, e0, nm in ks if "wave_tc_kernel" in nm or "wave_decode_kernel" in nm]
    n_att = len(per_layer)
    if tc and len(tc) % n_att == 0:
        print("  attention launch (position in the tick): mean us, K/V MB, GB/s")
        for i in range(n_att):
            m = sum(tc[i::n_att]) / len(tc[i::n_att])
            mb = per_layer[i] / ticks * rb / 1e6
            print(f"    {i}: {m:8.2f} us {mb:8.1f} MB {mb / 1e3 / (m * 1e-6):7.0f}")


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "cfg4":
        run_cfg4(args)
    elif args.workload == "cfg4tick":
        run_tick_profile(args)
    elif args.workload == "prefill":
        run_prefill(args)
    elif args.workload == "linear":
        run_linear(args)
    else:
        run_wfd(args)


if __name__ == "__main__":
    main()
