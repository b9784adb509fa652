"""bench.py's reference arm on the host: one JSON line with the keys and meanings
the benchmark contract fixes (impl, metric, unit, the same workload config as the
repository arm, a cpu_baseline describing the run, an e2e record with no host /
device copies).  The arm times the CPU restatement of the reference's decode path
and needs no GPU, so it runs here at its smallest size."""
from __future__ import annotations

import json
import os
import pathlib
import subprocess
import sys

ROOT = pathlib.Path(__file__).resolve().parent.parent


def _run(*args: str) -> dict:
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    p = subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], cwd=ROOT, env=env,
                       capture_output=True, text=True, timeout=600)
    assert p.returncode == 0, p.stderr[-2000:]
    lines = [ln for ln in p.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, p.stdout[-2000:]
    return json.loads(lines[0])


def test_reference_arm_line_for_config2():
    import bench
    d = _run("--impl", "reference", "--steps", "1", "--warmup", "1", "--cpu-seconds", "1")
    assert d["impl"] == "reference"
    assert d["metric"] == bench.METRIC and d["unit"] == bench.UNIT
    assert d["higher_is_better"] is True and d["n_gpus"] == 1
    assert d["value"] > 0 and d["ms_per_step"] > 0
    cfg = d["config"]
    assert cfg["workload"] == "cfg2_wavefront_decode_attention"
    assert (cfg["batch_per_gpu"], cfg["slots"], cfg["n_heads"], cfg["n_kv_heads"], cfg["head_dim"]) == \
        (bench.CFG2["B"], bench.CFG2["R"], bench.CFG2["H"], bench.CFG2["Hkv"], bench.CFG2["Dh"])
    base = d["cpu_baseline"]
    assert base["value"] == d["value"] and base["unit"] == d["unit"]
    assert base["kind"] in ("port", "reference") and base["cores"] >= 1 and base["sample"]
    e2e = d["e2e"]
    assert e2e == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
