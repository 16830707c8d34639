"""bench.py's reference arm runs on any host: its one JSON line carries the keys the driver reads.

The arm times the reference's own CPU attention (oracle/_ref, built from the reference's sources;
the restatement when that is absent) on a bounded sample of the headline workload, so it runs here
without a GPU. Standard output must hold exactly that one line.
"""
import json
import os
import subprocess
import sys

import bench

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_prints_one_contract_line():
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
                        "--steps", "1", "--warmup", "0"],
                       capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1, r.stdout[-2000:]
    d = json.loads(lines[0])
    for k in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
              "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
              "cpu_baseline", "e2e"):
        assert k in d, k
    assert d["impl"] == "reference"
    assert d["config"] == bench.workload_config(1)  # the b200 arm prints the same dict
    assert len(lines[0]) < 1400  # read whole from the tail of the run's output
    assert d["metric"] == bench.METRIC and d["unit"] == "TFLOP/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["steps"] == 1
    assert d["cpu_baseline"]["kind"] in ("reference", "port") and d["cpu_baseline"]["cores"] >= 1
    assert d["cpu_baseline"]["nproc"] >= 1
    assert d["cpu_baseline"]["value"] == d["value"]
    assert d["e2e"] == {"value": d["value"], "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_exit_quietly():
    env = dict(os.environ, RANK="1", WORLD_SIZE="2", LOCAL_RANK="1")
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
                        "--gpus", "2", "--steps", "1", "--warmup", "0"],
                       capture_output=True, text=True, timeout=300, cwd=ROOT, env=env)
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.strip() == ""


def test_cpu_baseline_reports_median_min_max_and_the_prompt_sweep():
    c = bench.cpu_reference_sample(0.0, max_layers=2, p=128)
    assert c["P"] == 128 and c["layers"] == 2
    assert c["min_s"] <= c["per_layer_s"] <= c["max_s"] and c["tflops"] > 0
    assert c["threads"] >= 1 and c["nproc"] >= 1
    sweep = bench.cpu_sweep(0.0)
    assert set(sweep) == {"P128", "P512"}
    for v in sweep.values():
        assert v["layers"] >= 2 and v["min_ms"] <= v["median_ms"] <= v["max_ms"] and v["tflops"] > 0


def test_algorithmic_work_conventions(lib):
    """The roofline numerators: prefill FLOPs 2*P^2*768 per layer (4*P^2*64*12/2), decode bytes
    2*L*H*len*64*2, the latter equal to the library's gpt2_kv_step_bytes (the reference's formula)."""
    import ctypes

    import gpt2_b200 as G
    assert bench.prefill_flops(128, 1) == 25165824.0
    assert bench.prefill_flops(1024, 1) == 1610612736.0
    assert bench.prefill_flops(1024) == 19327352832.0  # the headline launch: 19.33 GFLOP
    kv = G.cache_view(4096, 12, 1024)
    for n in (128, 512, 1023):
        assert bench.decode_bytes(n) == 36864.0 * n == lib.gpt2_kv_step_bytes_b200(ctypes.byref(kv), n)
