"""The benchmark's reference arm (`bench.py --impl reference`) runs on the host cores alone and prints
one JSON line with the keys the benchmark contract names; checked here on the CPU."""

from __future__ import annotations

import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_prints_the_contract_line():
    out = subprocess.run(
        [sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "3", "--warmup", "3"],
        cwd=ROOT, capture_output=True, text=True, timeout=600, check=True,
    ).stdout
    lines = [line for line in out.splitlines() if line.startswith("{")]
    assert len(lines) == 1, out
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e", "impl"):
        assert key in d, key
    assert d["impl"] == "reference" and d["steps"] == 3 and d["warmup"] == 3 and d["n_gpus"] == 1
    assert d["value"] > 0 and d["ms_per_step"] > 0 and d["cpu_baseline"]["value"] == d["value"]
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    assert d["config"]["workload"] == "llama8b" and d["cpu_baseline"]["cores"] >= 1


def test_reference_arm_under_torchrun_uses_every_core_and_the_gpu_arms_config():
    """torchrun sets OMP_NUM_THREADS=1 in every rank: the reference arm still runs on every host core it may
    use, and its config carries exactly the keys and values the GPU arm reports at the same N."""
    env = dict(os.environ, OMP_NUM_THREADS="1", RANK="0", LOCAL_RANK="0", WORLD_SIZE="2")
    out = subprocess.run(
        [sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--gpus", "2", "--steps", "3",
         "--warmup", "3"],
        cwd=ROOT, capture_output=True, text=True, timeout=600, check=True, env=env,
    ).stdout
    d = json.loads([line for line in out.splitlines() if line.startswith("{")][0])
    assert d["cpu_baseline"]["cores"] == len(os.sched_getaffinity(0))
    sys.path.insert(0, ROOT)
    import bench

    want = bench.line_config("llama8b", bench.CONFIGS["llama8b"], "reference", "deferred", 2)
    assert d["config"] == want
    # the other ranks print nothing and exit cleanly
    env["RANK"] = "1"
    other = subprocess.run(
        [sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--gpus", "2", "--steps", "3",
         "--warmup", "3"],
        cwd=ROOT, capture_output=True, text=True, timeout=600, check=True, env=env,
    ).stdout
    assert not [line for line in other.splitlines() if line.startswith("{")]
