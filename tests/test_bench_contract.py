"""The benchmark's reference arm on the CPU: `bench.py --impl reference` (run by the driver beside the GPU arm) prints
one JSON line with the keys of the benchmark contract, timing the C restatement of the reference's kernels."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_json_line():
    env = dict(os.environ, DECISION_REF_REQUESTS="1")
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                        "--warmup", "1"], cwd=ROOT, env=env, capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    for k in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
              "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert k in line, k
    assert line["impl"] == "reference" and line["metric"] == "requests/sec" and line["value"] > 0
    assert line["warmup"] >= 3 and line["higher_is_better"] is True and line["scaling"] == "weak"
    assert line["config"]["workload"].startswith("BASELINE config 2")
    cb = line["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == line["value"] and "texts" in cb["sample"]
    assert line["e2e"] == {"value": line["value"], "unit": line["unit"], "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_exit_quietly():
    """Under torchrun (N > 1) rank 0 alone times the CPU arm and prints its line; the other ranks exit 0 at once."""
    env = dict(os.environ, RANK="1", WORLD_SIZE="2", LOCAL_RANK="1", DECISION_REF_REQUESTS="1")
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--gpus", "2",
                        "--steps", "1", "--warmup", "1"], cwd=ROOT, env=env, capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.strip() == ""


def test_direct_sweep_needs_one_shape():
    """`bench.py --sweep --direct` times the direct form on the one shape --only names; without it, it stops with a
    message before touching a device."""
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--sweep", "--direct"], cwd=ROOT,
                       capture_output=True, text=True, timeout=300)
    assert r.returncode != 0 and "--direct needs --only" in r.stderr
