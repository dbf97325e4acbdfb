"""bench.py's reference arm on the host (it needs no GPU): one bounded step of the CPU restatement of the reference's
forward prints the benchmark line with the fields the harness reads, and ranks other than 0 exit without work."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(tmp_path, extra_env):
    env = dict(os.environ, XTB_BENCH_DIR=str(tmp_path), **extra_env)
    for k in ("RANK", "WORLD_SIZE", "LOCAL_RANK"):
        if k not in extra_env:
            env.pop(k, None)
    return subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                           "--warmup", "0"], cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)


def test_reference_arm_line(tmp_path):
    r = _run(tmp_path, {})
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["unit"] == "images/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["steps"] == 1 and d["n_gpus"] == 1
    assert d["config"]["workload"].startswith("config 3") and d["config"]["global_batch"] == 64
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == d["value"] and cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": "images/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert "no CUDA device" in d["reference_gpu_kernels"]["unavailable"]  # the reference's GPU kernels need a GPU


def test_reference_arm_other_ranks_exit_quietly(tmp_path):
    r = _run(tmp_path, {"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"})
    assert r.returncode == 0, r.stderr[-2000:]
    assert not [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert not os.listdir(tmp_path)      # no model written: rank 1 does no work
