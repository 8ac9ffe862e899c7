"""bench.py's reference arm on the host (no GPU): it prints one JSON line with
the keys the benchmark contract asks of it, on the workload config the device
arm uses. Runs the reference's own CPU build (oracle/_ref) on the small
config cfg0 so that it finishes in seconds."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_json_line(tmp_path):
    ref = os.path.join(ROOT, "oracle", "_ref")
    if not os.path.isdir(ref) or not any(f.endswith(".so") for f in os.listdir(ref)):
        pytest.skip("oracle/_ref not built")
    env = dict(os.environ, KRAFLA_MODEL_DIR=str(tmp_path))
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--config", "cfg0",
                          "--ctx", "32", "--steps", "2", "--warmup", "1"],
                         capture_output=True, text=True, env=env, timeout=600, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["metric"] == "batch-1 decode tok/s" and d["unit"] == "tok/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["steps"] == 2 and d["warmup"] == 1
    assert d["config"]["model"] == "cfg0" and d["config"]["batch"] == 1 and d["config"]["ctx"] == 32
    assert d["config"]["workload"] == "cfg0 batch-1 greedy decode at KV context 32"
    cb = d["cpu_baseline"]
    assert cb["kind"] == "reference" and cb["value"] == d["value"] and cb["cores"] >= 1 and cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_under_torchrun(tmp_path):
    """Two ranks (as the driver's scaling runs launch it): rank 0 alone prints the
    line, the other rank exits 0 without work; no process group is needed."""
    ref = os.path.join(ROOT, "oracle", "_ref")
    if not os.path.isdir(ref) or not any(f.endswith(".so") for f in os.listdir(ref)):
        pytest.skip("oracle/_ref not built")
    env = dict(os.environ, KRAFLA_MODEL_DIR=str(tmp_path))
    out = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
                          "--master-addr", "127.0.0.1", "--master-port", "29631", os.path.join(ROOT, "bench.py"),
                          "--impl", "reference", "--gpus", "2", "--config", "cfg0", "--ctx", "32", "--steps", "2",
                          "--warmup", "1"], capture_output=True, text=True, env=env, timeout=600, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["n_gpus"] == 2 and d["value"] > 0
