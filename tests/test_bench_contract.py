"""bench.py's reference arm on the host (no GPU): it prints one JSON line with
the keys the benchmark contract asks of it, on the workload config the device
arm uses, and its process maps no library of this repository (only the
reference's own build in oracle/_ref). Runs the reference's CPU build on the
small config cfg0 so that it finishes in seconds."""
import json
import os
import socket
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ARGS = ["--impl", "reference", "--config", "cfg0", "--ctx", "32", "--steps", "2", "--warmup", "1", "--repeats", "2"]

# runs bench.py in this interpreter, then lists the shared objects the process mapped
WRAP = """
import runpy, sys
sys.argv = [sys.argv[1]] + sys.argv[2:]
runpy.run_path(sys.argv[0], run_name="__main__")
maps = sorted({l.split()[-1] for l in open("/proc/self/maps") if l.rstrip().endswith(".so") or ".so." in l})
print("MAPS " + " ".join(maps), file=sys.stderr)
"""


def _need_ref():
    ref = os.path.join(ROOT, "oracle", "_ref")
    if not os.path.isdir(ref) or not any(f.endswith(".so") for f in os.listdir(ref)):
        pytest.skip("oracle/_ref not built")


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_reference_arm_json_line(tmp_path):
    _need_ref()
    env = dict(os.environ, KRAFLA_MODEL_DIR=str(tmp_path))
    out = subprocess.run([sys.executable, "-c", WRAP, os.path.join(ROOT, "bench.py"), *ARGS],
                         capture_output=True, text=True, env=env, timeout=600, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["metric"] == "batch-1 decode tok/s" and d["unit"] == "tok/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["steps"] == 2 and d["warmup"] == 1
    c = d["config"]
    assert c["baseline_config"] == "cfg0" and c["batch"] == 1 and c["ctx"] == 32 and c["kv_cache"] == "f32"
    assert c["workload"] == "cfg0 batch-1 greedy decode at KV context 32" and c["parallelism"] == "single device"
    cb = d["cpu_baseline"]
    assert cb["kind"] == "reference" and cb["value"] == d["value"] and cb["cores"] >= 1 and cb["sample"]
    assert cb["min"] <= cb["value"] <= cb["max"]
    assert d["e2e"] == {"value": d["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    # the process mapped the reference's build and no library of this repository
    maps = [l for l in out.stderr.splitlines() if l.startswith("MAPS ")][-1].split()[1:]
    ours = [m for m in maps if m.startswith(ROOT) and "/oracle/_ref/" not in m]
    assert not ours, ours
    assert any("/oracle/_ref/libkrafla_ref_" in m for m in maps)


def test_reference_arm_under_torchrun(tmp_path):
    """Two ranks (as the driver's scaling runs launch it): rank 0 alone prints the
    line, the other rank exits 0 without work; no process group is needed. At
    N > 1 the workload is the tensor-parallel config (here cfg0 stands in)."""
    _need_ref()
    env = dict(os.environ, KRAFLA_MODEL_DIR=str(tmp_path))
    out = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
                          "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
                          os.path.join(ROOT, "bench.py"), "--impl", "reference", "--gpus", "2", "--tp-config", "cfg0",
                          "--tp-ctx", "32", "--steps", "2", "--warmup", "1", "--repeats", "2"],
                         capture_output=True, text=True, env=env, timeout=600, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["n_gpus"] == 2 and d["value"] > 0
    assert d["config"]["parallelism"] == "tp2" and d["config"]["baseline_config"] == "cfg0"
