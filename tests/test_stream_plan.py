"""The step kernel's weight-stream plan, checked on the CPU.

make_plan (isa-lm_b200/csrc/kc_step.cuh) decides, for CTA j of G, which rows
of every matrix it streams, in which records and in which bulk copies; the
upload lays the weights out by it and the kernel's tagged-word ownership
follows it. tests/stream_plan_check.cu compiles that header for the host
(nvcc, nothing launched) and checks every CTA's plan for the BASELINE shapes,
cfg4's tensor-parallel shards, both scale types, both gate|up ownership units
and every bulk-copy size the runtime may pick (56 KB down to 32 KB): rows
handed out exactly once and in CTA order, whole records per copy within the
chunk, whole units in the gate|up phase, the ring slot equal to the largest
copy. The reference's counterpart is its matvec's split of a matrix's rows
among the pool's threads (ops/ops.c:16-25, aligned chunks per thread); here
the CTAs of one persistent kernel take that role.
"""
import os
import shutil
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "isa-lm_b200"))
import krafla_models as km  # noqa: E402

Q8, Q4 = 1, 2
SMS = 148


def shapes():
    """(label, dim, q_dim, kv_dim, hidden, vocab, types q k v o up down cls, bias) of the BASELINE configs,
    cfg4's TP shards (both ways of cutting the classifier rows) and a tiny model with idle CTAs."""
    out = []
    for name, c in km.CONFIGS.items():
        hd = c["dim"] // c["n_heads"]
        q8 = set(c.get("q8", ()))
        t = lambda cls: Q8 if c["wtype"] == "q8" or cls in q8 else Q4  # noqa: E731
        types = (t("qk"), t("qk"), t("v"), t("o"), t("up"), t("down"), t("emb" if c.get("shared") else "cls"))
        bias = int(bool(c.get("qkv_bias")))
        q, kv, hid, voc = c["n_heads"] * hd, c["n_kv_heads"] * hd, c["hidden_dim"], c["vocab"]
        out.append((name, c["dim"], q, kv, hid, voc, types, bias))
        if name == "cfg4":
            for n in (2, 4, 8):
                for v in (voc // n, voc - (n - 1) * (voc // n)):
                    out.append((f"{name}/tp{n}", c["dim"], q // n, kv // n, hid // n, v, types, bias))
    out.append(("tiny", 64, 64, 32, 128, 256, (Q4, Q4, Q8, Q8, Q4, Q8, Q8), 1))
    return out


def cases():
    lines = []
    for _, dim, q, kv, hid, voc, ty, b in shapes():
        G = min(SMS, dim)
        for d16 in (0, 1):
            for unit in (32, 4):
                for chunk in [0] + [kb * 1024 for kb in range(32, 57, 4)]:
                    lines.append(" ".join(map(str, (dim, q, kv, hid, voc, *ty, d16, b, b, b, G, unit, chunk))))
    return lines


@pytest.fixture(scope="module")
def checker(tmp_path_factory):
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(nvcc):
        pytest.skip("nvcc not found")
    exe = str(tmp_path_factory.mktemp("plan") / "stream_plan_check")
    subprocess.run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-O1", "-std=c++17",
                    "--expt-relaxed-constexpr", "-I", os.path.join(ROOT, "isa-lm_b200", "csrc"),
                    "-I", os.path.join(ROOT, "include"), os.path.join(ROOT, "tests", "stream_plan_check.cu"),
                    "-o", exe], check=True, capture_output=True)
    return exe


def run(exe, lines):
    return subprocess.run([exe], input="\n".join(lines) + "\n", capture_output=True, text=True, timeout=120)


def test_plan_of_every_shape_chunk_and_unit(checker):
    lines = cases()
    r = run(checker, lines)
    assert r.returncode == 0, r.stdout + r.stderr
    assert r.stdout.split() == ["ok", str(len(lines))]


def test_checker_rejects_a_plan_it_cannot_hold(checker):
    """A control: 20000 rows of x on 148 CTAs give a CTA 136 rows, more than
    the 128 it can own; the checker must say so rather than pass."""
    r = run(checker, ["20000 2048 512 8192 32000 2 2 1 1 2 1 2 1 0 0 0 148 32 0"])
    assert r.returncode != 0 and "more rows of x than a CTA can own" in r.stdout, r.stdout
