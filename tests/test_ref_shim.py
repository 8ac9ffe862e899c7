"""The drop-in boundary seen from the reference: its own apps (app/ml_run.c,
app/ml_bench.c) built as a `cuda` ISA (isa-lm_b200/ref_shim: isa_cuda.patch
on mk/isa.mk, Makefile and config/ml_config.h, and transformer_cuda.c in place
of model/transformer.c) link and run against libkrafla_cuda.so. On a host
without a GPU, ml_state_init returns ML_E_ISA and ml_run exits with its
message (app/ml_run.c:326-330), as the reference's ISA guard does for a CPU
that lacks the build's ISA (app/main_guard.c:8-15)."""
import os
import subprocess

import pytest

from conftest import GOLDEN, ROOT

import oracle

SHIM = os.path.join(ROOT, "isa-lm_b200", "ref_shim")
BIN = os.path.join(SHIM, "_build", "bin")


@pytest.fixture(scope="module")
def shim_bin(built):
    ref = oracle.reference_root()
    if ref:   # rebuilds only when a source changed
        subprocess.run(["make", "-s", "-C", SHIM, f"REF={ref}"], check=True, capture_output=True)
    if not os.path.exists(os.path.join(BIN, "ml_run")):
        pytest.skip("the reference tree is not here and the shim's apps were not built")
    return BIN


def test_patch_touches_only_the_build_files():
    text = open(os.path.join(SHIM, "isa_cuda.patch")).read()
    files = sorted(l.split()[1] for l in text.splitlines() if l.startswith("+++ "))
    assert files == ["b/Makefile", "b/config/ml_config.h", "b/mk/isa.mk"]
    assert "CHAIN_cuda" in text and '#define ML_ISA_NAME "cuda"' in text and "-lkrafla_cuda" in text


def test_apps_name_the_cuda_isa(shim_bin):
    r = subprocess.run([os.path.join(shim_bin, "ml_run"), "--help"], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0 and "build ISA: cuda" in r.stdout


def test_ml_run_without_gpu_is_the_isa_error(shim_bin):
    if os.path.exists("/dev/nvidia0"):
        pytest.skip("a GPU is present")
    model = os.path.join(GOLDEN, "models", "rand_q8.mlb")
    r = subprocess.run([os.path.join(shim_bin, "ml_run"), model, "--tokens", "1,2,3", "-n", "4"],
                       capture_output=True, text=True, timeout=60)
    assert r.returncode == 1
    assert "error: CPU lacks required ISA" in r.stderr   # ml_status_str(ML_E_ISA)
    assert "cuda: no B200 (sm_100) GPU" in r.stderr
