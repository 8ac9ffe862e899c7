"""The reference against itself: its SIMD builds (oracle/_ref, compiled from the
reference sources) against its scalar build on BASELINE config 0.

This is the yardstick of the model-level parity bar. The reference's own best
builds agree with its scalar build to ~1e-7 until one quantized activation
lands on the other side of a rounding boundary, and by ~1e-2 after it; they
satisfy the reference's two-implementations criterion, which is the bar the
GPU is held to on long runs (tests/test_model_gpu.py).
"""
import ctypes as C
import os

import numpy as np
import pytest

from conftest import MODEL_CACHE

import krafla_b200 as kb
import oracle

from test_model_gpu import RTOL, rel_err, valid_pair


def _build(isa):
    try:
        return oracle.RefBuild(isa)
    except (FileNotFoundError, RuntimeError, OSError):
        return None


@pytest.mark.parametrize("isa", ["avx512vnni", "avx2"])
def test_reference_simd_builds_vs_scalar(isa, built):
    simd, scalar = _build(isa), _build("scalar")
    if simd is None or scalar is None:
        pytest.skip(f"reference {isa} build not available on this host")
    path = kb.ensure_model("cfg0", MODEL_CACHE)
    prompt = np.random.default_rng(0).integers(0, 32000, 16).tolist()
    out = {}
    for name, r in (("scalar", scalar), (isa, simd)):
        h = r.open(path, os.cpu_count() or 1, 0, True)
        lg = np.zeros((16, 32000), np.float32)
        for p, t in enumerate(prompt):
            assert r.L.ref_forward(h, t, p, lg[p].ctypes.data_as(C.c_void_p)) == 0
        r.L.ref_close(h)
        out[name] = lg
    err = rel_err(out[isa], out["scalar"])
    strict_ok = int(np.argmax(err > RTOL)) if (err > RTOL).any() else len(err)
    print(f"reference {isa} vs scalar on cfg0: strict bar holds for the first {strict_ok} positions; "
          f"max rel err {err.max():.1e}")
    assert err[0] <= RTOL
    assert all(valid_pair(out[isa][i], out["scalar"][i]) for i in range(16))
