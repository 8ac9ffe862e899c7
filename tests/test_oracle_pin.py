"""Pins the CPU oracle (oracle/krafla_oracle.c) to the reference.

- bit for bit against the logits of the reference's own scalar build
  (golden/<model>.logits.npy, written by golden/gen_golden.py through
  ml_forward of the reference library);
- within the reference's e2e criterion (tests/compare_logits.py:27-30 of the
  reference: max|a-b| <= 1e-3 max|b| and equal argmax) against its numpy
  forward (tools/ref_forward.py);
- the Q8_0 rule against tools/mlb.py:125-142 and the known answers of the
  reference's tests/test_quant.c.
"""
import os

import numpy as np
import pytest

from conftest import GOLDEN

import oracle

TOKENS = [1, 5, 9, 13, 17, 21, 25, 29, 33, 37, 41, 45, 49, 53, 57, 61]
MODELS = sorted(f[:-4] for f in os.listdir(os.path.join(GOLDEN, "models")) if f.endswith(".mlb"))


@pytest.fixture(scope="module", autouse=True)
def _built(built):
    return built


@pytest.mark.parametrize("name", MODELS)
def test_oracle_equals_reference_scalar_build(name):
    m = oracle.OracleModel(os.path.join(GOLDEN, "models", f"{name}.mlb"), nthreads=1)
    got = np.stack([m.forward(t, p) for p, t in enumerate(TOKENS)])
    want = np.load(os.path.join(GOLDEN, f"{name}.logits.npy"))
    assert got.view(np.uint32).tolist() == want.view(np.uint32).tolist()


@pytest.mark.parametrize("name", MODELS)
def test_oracle_within_reference_numpy_forward(name):
    m = oracle.OracleModel(os.path.join(GOLDEN, "models", f"{name}.mlb"))
    got = m.prefill(TOKENS)
    ref = np.load(os.path.join(GOLDEN, f"{name}.numpy.npy")).astype(np.float64)
    err = np.abs(got - ref).max(axis=1) / np.abs(ref).max(axis=1)
    assert err.max() <= 1e-3
    assert (got.argmax(1) == ref.argmax(1)).all()


def test_oracle_thread_count_does_not_change_results():
    path = os.path.join(GOLDEN, "models", "mix_q4.mlb")
    a = oracle.OracleModel(path, nthreads=1).prefill(TOKENS)
    b = oracle.OracleModel(path, nthreads=7).prefill(TOKENS)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_quantize_q8_matches_reference_rule():
    z = np.load(os.path.join(GOLDEN, "quant.npz"))
    q, d = oracle.quantize_q8(z["x"])
    assert np.array_equal(q, z["q8_f32"])
    assert np.array_equal(d.view(np.uint32), z["d8_f32"].view(np.uint32))


def test_quantize_q8_known_answers():
    # tests/test_quant.c:47-60: amax 127 makes id = 1, ties round away from zero
    x = np.zeros(32, np.float32)
    x[0] = 127.0
    x[1:6] = [0.5, -0.5, 1.5, 2.5, -2.5]
    q, d = oracle.quantize_q8(x)
    assert d[0] == 1.0 and q[1:6].tolist() == [1, -1, 2, 3, -3]
    # :37-45 clamp to -127 at the negative amax
    x = np.linspace(-1, 1, 32).astype(np.float32)
    x[3], x[9] = -5.0, 4.999
    q, _ = oracle.quantize_q8(x)
    assert q[3] == -127 and q.min() >= -127 and q.max() <= 127
    # :64-70 tiny block -> d = 0, q = 0; zero block likewise
    x = np.array([0.0 if i % 3 == 0 else (1e-37 if i % 3 == 1 else -2e-37) for i in range(32)] + [0.0] * 32,
                 np.float32)
    q, d = oracle.quantize_q8(x)
    assert (d == 0).all() and (q == 0).all()


def test_block_sums_and_matvec_unit_scales_exact():
    # tests/test_kernels.c:87-108: with unit scales the matvec is exact
    rng = np.random.default_rng(5)
    for wtype, cols in ((1, 96), (2, 256)):
        rows = 7
        wq = (rng.integers(-127, 128, rows * cols).astype(np.int8) if wtype == 1
              else rng.integers(0, 256, rows * cols // 2).astype(np.uint8))
        xq = rng.integers(-127, 128, cols).astype(np.int8)
        s = oracle.block_sums(wtype, wq, rows, cols, xq)
        if wtype == 1:
            ref = (wq.reshape(rows, -1, 32).astype(np.int64) * xq.reshape(-1, 32)).sum(-1)
        else:
            p = wq.reshape(rows, -1, 16).astype(np.int64)
            w = np.concatenate([(p & 15) - 8, (p >> 4) - 8], -1)
            ref = (w * xq.reshape(-1, 32)).sum(-1)
        assert np.array_equal(s, ref)
        y = oracle.matvec(wtype, wq, np.ones((rows, cols // 32), np.float32), rows, cols, xq,
                          np.ones(cols // 32, np.float32))
        assert np.array_equal(y, ref.sum(1).astype(np.float32))


@pytest.mark.skipif(not os.path.exists(os.path.join(oracle.REF_DIR, "libkrafla_ref_scalar.so")),
                    reason="oracle/_ref not built (needs the reference sources)")
def test_oracle_kernels_equal_reference_kernels():
    import ctypes as C
    ref = oracle.RefBuild("scalar")
    rng = np.random.default_rng(11)
    x = (rng.standard_normal(4096) * 3).astype(np.float32)
    x[32:64] = 0.0
    q1, d1 = oracle.quantize_q8(x)
    q2, d2 = np.empty(4096, np.int8), np.empty(128, np.float32)
    ref.L.ref_quantize_q8_scalar(q2.ctypes.data_as(C.c_void_p), d2.ctypes.data_as(C.c_void_p),
                                 x.ctypes.data_as(C.c_void_p), 4096)
    assert np.array_equal(q1, q2) and np.array_equal(d1.view(np.uint32), d2.view(np.uint32))
    for wtype, rows, cols in ((1, 33, 8288), (2, 17, 256)):
        wq = (rng.integers(-127, 128, rows * cols).astype(np.int8) if wtype == 1
              else rng.integers(0, 256, rows * cols // 2).astype(np.uint8))
        wd = (rng.uniform(0.001, 0.05, (rows, cols // 32)) * rng.choice([-1, 1], (rows, cols // 32))).astype(np.float32)
        xq = rng.integers(-127, 128, cols).astype(np.int8)
        xd = rng.uniform(0.001, 0.05, cols // 32).astype(np.float32)
        y1 = oracle.matvec(wtype, wq, wd, rows, cols, xq, xd)
        y2 = np.empty(rows, np.float32)
        ref.L.ref_matvec_scalar(y2.ctypes.data_as(C.c_void_p), wtype, wq.ctypes.data_as(C.c_void_p),
                                wd.ctypes.data_as(C.c_void_p), rows, cols, xq.ctypes.data_as(C.c_void_p),
                                xd.ctypes.data_as(C.c_void_p), 0, rows)
        assert np.array_equal(y1.view(np.uint32), y2.view(np.uint32))
