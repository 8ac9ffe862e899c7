"""Kernel-level parity on the GPU, through the C ABI, against the CPU oracle.

Bar (the reference's own, tests/test_kernels.c): quantized activations and
int32 block dot products bit exact; matvec with unit scales exact; with real
scales within 1e-5 of the sum of |terms| (TT_CLOSE of tests/tt.h:27-32).
"""
import os

import numpy as np
import pytest

from conftest import GOLDEN

import krafla_b200 as kb
import oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _dev(built):
    kb.device_check()


@pytest.mark.parametrize("k", [32, 288, 896, 4096, 8192, 14336, 65536])
def test_quantize_q8_bit_exact(k):
    rng = np.random.default_rng(k)
    x = (rng.standard_normal(k) * rng.choice([1e-3, 1, 40], k)).astype(np.float32)
    if k >= 128:
        x[32:64] = 0.0
        x[64:96] = np.where(np.arange(32) % 2, 1e-37, -3e-37)
    q, d = kb.quantize_q8(x)
    rq, rd = oracle.quantize_q8(x)
    assert np.array_equal(q, rq)
    assert np.array_equal(d.view(np.uint32), rd.view(np.uint32))


def test_quantize_q8_reference_vectors():
    z = np.load(os.path.join(GOLDEN, "quant.npz"))
    q, d = kb.quantize_q8(z["x"])
    assert np.array_equal(q, z["q8_f32"])
    assert np.array_equal(d.view(np.uint32), z["d8_f32"].view(np.uint32))


def test_quantize_q8_known_answers():
    x = np.zeros(64, np.float32)
    x[0] = 127.0
    x[1:6] = [0.5, -0.5, 1.5, 2.5, -2.5]   # tests/test_quant.c:47-60
    x[32:64] = 1e-37                         # :64-70
    q, d = kb.quantize_q8(x)
    assert d[0] == 1.0 and q[1:6].tolist() == [1, -1, 2, 3, -3]
    assert d[1] == 0.0 and (q[32:] == 0).all()


@pytest.mark.parametrize("n", [64, 288, 2048, 4096])
def test_rmsnorm_quantize(n):
    rng = np.random.default_rng(n)
    x = rng.standard_normal(n).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(n)).astype(np.float32)
    q, d, xn = kb.rmsnorm_quantize(x, w, 1e-5)
    ref = oracle.rmsnorm(x, w, 1e-5)
    # the sum of squares is reduced in another order: normalized values agree to float rounding
    assert np.abs(xn - ref).max() <= 1e-6 * np.abs(ref).max()
    # the quantization of the kernel's own normalized values is the reference rule, bit for bit
    rq, rd = oracle.quantize_q8(xn)
    assert np.array_equal(q, rq) and np.array_equal(d.view(np.uint32), rd.view(np.uint32))


def make_w(rng, wtype, rows, cols, unit=False, f16=False):
    wq = (rng.integers(-127, 128, rows * cols).astype(np.int8) if wtype == kb.Q8_0
          else rng.integers(0, 256, rows * cols // 2).astype(np.uint8))
    if unit:
        wd = np.ones((rows, cols // 32), np.float32)
    else:
        wd = (rng.uniform(0.001, 0.05, (rows, cols // 32)) * rng.choice([-1, 1], (rows, cols // 32))).astype(np.float32)
    if f16:
        wd = wd.astype(np.float16)
    return wq, wd


def term_scale(wtype, wq, wd, rows, cols, xq, xd):
    """Sum of |w x d_w d_x| per row (ref_scale of tests/test_kernels.c:64-83)."""
    if wtype == kb.Q8_0:
        w = wq.reshape(rows, -1, 32).astype(np.int64)
    else:
        p = wq.reshape(rows, -1, 16).astype(np.int64)
        w = np.concatenate([(p & 15) - 8, (p >> 4) - 8], -1)
    a = np.abs(w * xq.reshape(-1, 32)).sum(-1).astype(np.float64)
    return (a * np.abs(wd.astype(np.float64)) * np.abs(xd)).sum(1)


SHAPES = [(1, 32), (3, 96), (4, 256), (7, 288), (64, 896), (5, 8288), (333, 2048), (2048, 8192)]


@pytest.mark.parametrize("wtype", [kb.Q8_0, kb.Q4_0])
@pytest.mark.parametrize("rows,cols", SHAPES)
def test_block_sums_bit_exact(wtype, rows, cols):
    rng = np.random.default_rng(rows * 131 + cols)
    wq, _ = make_w(rng, wtype, rows, cols)
    xq = rng.integers(-127, 128, cols).astype(np.int8)
    assert np.array_equal(kb.block_sums(wtype, wq, rows, cols, xq), oracle.block_sums(wtype, wq, rows, cols, xq))


@pytest.mark.parametrize("wtype", [kb.Q8_0, kb.Q4_0])
@pytest.mark.parametrize("rows,cols", SHAPES)
def test_matvec_unit_scales_exact(wtype, rows, cols):
    # exact while every partial sum stays below 2^24: |w x| <= 127*127 (Q8) or 8*127 (Q4) per element
    if wtype == kb.Q8_0 and cols * 127 * 127 >= 1 << 24:
        pytest.skip("float partial sums could round")
    rng = np.random.default_rng(rows + cols)
    wq, wd = make_w(rng, wtype, rows, cols, unit=True)
    xq = rng.integers(-127, 128, cols).astype(np.int8)
    xd = np.ones(cols // 32, np.float32)
    y = kb.matvec(wtype, wq, wd, rows, cols, xq, xd)
    exact = oracle.block_sums(wtype, wq, rows, cols, xq).astype(np.int64).sum(1)
    assert np.array_equal(y, exact.astype(np.float32))


@pytest.mark.parametrize("f16", [False, True])
@pytest.mark.parametrize("wtype", [kb.Q8_0, kb.Q4_0])
@pytest.mark.parametrize("rows,cols", SHAPES)
def test_matvec_scaled(wtype, rows, cols, f16):
    rng = np.random.default_rng(3 * rows + cols + f16)
    wq, wd = make_w(rng, wtype, rows, cols, f16=f16)
    xq = rng.integers(-127, 128, cols).astype(np.int8)
    xd = rng.uniform(0.001, 0.05, cols // 32).astype(np.float32)
    y = kb.matvec(wtype, wq, wd, rows, cols, xq, xd)
    ref = oracle.matvec(wtype, wq, wd.astype(np.float32), rows, cols, xq, xd)
    sc = term_scale(wtype, wq, wd, rows, cols, xq, xd)
    tol = 1e-5 * np.maximum(sc, np.maximum(np.abs(y), np.abs(ref)))
    assert (np.abs(y.astype(np.float64) - ref) <= tol).all()


MM_SHAPES = [(1, 32, 1), (7, 288, 5), (64, 896, 33), (333, 2048, 70), (2048, 8192, 40), (130, 14336, 3)]


@pytest.mark.parametrize("wtype", [kb.Q8_0, kb.Q4_0])
@pytest.mark.parametrize("rows,cols,n", MM_SHAPES)
def test_matmul_unit_scales_exact(wtype, rows, cols, n):
    # ml_matmul (ops/ops.c:51-79) on the int8 tensor cores: every block dot is an
    # exact int32, so with unit scales each row sum is exact below 2^24
    if wtype == kb.Q8_0 and cols * 127 * 127 >= 1 << 24:
        pytest.skip("float partial sums could round")
    rng = np.random.default_rng(rows * 7 + cols + n)
    wq, wd = make_w(rng, wtype, rows, cols, unit=True)
    xq = rng.integers(-127, 128, (n, cols)).astype(np.int8)
    xd = np.ones((n, cols // 32), np.float32)
    y = kb.matmul(wtype, wq, wd, rows, cols, xq, xd)
    for t in range(n):
        exact = oracle.block_sums(wtype, wq, rows, cols, xq[t]).astype(np.int64).sum(1)
        assert np.array_equal(y[t], exact.astype(np.float32)), t


@pytest.mark.parametrize("f16", [False, True])
@pytest.mark.parametrize("wtype", [kb.Q8_0, kb.Q4_0])
@pytest.mark.parametrize("rows,cols,n", MM_SHAPES)
def test_matmul_scaled(wtype, rows, cols, n, f16):
    # per token the reference's matvec within TT_CLOSE (1e-5 of the sum of |terms|)
    rng = np.random.default_rng(5 * rows + cols + n + f16)
    wq, wd = make_w(rng, wtype, rows, cols, f16=f16)
    xq = rng.integers(-127, 128, (n, cols)).astype(np.int8)
    xd = rng.uniform(0.001, 0.05, (n, cols // 32)).astype(np.float32)
    y = kb.matmul(wtype, wq, wd, rows, cols, xq, xd)
    for t in range(n):
        ref = oracle.matvec(wtype, wq, wd.astype(np.float32), rows, cols, xq[t], xd[t])
        sc = term_scale(wtype, wq, wd, rows, cols, xq[t], xd[t])
        tol = 1e-5 * np.maximum(sc, np.maximum(np.abs(y[t]), np.abs(ref)))
        assert (np.abs(y[t].astype(np.float64) - ref) <= tol).all(), t


def test_matmul_rejects_bad_shapes():
    assert kb.lib().kc_matmul_dev(None, kb.Q8_0, 0, None, None, 4, 33, None, None, 1, None) == kb.E_SHAPE
    assert kb.lib().kc_matmul_dev(None, kb.Q8_0, 0, None, None, 4, 32, None, None, 0, None) == kb.E_SHAPE


def test_matvec_wait_timeout_is_reported():
    """A kernel-level matvec whose first wait on each chunk of weights gives up
    at once (kc_debug_wait_limit 0) runs out of it: the device error word is
    flagged, the wait then drains the chunk (the result stays right), the next
    kc_dev_sync returns KC_E_IO with the reason and clears the word, and a call
    with the default limit afterwards syncs clean. No fault is involved."""
    rows, cols = 2048, 8192
    rng = np.random.default_rng(11)
    wq, wd = make_w(rng, kb.Q4_0, rows, cols, f16=True)
    xq = rng.integers(-127, 128, cols).astype(np.int8)
    xd = rng.uniform(0.001, 0.05, cols // 32).astype(np.float32)
    want = kb.matvec(kb.Q4_0, wq, wd, rows, cols, xq, xd)
    bw, bd = kb.DevBuf.of(wq), kb.DevBuf.of(wd, pad=16)
    bxq, bxd, by = kb.DevBuf.of(xq), kb.DevBuf.of(xd), kb.DevBuf(4 * rows)
    L = kb.lib()
    try:
        assert L.kc_debug_wait_limit(0) == kb.OK
        assert L.kc_matvec_dev(by.ptr, kb.Q4_0, 1, bw.ptr, bd.ptr, rows, cols, bxq.ptr, bxd.ptr, None) == kb.OK
        assert L.kc_dev_sync() == kb.E_IO
        assert "gave up" in kb.what_detail()
    finally:
        L.kc_debug_wait_limit(-1)
    assert np.array_equal(by.get(np.float32, rows), want)
    assert L.kc_dev_sync() == kb.OK   # the word was cleared by the report
    assert L.kc_matvec_dev(by.ptr, kb.Q4_0, 1, bw.ptr, bd.ptr, rows, cols, bxq.ptr, bxd.ptr, None) == kb.OK
    assert L.kc_dev_sync() == kb.OK
    assert np.array_equal(by.get(np.float32, rows), want)
