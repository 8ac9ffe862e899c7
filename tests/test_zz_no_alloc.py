"""kc_matvec_f32_noalloc: the matvec from a float activation whose quantized
activation lives in the library's static device scratch. It must give the
results of the allocating entry points (kc_quantize_q8_dev then
kc_matvec_dev), call after call, allocate no device memory, and refuse sizes
beyond its scratch. Collected last so that it also runs after every other GPU
test; it passes alone in a fresh process as well."""
import ctypes as C

import numpy as np
import pytest

import krafla_b200 as kb

pytestmark = pytest.mark.gpu

MAX_COLS = 16384   # KC_NOALLOC_MAX_COLS in include/krafla_cuda.h
TOL = 1e-6         # relative to max|y|; the two paths run the same kernels, so they agree exactly


@pytest.fixture(scope="module", autouse=True)
def _dev(built):
    kb.device_check()


def _weights(rng, wtype, rows, cols, f16):
    wq = (rng.integers(-127, 128, rows * cols).astype(np.int8) if wtype == kb.Q8_0
          else rng.integers(0, 256, rows * cols // 2).astype(np.uint8))
    wd = (rng.uniform(0.001, 0.05, (rows, cols // 32)) * rng.choice([-1, 1], (rows, cols // 32))).astype(np.float32)
    return wq, (wd.astype(np.float16) if f16 else wd)


def _existing(bw, bd, wtype, f16, rows, cols, bx):
    bq, bxd, by = kb.DevBuf(cols), kb.DevBuf(4 * (cols // 32)), kb.DevBuf(4 * rows)
    assert kb.lib().kc_quantize_q8_dev(bq.ptr, bxd.ptr, bx.ptr, cols, None) == kb.OK
    assert kb.lib().kc_matvec_dev(by.ptr, wtype, int(f16), bw.ptr, bd.ptr, rows, cols, bq.ptr, bxd.ptr, None) == kb.OK
    assert kb.lib().kc_dev_sync() == kb.OK
    return by.get(np.float32, rows)


def _noalloc(by, bw, bd, wtype, f16, rows, cols, bx):
    st = kb.lib().kc_matvec_f32_noalloc(by.ptr, wtype, int(f16), bw.ptr, bd.ptr, rows, cols, bx.ptr, None)
    assert st == kb.OK, kb.what_detail()
    assert kb.lib().kc_dev_sync() == kb.OK
    return by.get(np.float32, rows)


@pytest.mark.parametrize("wtype,f16,rows,cols", [(kb.Q4_0, True, 1000, 2048), (kb.Q8_0, False, 333, 896),
                                                 (kb.Q4_0, False, 300, MAX_COLS)])
def test_noalloc_matches_allocating_entry_points(wtype, f16, rows, cols):
    rng = np.random.default_rng(rows + cols)
    wq, wd = _weights(rng, wtype, rows, cols, f16)
    x = rng.normal(0.0, 1.0, cols).astype(np.float32)
    bw, bd, bx = kb.DevBuf.of(wq), kb.DevBuf.of(wd, pad=16), kb.DevBuf.of(x)
    want = _existing(bw, bd, wtype, f16, rows, cols, bx)
    by = kb.DevBuf(4 * rows)
    first = _noalloc(by, bw, bd, wtype, f16, rows, cols, bx)
    second = _noalloc(by, bw, bd, wtype, f16, rows, cols, bx)   # two calls in a row reuse the scratch
    scale = float(np.abs(want).max())
    assert np.abs(first.astype(np.float64) - want).max() <= TOL * scale
    assert np.abs(second.astype(np.float64) - want).max() <= TOL * scale


def test_noalloc_allocates_nothing():
    torch = pytest.importorskip("torch")
    rows, cols = 512, 4096
    rng = np.random.default_rng(7)
    wq, wd = _weights(rng, kb.Q4_0, rows, cols, True)
    bw, bd = kb.DevBuf.of(wq), kb.DevBuf.of(wd, pad=16)
    bx, by = kb.DevBuf.of(rng.normal(0.0, 1.0, cols).astype(np.float32)), kb.DevBuf(4 * rows)
    _noalloc(by, bw, bd, kb.Q4_0, True, rows, cols, bx)            # set-up call
    free0 = torch.cuda.mem_get_info()[0]
    for _ in range(5):
        _noalloc(by, bw, bd, kb.Q4_0, True, rows, cols, bx)
    assert torch.cuda.mem_get_info()[0] == free0


def test_noalloc_rejects_columns_beyond_scratch():
    rows, cols = 4, MAX_COLS + 32
    rng = np.random.default_rng(9)
    wq, wd = _weights(rng, kb.Q8_0, rows, cols, False)
    bw, bd, bx = kb.DevBuf.of(wq), kb.DevBuf.of(wd, pad=16), kb.DevBuf.of(np.ones(cols, np.float32))
    sentinel = np.full(rows, 123.0, np.float32)
    by = kb.DevBuf.of(sentinel)
    st = kb.lib().kc_matvec_f32_noalloc(by.ptr, kb.Q8_0, 0, bw.ptr, bd.ptr, rows, cols, bx.ptr, None)
    assert st == kb.E_SHAPE
    assert "scratch" in kb.what_detail()
    assert np.array_equal(by.get(np.float32, rows), sentinel)   # nothing launched
