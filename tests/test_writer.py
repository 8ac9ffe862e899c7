"""The synthetic model writer (isa-lm_b200/csrc/mlb_writer.c) against the
reference's own writer: quantization bytes of tools/mlb.py (quantize_q8,
fitted quantize_q4, f32 and f16 scales) and a whole .mlb file written by
tools/mlb.py:write_mlb from the same float weights."""
import ctypes as C
import os

import numpy as np
import pytest

from conftest import GOLDEN

import krafla_b200 as kb


@pytest.fixture(scope="module", autouse=True)
def _built(built):
    return built


def mine(x, wtype, f16):
    nb = x.size // 32
    q = np.zeros(nb * (32 if wtype == 1 else 16), np.uint8)
    d = np.zeros(nb, np.float16 if f16 else np.float32)
    st = kb.gen().kw_quantize(wtype, int(f16), x.ctypes.data_as(C.c_void_p), nb, q.ctypes.data_as(C.c_void_p),
                              d.ctypes.data_as(C.c_void_p))
    assert st == 0
    return q, d


@pytest.mark.parametrize("f16", [False, True])
def test_quantizers_equal_reference_bytes(f16):
    z = np.load(os.path.join(GOLDEN, "quant.npz"))
    tag = "f16" if f16 else "f32"
    x = z["x"]
    q8, d8 = mine(x, 1, f16)
    assert np.array_equal(q8.view(np.int8), z[f"q8_{tag}"])
    assert d8.tobytes() == z[f"d8_{tag}"].tobytes()
    q4, d4 = mine(x, 2, f16)
    assert np.array_equal(q4, z[f"q4_{tag}"])
    assert d4.tobytes() == z[f"d4_{tag}"].tobytes()


def test_model_file_equals_reference_writer(tmp_path):
    import importlib.util
    spec = importlib.util.spec_from_file_location("gen_golden_cfg", os.path.join(GOLDEN, "gen_golden.py"))
    # the config is read from the generator's source without importing the reference tools
    src = open(os.path.join(GOLDEN, "gen_golden.py")).read()
    start = src.index("WRITER_CFG = dict(")
    end = src.index("\n\n", start)
    ns = {}
    exec(src[start:end], ns)
    cfg = dict(ns["WRITER_CFG"])
    del spec
    path = tmp_path / "mine.mlb"
    kb.write_model(str(path), **cfg)
    assert path.read_bytes() == open(os.path.join(GOLDEN, "writer_tiny.mlb"), "rb").read()


def test_writer_independent_of_thread_count(tmp_path):
    cfg = dict(dim=64, n_layers=1, n_heads=2, n_kv_heads=1, hidden_dim=96, vocab=50, max_seq=16, wtype="q4",
               q8=("v",), seed=9)
    a, b = tmp_path / "a.mlb", tmp_path / "b.mlb"
    kb.write_model(str(a), nthreads=1, **cfg)
    kb.write_model(str(b), nthreads=5, **cfg)
    assert a.read_bytes() == b.read_bytes()


def test_normal_statistics():
    out = np.empty(1 << 20, np.float32)
    kb.gen().kw_normal(7, 1, 0, out.size, 0.02, out.ctypes.data_as(C.c_void_p))
    assert abs(out.mean()) < 1e-4 and abs(out.std() - 0.02) < 2e-4
