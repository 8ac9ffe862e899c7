"""The .mlb loader of the CUDA build (kc_model_load, host side only: no GPU).

Mirrors the reference's tests/test_load.c:89-284: a valid file loads with the
header the reference reads; patched files (truncated, bad magic, bad shapes,
Q8 quants of -128, bad RoPE / q8_mask / attention fields) are refused with
the reference's status codes.
"""
import os
import struct

import numpy as np
import pytest

from conftest import GOLDEN

import krafla_b200 as kb


@pytest.fixture(scope="module", autouse=True)
def _built(built):
    return built


def load(path):
    return kb.Model(path, upload=False)


def status_of(path):
    try:
        load(path).free()
        return kb.OK
    except kb.KraflaError as e:
        return e.status


def patched(tmp_path, src, edits=(), truncate=None, name="p.mlb"):
    data = bytearray(open(src, "rb").read())
    for off, fmt, val in edits:
        struct.pack_into(fmt, data, off, val)
    if truncate is not None:
        data = data[:truncate]
    p = tmp_path / name
    p.write_bytes(bytes(data))
    return str(p)


SRC = os.path.join(GOLDEN, "models", "bias_q4.mlb")
Q8 = os.path.join(GOLDEN, "models", "rand_q8.mlb")


def test_valid_header():
    c = load(SRC).config
    assert (c["dim"], c["n_layers"], c["n_heads"], c["n_kv_heads"], c["hidden_dim"], c["vocab"]) == (64, 2, 4, 2, 128, 96)
    assert c["head_dim"] == 16 and c["q_dim"] == 64 and c["kv_dim"] == 32 and c["qkv_bias"] == 1
    assert abs(c["attn_scale"] - 0.25) < 1e-7 and c["embed_scale"] == 1.0


def test_missing_file(tmp_path):
    assert status_of(str(tmp_path / "nope.mlb")) == kb.E_IO


@pytest.mark.parametrize("cut", [10, 255, 300, 20000])
def test_truncated(tmp_path, cut):
    assert status_of(patched(tmp_path, SRC, truncate=cut)) == kb.E_FORMAT


def test_bad_magic_and_version(tmp_path):
    assert status_of(patched(tmp_path, SRC, [(0, "4s", b"MLB2")])) == kb.E_FORMAT
    assert status_of(patched(tmp_path, SRC, [(4, "<I", 2)])) == kb.E_FORMAT


@pytest.mark.parametrize("off,val", [(8, 0), (8, 70000), (28, 2), (24, 100), (8, 65), (16, 3)])
def test_bad_shapes(tmp_path, off, val):
    assert status_of(patched(tmp_path, SRC, [(off, "<I", val)])) == kb.E_SHAPE


@pytest.mark.parametrize("off,fmt,val", [(44, "<I", 3), (72, "<I", 128), (76, "<I", 2), (84, "<I", 2), (104, "<I", 2),
                                         (120, "<I", 2), (52, "<I", 7), (52, "<I", 1), (88, "<f", 1.5),
                                         (112, "<f", -1.0), (124, "<f", float("nan"))])
def test_bad_fields(tmp_path, off, fmt, val):
    assert status_of(patched(tmp_path, SRC, [(off, fmt, val)])) == kb.E_FORMAT


def test_q8_minus_128_refused(tmp_path):
    # model/mlb.c:34-36: a Q8 quant of -128 has no int8 negation
    assert status_of(patched(tmp_path, Q8, [(256 + 5, "<B", 0x80)])) == kb.E_FORMAT


def test_llama3_rope_fields_round_trip():
    c = load(os.path.join(GOLDEN, "models", "llama3_q4.mlb")).config
    assert c["rope_type"] == 1 and c["rope_factor"] == 32.0 and c["rope_orig_max_seq"] == 8
    assert c["scale_f16"] == 1


def test_all_golden_models_load():
    for f in os.listdir(os.path.join(GOLDEN, "models")):
        m = load(os.path.join(GOLDEN, "models", f))
        assert m.config["vocab"] > 2
        m.free()


def test_written_model_loads(tmp_path):
    p = str(tmp_path / "w.mlb")
    kb.write_model(p, dim=64, n_layers=2, n_heads=4, n_kv_heads=2, hidden_dim=128, vocab=100, max_seq=32,
                   wtype="q4", q8=("v", "o", "down"), shared=1, qkv_bias=1, rope_scaling=("llama3", 32.0, 1.0, 4.0, 8192))
    c = load(p).config
    assert c["wtype"] == 2 and c["q8_mask"] == 88 and c["qkv_bias"] == 1 and c["rope_type"] == 1
    assert np.isclose(c["rope_theta"], 10000.0)
