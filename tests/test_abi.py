"""The C-ABI boundary: libkrafla_cuda.so loads on a machine without a GPU and
exports every function include/krafla_cuda.h declares; the status strings
follow the reference's ml_status (core/ml.h:7-14)."""
import ctypes as C
import os
import re

import pytest

from conftest import ROOT

import krafla_b200 as kb

HEADER = os.path.join(ROOT, "include", "krafla_cuda.h")


@pytest.fixture(scope="module", autouse=True)
def _built(built):
    return built


def declared():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(kc_[a-z0-9_]+)\s*\(", src)))


def test_every_declared_symbol_is_exported():
    lib = C.CDLL(kb.LIB_PATH)
    names = declared()
    assert len(names) >= 20
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_status_strings():
    lib = kb.lib()
    assert lib.kc_status_str(kb.OK) == b"ok"
    assert lib.kc_status_str(kb.E_SHAPE) == b"bad tensor shape"
    assert lib.kc_status_str(kb.E_NOMEM) == b"out of memory"


def test_no_device_is_an_isa_error_not_a_crash():
    if os.path.exists("/dev/nvidia0"):
        pytest.skip("a GPU is present")
    assert kb.lib().kc_device_check() == kb.E_ISA
