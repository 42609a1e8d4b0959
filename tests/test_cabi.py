"""The C-ABI library loads and exports every symbol include/tensorgrad_b200.h
declares; error plumbing works without a GPU (no compute calls)."""
import ctypes
import os
import re

import pytest

from tensorgrad_b200 import backend as BK
from tensorgrad_b200.build import build

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def lib():
    build()
    return BK.load()


def declared():
    src = open(os.path.join(ROOT, "include", "tensorgrad_b200.h")).read()
    return sorted(set(re.findall(r"\b(tg_[a-z_]+)\s*\(", src)))


def test_all_declared_symbols_exported(lib):
    names = declared()
    assert len(names) >= 20
    for n in names:
        assert hasattr(lib, n), n
    assert set(BK.EXPORTED) == set(names)


def test_error_plumbing_without_gpu(lib):
    h = ctypes.c_void_p()
    rc = lib.tg_ctx_create(0, 0, 1, None, ctypes.byref(h))
    if rc == 0:
        pytest.skip("a GPU is visible; covered by the GPU tests")
    assert lib.tg_last_error_name().decode() == "CudaError"
    assert lib.tg_last_error_message().decode()
    assert lib.tg_graph_info(None, 1, None, 0, None) != 0
    assert lib.tg_last_error_name().decode() == "Error"
