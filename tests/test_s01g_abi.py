"""The libstage01_to_gpu.so ABI (include/stage01_to_gpu.h): every declared
s01g_* symbol is exported under both library names, and the reference's
NULL-handle conventions hold without a GPU (src/lib_stage01_to_gpu.cpp:
every call returns silently on a NULL handle; init returns NULL when it
cannot load)."""
import ctypes as C
import os
import re

import numpy as np
import pytest

from ssla_rt_b200 import abi, s01g
from ssla_rt_b200.engine import LIB_PATH
from conftest import REPO, gpu_available


def test_s01g_exports_match_header():
    hdr = open(os.path.join(REPO, "include", "stage01_to_gpu.h")).read()
    declared = set(re.findall(r"\b(s01g_[a-z0-9_]+)\s*\(", hdr))
    assert declared == set(abi.S01G_EXPORTED)
    for path in (LIB_PATH, s01g.LIB_PATH):
        lib = C.CDLL(path)
        for name in declared:
            assert hasattr(lib, name), (path, name)


def test_null_handle_calls_are_noops():
    api = s01g.S01gAPI()
    L = api.lib
    out = np.full(32, 7.0)
    L.s01g_snapshot_stats(None, out.ctypes.data_as(C.POINTER(C.c_double)))
    assert (out == 0.0).all()
    ev = np.zeros((4, 4), np.float32)
    assert L.s01g_submit_batch(None, ev.ctypes.data_as(C.POINTER(C.c_float)), 4) == 0
    assert L.s01g_synthetic_n_pushed(None) == 0
    assert L.s01g_flush(None, 0.01) == -1
    L.s01g_reset_stats(None)
    L.s01g_stop_synthetic(None)
    L.s01g_shutdown(None)
    L.s01g_attach_gpu_rings(None, None, None, None, None, 0, 20, 16, 0, 10, 10, 20)


def test_init_with_missing_weights_returns_null(tmp_path):
    api = s01g.S01gAPI()
    assert not api.lib.s01g_init(str(tmp_path / "nope").encode(), 4, 2, -1, 1024)


@pytest.mark.skipif(gpu_available(), reason="CPU-only behaviour")
def test_init_without_gpu_returns_null(stub_dir):
    api = s01g.S01gAPI()
    with pytest.raises(RuntimeError):
        api.init(stub_dir())
