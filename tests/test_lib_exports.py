"""The C-ABI library loads on a CPU-only host, exports every symbol that
include/ssla_b200.h declares, reports a missing GPU cleanly, and its exp
(the device code's twin) is bit-identical to the oracle's restatement."""
import ctypes as C
import math
import os
import re

import numpy as np
import pytest

from ssla_rt_b200 import abi
from ssla_rt_b200.engine import LIB_PATH, SslaError, SslaEngine, load_library
from conftest import REPO, gpu_available


def test_library_built_and_loads():
    assert os.path.exists(LIB_PATH), "run __graft_entry__.build() or ssla_rt_b200/build.py"
    lib = load_library()
    assert b"sm_100a" in lib.ssla_version()


def test_exports_match_header():
    hdr = open(os.path.join(REPO, "include", "ssla_b200.h")).read()
    declared = set(re.findall(r"\b(ssla_[a-z0-9_]+)\s*\(", hdr))
    assert declared == set(abi.EXPORTED)
    lib = C.CDLL(LIB_PATH)
    for name in declared:
        assert hasattr(lib, name), name


@pytest.mark.skipif(gpu_available(), reason="CPU-only behaviour")
def test_no_device_is_a_clean_error(stub_dir):
    with pytest.raises(SslaError) as ei:
        SslaEngine(stub_dir(), n_partitions=1, max_events=16)
    assert ei.value.code == abi.SSLA_ERR_NO_DEVICE


def test_expf_twin_is_bit_identical_to_oracle(oracle_mod):
    lib = load_library()
    olib = C.CDLL(oracle_mod.ORACLE_SO)
    olib.or_expf.restype = C.c_float
    olib.or_expf.argtypes = [C.c_float]
    rng = np.random.default_rng(0)
    xs = np.concatenate([rng.uniform(-110, 95, 20000), rng.normal(0, 3, 20000),
                         [0.0, -0.0, 88.7, 88.8, -103.9, -104.0, 1e-30, -1e-30]]).astype(np.float32)
    for x in xs:
        a = lib.ssla_expf_host(float(x))
        b = olib.or_expf(float(x))
        assert np.float32(a).view(np.uint32) == np.float32(b).view(np.uint32), x


def test_expf_accuracy_vs_libm():
    lib = load_library()
    rng = np.random.default_rng(1)
    xs = np.concatenate([rng.uniform(-87, 88, 50000), rng.normal(0, 4, 50000)]).astype(np.float32)
    worst = 0.0
    for x in xs:
        got = np.float32(lib.ssla_expf_host(float(x)))
        ref = math.exp(float(x))
        if ref < 1.2e-38:       # subnormal range: absolute check
            assert abs(float(got) - ref) <= 1.5e-45 * 4
            continue
        ulp = float(np.spacing(np.float32(ref)))
        worst = max(worst, abs(float(got) - ref) / ulp)
    assert worst <= 2.0, worst


def test_noalloc_source_names_no_allocating_call():
    """The allocation-free entry point's translation unit calls nothing that
    allocates device, pinned or managed memory (comments excluded)."""
    src = open(os.path.join(REPO, "ssla_rt_b200", "csrc", "ssla_noalloc.cu")).read()
    code = re.sub(r"//[^\n]*", "", re.sub(r"/\*.*?\*/", "", src, flags=re.S))
    for name in ("cudaMalloc", "cudaFree", "cudaHostAlloc", "cudaMallocHost", "cudaMallocAsync",
                 "cudaMallocManaged", "cudaMallocPitch", "cudaMalloc3D", "cudaMallocArray", "cuMemAlloc",
                 "cuMemCreate", "malloc(", "new ", "std::vector", "torch"):
        assert name not in code, name


def test_sigmoid_twin_is_bit_identical_to_oracle(oracle_mod):
    lib = load_library()
    olib = C.CDLL(oracle_mod.ORACLE_SO)
    olib.or_sigmoidf.restype = C.c_float
    olib.or_sigmoidf.argtypes = [C.c_float]
    rng = np.random.default_rng(2)
    xs = np.concatenate([rng.uniform(-120, 120, 20000), rng.normal(0, 4, 20000),
                         [0.0, -0.0, 16.99, 17.0, 17.01, -87.9, -88.0, -88.1, 1e-30]]).astype(np.float32)
    for x in xs:
        a = np.float32(lib.ssla_sigmoidf_host(float(x)))
        b = np.float32(olib.or_sigmoidf(float(x)))
        assert a.view(np.uint32) == b.view(np.uint32), x


def test_sigmoid_accuracy():
    """Within 2.3 ulp of the exact sigmoid wherever the result is normal."""
    lib = load_library()
    rng = np.random.default_rng(3)
    xs = np.concatenate([rng.uniform(-87, 30, 60000), rng.normal(0, 4, 60000),
                         np.linspace(-17.5, 17.5, 20001)]).astype(np.float32)
    worst = 0.0
    for x in xs:
        got = np.float32(lib.ssla_sigmoidf_host(float(x)))
        ref = 1.0 / (1.0 + math.exp(-float(x)))
        if ref < 1.2e-38:
            continue
        worst = max(worst, abs(float(got) - ref) / float(np.spacing(np.float32(ref))))
    assert worst <= 2.3, worst
    assert lib.ssla_sigmoidf_host(17.0) == 1.0 and lib.ssla_sigmoidf_host(40.0) == 1.0
