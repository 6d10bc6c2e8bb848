"""The stage-2/3 ring consumer module (ssla_rt_b200/kernels/) builds the way
the reference's runners build theirs -- NVRTC, the runners' options
(--use_fast_math, -std=c++17), for their default compute_87 and for
compute_100a -- and as the prebuilt sm_100a cubin; the reference buffer
layouts it declares are the ones the C ABI and the ctypes mirror declare
(its static_asserts hold under NVRTC).  No GPU needed."""
import ctypes as C
import os

import pytest

from ssla_rt_b200 import abi, consumer


@pytest.mark.parametrize("arch", ["compute_87", "compute_100a"])
def test_nvrtc_compiles_with_runner_options(arch):
    pytest.importorskip("cuda.bindings.nvrtc")
    ptx = consumer.nvrtc_compile(arch)
    assert len(ptx) > 1000


def test_layouts_match_ctypes_mirror():
    assert C.sizeof(abi.HybridS2S3Config) == 4616
    assert abi.INPUT_DTYPE.itemsize == 128 and abi.OUTPUT_DTYPE.itemsize == 392
    src = open(consumer.SOURCE).read()
    assert "sizeof(HybridS2S3Config) == 4616" in src and "sizeof(HybridInputRec) == 128" in src


def test_prebuilt_cubin_and_reference_launch_shape():
    assert os.path.exists(consumer.CUBIN), "run ssla_rt_b200/build.py"
    # the runners' dynamic shared memory, orin/bench_s2_s3_head_celled.py:89-108
    assert consumer.reference_smem_bytes() == 166128
    assert consumer.THREADS == 288
