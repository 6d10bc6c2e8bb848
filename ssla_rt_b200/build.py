"""Builds libssla_b200.so in-tree (nvcc, sm_100a).

The library is a plain C-ABI shared object (include/ssla_b200.h); the CUDA
runtime is linked statically so the .so needs only the driver on the GPU box.
Flags: -fmad=false keeps every floating-point contraction explicit (the
kernels write fmaf where the reference's arithmetic is a fused
multiply-add), which is what makes results bit-identical to the CPU oracle.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libssla_b200.so")
# The same library under the reference's name, for callers that load the
# s01g_* ABI as libstage01_to_gpu.so (orin/orin/hybrid_common.py S01gAPI).
S01G_LIB = os.path.join(HERE, "libstage01_to_gpu.so")
SOURCES = ["ssla_kernels.cu", "ssla_engine.cu", "ssla_weights.cpp", "ssla_noalloc.cu", "ssla_s01g.cpp", "ssla_step.cu", "ssla_live.cu", "ssla_dump.cpp", "ssla_strip.cu", "ssla_rings.cu", "ssla_replay.cpp", "ssla_head_tc.cu"]
HEADERS = ["ssla_device.cuh", "ssla_kernels.cuh", "ssla_weights.h", "ssla_cluster.cuh"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a",
              "-lineinfo", "-fmad=false", "-Xcompiler", "-fPIC", "-shared",
              "-cudart", "static"]


def _nvcc() -> str:
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if c and (os.path.isabs(c) and os.path.exists(c) or not os.path.isabs(c)):
            return c
    return "nvcc"


def _stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = [os.path.join(CSRC, f) for f in SOURCES + HEADERS]
    deps += [os.path.join(REPO, "include", f) for f in ("ssla_b200.h", "ssla_abi_types.h", "stage01_to_gpu.h")]
    return any(os.path.getmtime(d) > t for d in deps) or not os.path.exists(S01G_LIB)


# The stage-2/3 ring consumer module (kernels/), prebuilt for sm_100a: the
# same source the reference's runners NVRTC-compile, loadable by name.
KERNELS = os.path.join(HERE, "kernels")
CONSUMER_SRC = os.path.join(KERNELS, "ssla_s2_s3_head_celled.cuh")
CONSUMER_HDR = os.path.join(KERNELS, "proto_layer_pair.cuh")
CONSUMER_CUBIN = os.path.join(HERE, "ssla_s2s3_consumer.cubin")


def build_consumer(force: bool = False, verbose: bool = False) -> str:
    if (not force and os.path.exists(CONSUMER_CUBIN) and
            os.path.getmtime(CONSUMER_CUBIN) >= max(os.path.getmtime(CONSUMER_SRC), os.path.getmtime(CONSUMER_HDR))):
        return CONSUMER_CUBIN
    cmd = [_nvcc(), "-x", "cu", "-cubin", "-O3", "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a",
           "-lineinfo", f"-I{KERNELS}", CONSUMER_SRC, "-o", CONSUMER_CUBIN]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    return CONSUMER_CUBIN


def build(force: bool = False, verbose: bool = False) -> str:
    build_consumer(force=force, verbose=verbose)
    if not force and not _stale():
        return LIB
    cmd = [_nvcc(), *NVCC_FLAGS, f"-I{os.path.join(REPO, 'include')}", f"-I{CSRC}",
           *[os.path.join(CSRC, f) for f in SOURCES], "-o", LIB]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    shutil.copyfile(LIB, S01G_LIB)
    os.chmod(S01G_LIB, 0o755)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
    print(LIB)
