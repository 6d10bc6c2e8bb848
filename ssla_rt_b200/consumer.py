"""Loader of the B200 stage-2/3 ring consumer module (ssla_rt_b200/kernels/).

The reference's runners NVRTC-compile ``ssla_s2_s3_head_celled.cuh`` with
``proto_layer_pair.cuh`` from one directory and launch four kernels by name
(orin/orin/nvrtc_util.py:74-208, orin/bench_s2_s3_head_celled.py:195-244,
orin/hybrid_runner_multi.py:465-557).  This module offers the same module
both ways -- compiled here by NVRTC with the runners' options, or loaded
from the prebuilt sm_100a image that ssla_rt_b200/build.py writes -- and a
launcher with the runners' launch shape: one block of 288 threads per ring
and the dynamic shared memory the runners compute.  It uses cuda-python's
driver and NVRTC bindings, as the runners do.
"""
from __future__ import annotations

import ctypes as C
import os
from typing import Optional, Sequence

HERE = os.path.dirname(os.path.abspath(__file__))
KERNELS_DIR = os.path.join(HERE, "kernels")
SOURCE = os.path.join(KERNELS_DIR, "ssla_s2_s3_head_celled.cuh")
HEADER = os.path.join(KERNELS_DIR, "proto_layer_pair.cuh")
CUBIN = os.path.join(HERE, "ssla_s2s3_consumer.cubin")
ENTRY_POINTS = ("k_ssla_s2s3_celled_drain_n", "k_ssla_s2s3_celled_drain_n_multi",
                "k_ssla_s2s3_celled_persistent", "k_ssla_s2s3_celled_persistent_multi")
THREADS = 288                      # 9 warps: one per patch-cell owner class
BATCH = 8


def reference_smem_bytes() -> int:
    """The dynamic shared memory the reference's runners pass
    (orin/bench_s2_s3_head_celled.py:89-108): batch slots, contribution
    staging, per-warp scratch, task lists and layer 4's qvg block."""
    out_max, n_warps, c1, c2 = 96, 9, 24, 48
    event_slot = out_max * 4 + out_max * 4 + 5 * 4 + 4 + 8 + 8
    smem = (event_slot * BATCH + BATCH * n_warps * out_max * 4 + 2 * n_warps * out_max * 4
            + 2 * n_warps * BATCH * 4 + n_warps * 4 + 2 * BATCH * 4 + 9 * 3 * c2 * c1 * 4)
    return ((smem + 15) // 16) * 16


def _drv():
    from cuda.bindings import driver
    return driver


def _check(err, what: str) -> None:
    d = _drv()
    if int(err) != int(d.CUresult.CUDA_SUCCESS):
        raise RuntimeError(f"{what} failed: {err}")


def nvrtc_compile(arch: str = "compute_100a", options: Optional[Sequence[str]] = None) -> bytes:
    """PTX of the module, compiled by NVRTC with the runners' default options
    (--gpu-architecture, -std=c++17, --use_fast_math) unless given."""
    from cuda.bindings import nvrtc
    src = open(SOURCE).read().encode()
    hdr = open(HEADER).read().encode()
    opts = [o.encode() for o in (options or (f"--gpu-architecture={arch}", "-std=c++17", "--use_fast_math"))]
    err, prog = nvrtc.nvrtcCreateProgram(src, b"ssla_s2_s3_head_celled.cu", 1, [hdr], [b"proto_layer_pair.cuh"])
    if err != nvrtc.nvrtcResult.NVRTC_SUCCESS:
        raise RuntimeError(f"nvrtcCreateProgram: {err}")
    try:
        err, = nvrtc.nvrtcCompileProgram(prog, len(opts), opts)
        if err != nvrtc.nvrtcResult.NVRTC_SUCCESS:
            _, n = nvrtc.nvrtcGetProgramLogSize(prog)
            log = b" " * n
            nvrtc.nvrtcGetProgramLog(prog, log)
            raise RuntimeError("NVRTC compile failed:\n" + log.decode(errors="replace"))
        _, n = nvrtc.nvrtcGetPTXSize(prog)
        ptx = b" " * n
        nvrtc.nvrtcGetPTX(prog, ptx)
        return ptx
    finally:
        nvrtc.nvrtcDestroyProgram(prog)


class ConsumerModule:
    """The four kernels, loaded into the current CUDA context (the one torch
    or the runner made current).  image: PTX from nvrtc_compile(), or None
    for the prebuilt sm_100a cubin."""

    def __init__(self, image: Optional[bytes] = None):
        d = _drv()
        if image is None:
            if not os.path.exists(CUBIN):
                raise RuntimeError(f"{CUBIN} missing: build it with `python ssla_rt_b200/build.py`")
            image = open(CUBIN, "rb").read()
        err, self.mod = d.cuModuleLoadData(image)
        _check(err, "cuModuleLoadData")
        self.fn = {}
        for name in ENTRY_POINTS:
            err, f = d.cuModuleGetFunction(self.mod, name.encode())
            _check(err, f"cuModuleGetFunction({name})")
            self.fn[name] = f

    def close(self) -> None:
        if getattr(self, "mod", None) is not None:
            _drv().cuModuleUnload(self.mod)
            self.mod = None

    def global_ptr(self, name: str):
        """(device address, bytes) of a module global (ssla_consumer_idle_ns,
        ssla_consumer_status)."""
        err, ptr, size = _drv().cuModuleGetGlobal(self.mod, name.encode())
        _check(err, f"cuModuleGetGlobal({name})")
        return int(ptr), int(size)

    def launch(self, name: str, grid: int, args: Sequence, smem: Optional[int] = None, stream: int = 0) -> None:
        """Launches `name` with the runners' shape: grid blocks of 288
        threads and `smem` bytes of dynamic shared memory (the reference's
        size by default).  args: ctypes scalars in parameter order."""
        d = _drv()
        smem = reference_smem_bytes() if smem is None else smem
        f = self.fn[name]
        _check(d.cuFuncSetAttribute(f, d.CUfunction_attribute.CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES,
                                    smem)[0], "cuFuncSetAttribute")
        keep = list(args)
        addrs = (C.c_void_p * len(keep))(*[C.addressof(a) for a in keep])
        st = stream if isinstance(stream, d.CUstream) else d.CUstream(int(stream))
        _check(d.cuLaunchKernel(f, grid, 1, 1, THREADS, 1, 1, smem, st, addrs, 0)[0], f"cuLaunchKernel({name})")


def ptr(v: int) -> C.c_void_p:
    return C.c_void_p(int(v))


def i32(v: int) -> C.c_int32:
    return C.c_int32(int(v))


def u32(v: int) -> C.c_uint32:
    return C.c_uint32(int(v))


def u64(v: int) -> C.c_uint64:
    return C.c_uint64(int(v))
