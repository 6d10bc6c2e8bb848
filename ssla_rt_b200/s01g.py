"""ctypes mirror of the libstage01_to_gpu.so ABI (include/stage01_to_gpu.h),
shaped like the reference's own wrapper S01gAPI
(orin/orin/hybrid_common.py:470-602): same method names and argument
meaning, so a runner can swap the library path and keep its calls."""
from __future__ import annotations

import ctypes as C
import os
from typing import Optional, Sequence

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libstage01_to_gpu.so")


class S01gAPI:
    """One s01g handle; stages 0-1 on the GPU, records published to the
    attached host rings."""

    def __init__(self, lib_path: str = LIB_PATH):
        if not os.path.exists(lib_path):
            raise RuntimeError(f"{lib_path} missing: build it with `python ssla_rt_b200/build.py`")
        self.lib = C.CDLL(lib_path)
        L, vp, i = self.lib, C.c_void_p, C.c_int
        sig = {
            "s01g_init": (vp, [C.c_char_p, i, i, i, i]),
            "s01g_init_full": (vp, [C.c_char_p, i, i, i, i, C.c_uint]),
            "s01g_attach_gpu_rings": (None, [vp, vp, vp, vp, vp, C.c_uint64, i, i, i, i, i, i]),
            "s01g_attach_gpu_rings_multi": (None, [vp, i, C.POINTER(vp), C.POINTER(vp), C.c_uint64, i, i,
                                                   C.POINTER(i), C.POINTER(i), C.POINTER(i), C.POINTER(i)]),
            "s01g_submit_batch": (i, [vp, C.POINTER(C.c_float), i]),
            "s01g_snapshot_stats": (None, [vp, C.POINTER(C.c_double)]),
            "s01g_reset_stats": (None, [vp]),
            "s01g_start_synthetic": (None, [vp, C.c_double, i, C.c_uint64]),
            "s01g_stop_synthetic": (None, [vp]),
            "s01g_synthetic_n_pushed": (C.c_uint64, [vp]),
            "s01g_shutdown": (None, [vp]),
            "s01g_flush": (i, [vp, C.c_double]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        self.handle = None

    def init(self, weights_dir: str, n_shards: int = 1, halo: int = 2, base_core: int = -1,
             sample_cap: int = 1 << 16, shard_ring_cap: int = 1 << 16) -> None:
        self.handle = self.lib.s01g_init_full(weights_dir.encode(), n_shards, halo, base_core,
                                              sample_cap, shard_ring_cap)
        if not self.handle:
            raise RuntimeError("s01g_init returned NULL (check weights_dir / meta.json / CUDA device)")

    def attach(self, ring_buf_0, ring_head_0, ring_buf_1, ring_head_1, ring_mask, W2, H2,
               proc_lo_0, proc_hi_0, proc_lo_1, proc_hi_1) -> None:
        self.lib.s01g_attach_gpu_rings(self.handle, ring_buf_0, ring_head_0, ring_buf_1, ring_head_1,
                                       ring_mask, W2, H2, proc_lo_0, proc_hi_0, proc_lo_1, proc_hi_1)

    def attach_multi(self, ring_bufs: Sequence[int], ring_heads: Sequence[int], ring_mask: int,
                     W2: int, H2: int, x_los, x_his, y_los, y_his) -> None:
        n = len(ring_bufs)
        ia = lambda v: (C.c_int * n)(*v)  # noqa: E731
        self.lib.s01g_attach_gpu_rings_multi(self.handle, n, (C.c_void_p * n)(*ring_bufs),
                                             (C.c_void_p * n)(*ring_heads), ring_mask, W2, H2,
                                             ia(x_los), ia(x_his), ia(y_los), ia(y_his))

    def submit(self, events: np.ndarray) -> int:
        ev = np.ascontiguousarray(events, dtype=np.float32).reshape(-1, 4)
        return self.lib.s01g_submit_batch(self.handle, ev.ctypes.data_as(C.POINTER(C.c_float)), ev.shape[0])

    def snapshot(self) -> np.ndarray:
        out = np.zeros(32, dtype=np.float64)
        self.lib.s01g_snapshot_stats(self.handle, out.ctypes.data_as(C.POINTER(C.c_double)))
        return out

    def reset_stats(self) -> None:
        self.lib.s01g_reset_stats(self.handle)

    def start_synthetic(self, rate_mev: float, pin_core: int = -1, seed: int = 1) -> None:
        self.lib.s01g_start_synthetic(self.handle, rate_mev, pin_core, seed)

    def stop_synthetic(self) -> None:
        self.lib.s01g_stop_synthetic(self.handle)

    def synthetic_n_pushed(self) -> int:
        return int(self.lib.s01g_synthetic_n_pushed(self.handle))

    def flush(self, timeout_s: float = 30.0) -> bool:
        return self.lib.s01g_flush(self.handle, timeout_s) == 0

    def shutdown(self) -> None:
        if self.handle:
            self.lib.s01g_shutdown(self.handle)
            self.handle = None
