"""Pinned event rings for many independent streams, and the paced replay
producer that feeds them (include/ssla_b200.h: SslaLiveRing,
ssla_engine_rings_attach / drain_rings / serve_rings, ssla_replay_*).

A ``RingSet`` holds n rings in the SslaLiveRing layout -- the raw-event
counterpart of the reference's pinned GPU rings (``RingBuffer`` /
``PinnedRing``, orin/orin/ring.py:34-152; SPSC head / tail words,
include/spsc.h:9-11): events [n][capacity][4] float32 (t, x, y, p), the
words head / tail / events_done / stop per ring, and per-slot outputs flags
[n][capacity] and decoded prediction rows preds [n][capacity][cols].
"""
from __future__ import annotations

import ctypes as C
from typing import Sequence

import numpy as np

from . import abi
from .engine import SslaError, load_library


class RingSet:
    """n rings of ``capacity`` slots (a power of two).  ``pinned`` buffers
    (page-locked, device-mapped; needs CUDA) are what an engine drains;
    plain host memory serves host-only producers and consumers."""

    def __init__(self, n: int, capacity: int, cols: int = 7, flags: bool = True, preds: bool = True,
                 pinned: bool = True):
        if n < 1 or capacity < 2 or capacity & (capacity - 1):
            raise ValueError("n >= 1 rings, capacity a power of two >= 2")
        self.n, self.capacity, self.cols = n, capacity, cols
        self._keep = []

        def alloc(shape, dtype):
            if pinned:
                import torch
                tdt = {np.float32: torch.float32, np.uint8: torch.uint8, np.int64: torch.int64}[dtype]
                t = torch.zeros(shape, dtype=tdt).pin_memory()
                self._keep.append(t)
                return t.numpy()
            a = np.zeros(shape, dtype=dtype)
            self._keep.append(a)
            return a

        self.events = alloc((n, capacity, 4), np.float32)
        self.words = alloc((n, 4), np.int64)          # head, tail, events_done, stop
        self.flags = alloc((n, capacity), np.uint8) if flags else None
        self.preds = alloc((n, capacity, cols), np.float32) if preds else None
        self.descs = (abi.SslaLiveRing * n)()
        ev0, w0 = self.events.ctypes.data, self.words.ctypes.data
        for r in range(n):
            w = w0 + 32 * r
            self.descs[r] = abi.SslaLiveRing(
                ev0 + 16 * capacity * r, capacity, w, w + 8, w + 16,
                None if self.flags is None else self.flags.ctypes.data + capacity * r,
                None if self.preds is None else self.preds.ctypes.data + 4 * cols * capacity * r,
                w + 24)

    def head(self, r: int) -> int:
        return int(self.words[r, 0])

    def tail(self, r: int) -> int:
        return int(self.words[r, 1])

    def done(self, r: int) -> int:
        return int(self.words[r, 2])


class Replay:
    """ssla_replay_*: a native thread publishing ``streams[r]`` (float32
    rows t, x, y, p; t in microseconds) into ring r at their timestamps,
    time_scale wall microseconds per event microsecond (0: as fast as ring
    space allows), event time 0 at CLOCK_MONOTONIC ``start_ns`` (0: 2 ms
    after the start)."""

    def __init__(self, rings: RingSet, streams: Sequence[np.ndarray], time_scale: float = 1.0,
                 start_ns: int = 0):
        if len(streams) != rings.n:
            raise ValueError("one stream per ring")
        self.lib = load_library()
        self._rings = rings
        self._ev = [np.ascontiguousarray(s, dtype=np.float32).reshape(-1, 4) for s in streams]
        self._ptrs = (C.c_void_p * rings.n)(*[e.ctypes.data for e in self._ev])
        self._counts = np.array([len(e) for e in self._ev], dtype=np.uint64)
        h = self.lib.ssla_replay_start(C.addressof(rings.descs), rings.n, C.addressof(self._ptrs),
                                       self._counts.ctypes.data, float(time_scale), int(start_ns))
        if not h:
            raise SslaError(abi.SSLA_ERR_ARG, self.lib.ssla_last_error().decode())
        self.h = h

    def stop(self) -> None:
        if self.h:
            self.lib.ssla_replay_stop(self.h)

    def __del__(self):
        if getattr(self, "h", None):
            self.stop()
            self.join()

    def join(self) -> dict:
        """Waits for every event to be published (or the stop); returns the
        producer's statistics."""
        st = abi.SslaReplayStats()
        rc = self.lib.ssla_replay_join(self.h, C.byref(st))
        self.h = None
        if rc != abi.SSLA_OK:
            raise SslaError(rc, self.lib.ssla_last_error().decode())
        return {"published": st.published, "start_ns": st.start_ns, "max_lag_ns": st.max_lag_ns,
                "full_waits": st.full_waits}
