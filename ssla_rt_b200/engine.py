"""Python host mirror of the C ABI (include/ssla_b200.h).

``SslaEngine`` plays the role of the reference's host objects for this path:
``deploy::SslaSPipeline`` (load / reset / per-event step, single stream,
src/ssla_kernels.cpp) and the ``s01g_*`` library (many shard streams,
src/lib_stage01_to_gpu.cpp), with all the per-event math on the GPU.
``drain_n_multi`` is the reference's P1 ``k_ssla_s2s3_celled_drain_n_multi``
contract.  There is no CPU fallback: loading fails loudly without the built
library or a CUDA device.
"""
from __future__ import annotations

import ctypes as C
import os
from typing import Optional, Sequence, Tuple

import numpy as np

from . import abi

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libssla_b200.so")
_lib = None


class SslaError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"ssla error {code}: {msg}")
        self.code = code


def load_library() -> C.CDLL:
    """Load libssla_b200.so (built by ssla_rt_b200/build.py); raises if absent."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(f"{LIB_PATH} missing: build it with `python ssla_rt_b200/build.py`")
    lib = C.CDLL(LIB_PATH)
    vp, i, f = C.c_void_p, C.c_int, C.c_float
    sig = {
        "ssla_engine_create": (i, [C.c_char_p, C.POINTER(abi.SslaEngineConfig), C.POINTER(vp)]),
        "ssla_engine_destroy": (None, [vp]),
        "ssla_engine_reset": (i, [vp, vp]),
        "ssla_engine_drain_device": (i, [vp, vp, vp, vp, vp]),
        "ssla_engine_drain_host": (i, [vp, vp, vp, vp, vp]),
        "ssla_engine_drain_host_async": (i, [vp, vp, vp, vp, vp, vp]),
        "ssla_engine_state_bytes": (i, [vp, i, i, C.POINTER(C.c_size_t)]),
        "ssla_engine_read_state": (i, [vp, i, i, i, vp, C.c_size_t]),
        "ssla_engine_write_state": (i, [vp, i, i, i, vp, C.c_size_t]),
        "ssla_engine_state_ptr": (vp, [vp, i, i, i]),
        "ssla_engine_info": (i, [vp, C.POINTER(abi.SslaEngineInfo)]),
        "ssla_engine_drain_records": (i, [vp, vp, vp, vp, i, vp, vp, vp]),
        "ssla_engine_step": (i, [vp, i, vp, vp, vp, vp]),
        "ssla_engine_step_latency": (i, [vp, i, vp, i, vp, vp]),
        "ssla_engine_live_start": (i, [vp, i, C.POINTER(abi.SslaLiveRing), C.c_uint, vp]),
        "ssla_engine_live_join": (i, [vp, C.POINTER(C.c_uint)]),
        "ssla_engine_live_withhold_completion": (i, [vp, C.c_longlong]),
        "ssla_engine_fill_s2s3_config": (i, [vp, C.POINTER(abi.HybridS2S3Config), i]),
        "ssla_engine_set_head_mode": (i, [vp, i]),
        "ssla_engine_head_status": (i, [vp, C.POINTER(C.c_uint)]),
        "ssla_engine_live_latency": (i, [vp, i, vp, i, vp, vp, vp]),
        "ssla_engine_set_owned": (i, [vp, i, i, i, i, i, vp]),
        "ssla_engine_strip_init": (i, [vp, i, i, i, i, i, i]),
        "ssla_engine_strip_recv_buffer": (i, [vp, i, C.POINTER(vp), vp]),
        "ssla_engine_strip_connect": (i, [vp, i, vp, vp]),
        "ssla_engine_strip_drain": (i, [vp, vp, i, vp, vp]),
        "ssla_strip_drain_lockstep": (i, [vp, i, vp, vp, vp, vp]),
        "ssla_engine_strip_status": (i, [vp, C.POINTER(C.c_uint)]),
        "ssla_engine_rings_attach": (i, [vp, vp, i]),
        "ssla_engine_drain_rings": (i, [vp, i, C.c_longlong, vp, C.POINTER(i), vp]),
        "ssla_engine_serve_rings": (i, [vp, i, C.c_uint64, C.c_uint, C.POINTER(abi.SslaServeLog),
                                        C.POINTER(C.c_uint64), vp]),
        "ssla_replay_start": (vp, [vp, i, vp, vp, C.c_double, C.c_uint64]),
        "ssla_replay_stop": (None, [vp]),
        "ssla_replay_join": (i, [vp, C.POINTER(abi.SslaReplayStats)]),
        "ssla_write_oracle_dump": (i, [C.c_char_p, i, i, i, vp, vp]),
        "ssla_engine_oracle_dump": (i, [vp, i, vp, i, i, C.c_char_p]),
        "ssla_s2s3_drain_n_multi": (i, [C.POINTER(abi.HybridS2S3Config), vp, vp, vp, vp, vp]),
        "ssla_s2s3_drain_n": (i, [C.POINTER(abi.HybridS2S3Config), vp, vp, i, i, vp, vp, vp, vp, vp]),
        "ssla_s2s3_gate_codes_noalloc": (i, [C.POINTER(abi.HybridS2S3Config), vp, vp, vp, vp]),
        "ssla_engine_set_profiling": (i, [vp, i]),
        "ssla_engine_phase_times": (i, [vp, vp, i, C.POINTER(C.c_int)]),
        "ssla_measure_fp32_peak": (i, [i, C.POINTER(C.c_double)]),
        "ssla_selftest_reciprocal": (i, [i, C.POINTER(C.c_ulonglong), C.POINTER(C.c_uint)]),
        "ssla_selftest_sigmoid_pair": (i, [i, C.POINTER(C.c_ulonglong), C.POINTER(C.c_uint)]),
        "ssla_expf_host": (f, [f]),
        "ssla_sigmoidf_host": (f, [f]),
        "ssla_last_error": (C.c_char_p, []),
        "ssla_version": (C.c_char_p, []),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def _check(rc: int) -> None:
    if rc != abi.SSLA_OK:
        raise SslaError(rc, load_library().ssla_last_error().decode())


def _ptr(x) -> Optional[int]:
    """Address of a numpy array or a torch tensor (None passes through)."""
    if x is None:
        return None
    if hasattr(x, "data_ptr"):
        return x.data_ptr()
    if isinstance(x, np.ndarray):
        return x.ctypes.data
    return int(x)


def _stream(stream) -> Optional[int]:
    if stream is None:
        return None
    if hasattr(stream, "cuda_stream"):
        return stream.cuda_stream
    return int(stream)


class SslaEngine:
    """One model, ``n_partitions`` independent event streams on one GPU."""

    CHANS = (12, 24, 48, 96)

    def __init__(self, weights_dir: str, *, n_partitions: int = 1, max_events: int = 65536,
                 layout: int = abi.LAYOUT_HYBRID, device: int = 0,
                 record_stage_outputs: bool = False, max_events_per_partition: int = 0):
        self.lib = load_library()
        cfg = abi.SslaEngineConfig(n_partitions, max_events, layout, device,
                                   1 if record_stage_outputs else 0, max_events_per_partition)
        h = C.c_void_p()
        _check(self.lib.ssla_engine_create(weights_dir.encode(), C.byref(cfg), C.byref(h)))
        self.h = h
        info = self.info()
        self.H, self.W, self.ncls = info.H, info.W, info.ncls
        self.n_partitions, self.max_events, self.layout = n_partitions, max_events, layout
        self.device = device

    def close(self) -> None:
        if getattr(self, "h", None):
            self.lib.ssla_engine_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def info(self) -> abi.SslaEngineInfo:
        inf = abi.SslaEngineInfo()
        _check(self.lib.ssla_engine_info(self.h, C.byref(inf)))
        return inf

    def reset(self, stream=None) -> None:
        _check(self.lib.ssla_engine_reset(self.h, _stream(stream)))

    @staticmethod
    def offsets(counts: Sequence[int]) -> np.ndarray:
        return np.concatenate([[0], np.cumsum(np.asarray(counts, dtype=np.int64))]).astype(np.int32)

    def drain(self, events, part_offsets, flags=None, stream=None) -> None:
        """Device path: ``events`` a CUDA tensor (n, 4) float32, ``flags`` an
        optional CUDA uint8 tensor (n,); asynchronous on ``stream``."""
        off = np.ascontiguousarray(part_offsets, dtype=np.int32)
        _check(self.lib.ssla_engine_drain_device(self.h, _ptr(events), off.ctypes.data,
                                                 _ptr(flags), _stream(stream)))

    def drain_host(self, events: np.ndarray, part_offsets, flags: Optional[np.ndarray] = None,
                   stream=None) -> None:
        """Host path: copies in, drains, copies flags out, synchronises."""
        off = np.ascontiguousarray(part_offsets, dtype=np.int32)
        _check(self.lib.ssla_engine_drain_host(self.h, _ptr(events), off.ctypes.data,
                                               _ptr(flags), _stream(stream)))

    def drain_host_async(self, events, part_offsets, flags=None, preds=None, stream=None) -> None:
        """Pipelined host drain: pinned ``events`` in (copied on the engine's
        copy stream, overlapping the previous drain), flags and all decoded
        predictions (``preds``: (P, cells, 5+ncls) float32, pinned) out on
        ``stream``; returns without waiting."""
        off = np.ascontiguousarray(part_offsets, dtype=np.int32)
        _check(self.lib.ssla_engine_drain_host_async(self.h, _ptr(events), off.ctypes.data, _ptr(flags),
                                                     _ptr(preds), _stream(stream)))

    def step(self, event, partition: int = 0, flag_out=None, pred_out=None, stream=None) -> None:
        """One event (4 floats t, x, y, p) through the whole path in one
        launch; outputs (device or pinned host buffers) written by the
        kernel.  Asynchronous."""
        e = np.ascontiguousarray(event, dtype=np.float32).reshape(4)
        _check(self.lib.ssla_engine_step(self.h, partition, e.ctypes.data, _ptr(flag_out), _ptr(pred_out),
                                         _stream(stream)))

    def step_latency(self, events: np.ndarray, partition: int = 0):
        """Per-event host latency (us) of ssla_engine_step + synchronize,
        measured inside the library; returns (latency_us, flags)."""
        ev = np.ascontiguousarray(events, dtype=np.float32).reshape(-1, 4)
        lat = np.zeros(ev.shape[0], dtype=np.float64)
        fl = np.zeros(ev.shape[0], dtype=np.uint8)
        _check(self.lib.ssla_engine_step_latency(self.h, partition, ev.ctypes.data, ev.shape[0],
                                                 lat.ctypes.data, fl.ctypes.data))
        return lat, fl

    def oracle_dump(self, events: np.ndarray, every: int, path: str, partition: int = 0) -> None:
        """Runs the host events through `partition` and writes the decoded
        predictions after events 0, every, 2*every, ... as an OracleRecorder
        dump (include/oracle.h:10-19)."""
        ev = np.ascontiguousarray(events, dtype=np.float32).reshape(-1, 4)
        _check(self.lib.ssla_engine_oracle_dump(self.h, partition, ev.ctypes.data, ev.shape[0], every,
                                                os.fsencode(path)))

    # ---- exact strip sharding ----
    def strip_init(self, lo: int, hi: int, band_rows: int, has_up: bool, has_down: bool, cap_rows: int) -> None:
        """Own stage-0 rows [lo, hi) of the sensor; neighbours' band rows
        exchanged per layer (one partition)."""
        _check(self.lib.ssla_engine_strip_init(self.h, lo, hi, band_rows, int(has_up), int(has_down), cap_rows))

    def strip_recv_buffer(self, side: int):
        """(device address, 64-byte IPC handle) of this engine's receive
        buffer for `side` (0 = neighbour above, 1 = below)."""
        ptr = C.c_void_p()
        handle = (C.c_ubyte * 64)()
        _check(self.lib.ssla_engine_strip_recv_buffer(self.h, side, C.byref(ptr), handle))
        return ptr.value, bytes(handle)

    def strip_connect(self, side: int, peer_ptr: Optional[int] = None, peer_handle: Optional[bytes] = None) -> None:
        """Send `side`'s rows to the neighbour's receive buffer (its opposite
        side), by device address (same process) or IPC handle."""
        h = (C.c_ubyte * 64).from_buffer_copy(peer_handle) if peer_handle is not None else None
        _check(self.lib.ssla_engine_strip_connect(self.h, side, peer_ptr, h))

    def strip_drain(self, events, n: int, flags=None, stream=None) -> None:
        """One strip drain with device-side waits for the neighbours' rows."""
        _check(self.lib.ssla_engine_strip_drain(self.h, _ptr(events), n, _ptr(flags), _stream(stream)))

    def strip_status(self) -> int:
        st = C.c_uint(0)
        _check(self.lib.ssla_engine_strip_status(self.h, C.byref(st)))
        return st.value

    def set_owned(self, partition: int, x0: int, x1: int, y0: int, y1: int, stream=None) -> None:
        """Owned stage-2 range [x0, x1) x [y0, y1) of a partition (the rest is
        halo: state only, no committed predictions)."""
        _check(self.lib.ssla_engine_set_owned(self.h, partition, x0, x1, y0, y1, _stream(stream)))

    def live_start(self, ring: "abi.SslaLiveRing", partition: int = 0, idle_timeout_ms: int = 2000,
                   stream=None) -> None:
        """Launches the live loop on ``ring`` (pinned host buffers) and
        returns; end it with the ring's stop flag, then ``live_join``."""
        self._live_ring = ring
        _check(self.lib.ssla_engine_live_start(self.h, partition, C.byref(ring), idle_timeout_ms,
                                               _stream(stream)))

    def live_join(self, check: bool = True) -> int:
        """Waits for the live loop to end; returns its SSLA_LIVE_* status.
        With ``check`` a bounded wait that ran out inside the loop raises
        SslaError; without it the status is returned either way."""
        st = C.c_uint(0)
        rc = self.lib.ssla_engine_live_join(self.h, C.byref(st))
        self._live_ring = None
        if check or rc != abi.SSLA_ERR_CUDA:
            _check(rc)
        return st.value

    def set_head_mode(self, mode: int) -> None:
        """abi.HEAD_EXACT (CUDA cores, bit-exact) or abi.HEAD_TENSOR (the
        head's convolutions on tcgen05 tensor cores, split TF32)."""
        _check(self.lib.ssla_engine_set_head_mode(self.h, mode))

    def head_status(self) -> int:
        """Status bits of the tensor-core head since the last call (0: fine)."""
        st = C.c_uint(0)
        _check(self.lib.ssla_engine_head_status(self.h, C.byref(st)))
        return st.value

    def fill_s2s3_config(self, cfg: "abi.HybridS2S3Config", block: int) -> None:
        """Layer 4-7 and head weight pointers of ``cfg`` (block ``block``)
        from this engine's device weights (the reference's GPU layout)."""
        _check(self.lib.ssla_engine_fill_s2s3_config(self.h, C.byref(cfg), block))

    def live_withhold_completion(self, ring_index: int) -> None:
        """Test hook of the loop's timeout path: the next live loop withholds
        the completion message of ring event ``ring_index`` (-1: none)."""
        _check(self.lib.ssla_engine_live_withhold_completion(self.h, ring_index))

    def live_latency(self, events: np.ndarray, partition: int = 0):
        """Per-event host latency (us) from publishing an event in the live
        loop's pinned ring to seeing events_done pass it, measured inside the
        library; returns (latency_us, flags, preds) with the decoded row of
        every head event."""
        ev = np.ascontiguousarray(events, dtype=np.float32).reshape(-1, 4)
        lat = np.zeros(ev.shape[0], dtype=np.float64)
        fl = np.zeros(ev.shape[0], dtype=np.uint8)
        pr = np.zeros((ev.shape[0], 5 + self.ncls), dtype=np.float32)
        _check(self.lib.ssla_engine_live_latency(self.h, partition, ev.ctypes.data, ev.shape[0],
                                                 lat.ctypes.data, fl.ctypes.data, pr.ctypes.data))
        return lat, fl, pr

    def rings_attach(self, rings) -> None:
        """One pinned ring per partition (a ``rings.RingSet``); draining
        starts at each ring's current tail."""
        if rings.n != self.n_partitions:
            raise ValueError("one ring per partition")
        self._rings = rings
        _check(self.lib.ssla_engine_rings_attach(self.h, C.addressof(rings.descs), rings.n))

    def drain_rings(self, max_per_ring: int, max_total: int = 1 << 62, stream=None) -> np.ndarray:
        """One ring drain (asynchronous); returns each ring's share."""
        taken = np.zeros(self.n_partitions, dtype=np.int32)
        n = C.c_int(0)
        _check(self.lib.ssla_engine_drain_rings(self.h, max_per_ring, max_total, taken.ctypes.data,
                                                C.byref(n), _stream(stream)))
        return taken

    def serve_rings(self, max_per_ring: int, total: int, idle_timeout_ms: int = 2000, log_cap: int = 0,
                    flags_hist: Optional[Sequence[np.ndarray]] = None, stream=None) -> dict:
        """Drains the attached rings until ``total`` events are done (or idle);
        returns {"served", "drains", "done_ns" [n], "taken" [n, P]} and fills
        ``flags_hist`` (per ring, flags by ring index since attach)."""
        P = self.n_partitions
        done = np.zeros(max(log_cap, 1), dtype=np.uint64)
        taken = np.zeros((max(log_cap, 1), P), dtype=np.int32)
        log = abi.SslaServeLog(done.ctypes.data, taken.ctypes.data, log_cap, 0, 0, None, 0)
        keep = None
        if flags_hist is not None:
            hl = len(flags_hist[0])
            if len(flags_hist) != P or any(len(h) != hl or h.dtype != np.uint8 for h in flags_hist):
                raise ValueError("flags_hist: one uint8 array per ring, all of one length")
            keep = (C.c_void_p * P)(*[h.ctypes.data for h in flags_hist])
            log.flags_hist = C.addressof(keep)
            log.hist_len = hl
        served = C.c_uint64(0)
        _check(self.lib.ssla_engine_serve_rings(self.h, max_per_ring, total, idle_timeout_ms, C.byref(log),
                                                C.byref(served), _stream(stream)))
        return {"served": served.value, "drains": log.drains, "done_ns": done[:log.n].copy(),
                "taken": taken[:log.n].copy()}

    def drain_records(self, events, part_offsets, records, records_cap: int, flags=None,
                      stream=None) -> np.ndarray:
        """Stages 0-1 only; one HybridInputRec per event passing gate 1 into
        the device buffer ``records``.  Returns the per-partition record
        offsets (synchronises)."""
        off = np.ascontiguousarray(part_offsets, dtype=np.int32)
        rec_off = np.zeros(self.n_partitions + 1, dtype=np.int32)
        _check(self.lib.ssla_engine_drain_records(self.h, _ptr(events), off.ctypes.data, _ptr(records),
                                                  records_cap, rec_off.ctypes.data, _ptr(flags),
                                                  _stream(stream)))
        return rec_off

    def _read(self, kind: int, partition: int, index: int, dtype) -> np.ndarray:
        nb = C.c_size_t()
        _check(self.lib.ssla_engine_state_bytes(self.h, kind, index, C.byref(nb)))
        out = np.empty(nb.value // np.dtype(dtype).itemsize, dtype=dtype)
        _check(self.lib.ssla_engine_read_state(self.h, kind, partition, index, out.ctypes.data, nb.value))
        return out

    def _write(self, kind: int, partition: int, index: int, values: np.ndarray) -> None:
        v = np.ascontiguousarray(values)
        _check(self.lib.ssla_engine_write_state(self.h, kind, partition, index, v.ctypes.data, v.nbytes))

    def hidden(self, layer: int, partition: int = 0) -> np.ndarray:
        return self._read(abi.STATE_HIDDEN, partition, layer, np.float32)

    def set_hidden(self, layer: int, values: np.ndarray, partition: int = 0) -> None:
        self._write(abi.STATE_HIDDEN, partition, layer, np.asarray(values, np.float32))

    def counters(self, gate: int, partition: int = 0) -> np.ndarray:
        return self._read(abi.STATE_COUNTER, partition, gate, np.uint8)

    def last_t(self, partition: int = 0) -> np.ndarray:
        return self._read(abi.STATE_LAST_T, partition, 0, np.float64)

    def preds_dec(self, partition: int = 0) -> np.ndarray:
        return self._read(abi.STATE_PREDS_DEC, partition, 0, np.float32).reshape(-1, 5 + self.ncls)

    def preds_dec_all(self) -> np.ndarray:
        """Decoded predictions of every partition, (P, cells, 5+ncls), one copy."""
        nb = C.c_size_t()
        _check(self.lib.ssla_engine_state_bytes(self.h, abi.STATE_PREDS_DEC, 0, C.byref(nb)))
        out = np.empty((self.n_partitions, nb.value // 4 // (5 + self.ncls), 5 + self.ncls), dtype=np.float32)
        _check(self.lib.ssla_engine_read_state(self.h, abi.STATE_PREDS_DEC, -1, 0, out.ctypes.data, out.nbytes))
        return out

    def preds_raw(self, partition: int = 0) -> np.ndarray:
        return self._read(abi.STATE_PREDS_RAW, partition, 0, np.float32).reshape(-1, 5 + self.ncls)

    def version(self, partition: int = 0) -> np.ndarray:
        return self._read(abi.STATE_VERSION, partition, 0, np.uint32)

    def stage_out(self, stage: int, n: int) -> np.ndarray:
        a = self._read(abi.STATE_STAGE_OUT, 0, stage, np.float32)
        return a.reshape(-1, self.CHANS[stage])[:n]

    def flags(self, n: int) -> np.ndarray:
        return self._read(abi.STATE_FLAGS, 0, 0, np.uint8)[:n]

    def set_profiling(self, on: bool) -> None:
        _check(self.lib.ssla_engine_set_profiling(self.h, 1 if on else 0))

    def phase_times(self):
        """[(name, ms, launches)] of the last profiled drain, launch order."""
        buf = (abi.SslaPhaseTime * 128)()
        n = C.c_int()
        _check(self.lib.ssla_engine_phase_times(self.h, C.cast(buf, C.c_void_p), 128, C.byref(n)))
        return [(buf[i].name.decode(), buf[i].ms, buf[i].launches) for i in range(n.value)]

    def state_ptr(self, kind: int, partition: int = 0, index: int = 0) -> int:
        return self.lib.ssla_engine_state_ptr(self.h, kind, partition, index) or 0


def measure_fp32_peak(device: int = 0) -> float:
    """Measured FP32 FFMA peak of the device in TFLOP/s."""
    v = C.c_double()
    _check(load_library().ssla_measure_fp32_peak(device, C.byref(v)))
    return v.value


def selftest_reciprocal(device: int = 0) -> Tuple[int, int]:
    """(mismatches, first mismatching bit pattern) of the device sigmoid's
    reciprocal against IEEE round-to-nearest over every float in [1, 2^126)."""
    n = C.c_ulonglong()
    first = C.c_uint()
    _check(load_library().ssla_selftest_reciprocal(device, C.byref(n), C.byref(first)))
    return n.value, first.value


def selftest_sigmoid_pair(device: int = 0) -> Tuple[int, int]:
    """(mismatches, first mismatching bit pattern) of the packed device
    sigmoid against two scalar device sigmoids over every float."""
    n = C.c_ulonglong()
    first = C.c_uint()
    _check(load_library().ssla_selftest_sigmoid_pair(device, C.byref(n), C.byref(first)))
    return n.value, first.value


def drain_n_multi(cfg: abi.HybridS2S3Config, rings: Sequence[int], ns: Sequence[int],
                  outs: Optional[Sequence[int]] = None, batch_clks: Optional[Sequence[int]] = None,
                  stream=None) -> None:
    """k_ssla_s2s3_celled_drain_n_multi contract; device pointers as ints."""
    lib = load_library()
    P = len(rings)
    r = (C.c_void_p * P)(*rings)
    n = (C.c_int * P)(*ns)
    o = (C.c_void_p * P)(*outs) if outs is not None else None
    k = (C.c_void_p * P)(*batch_clks) if batch_clks is not None else None
    _check(lib.ssla_s2s3_drain_n_multi(C.byref(cfg), C.cast(r, C.c_void_p), C.cast(n, C.c_void_p),
                                       C.cast(o, C.c_void_p) if o is not None else None,
                                       C.cast(k, C.c_void_p) if k is not None else None,
                                       _stream(stream)))


def gate_codes_noalloc(cfg: abi.HybridS2S3Config, rings: Sequence[int], ns: Sequence[int],
                       outs: Optional[Sequence[int]] = None, stream=None) -> None:
    """Allocation-free gate pass (ssla_s2s3_gate_codes_noalloc): pass2 / pass3
    codes and tdrop counter updates of a drain_n call, enqueued on `stream`."""
    lib = load_library()
    P = len(rings)
    r = (C.c_void_p * P)(*rings)
    n = (C.c_int * P)(*ns)
    o = (C.c_void_p * P)(*outs) if outs is not None else None
    _check(lib.ssla_s2s3_gate_codes_noalloc(C.byref(cfg), C.cast(r, C.c_void_p), C.cast(n, C.c_void_p),
                                            C.cast(o, C.c_void_p) if o is not None else None,
                                            _stream(stream)))


def strip_drain_lockstep(engines: Sequence["SslaEngine"], events: Sequence, flags: Optional[Sequence] = None,
                         stream=None) -> None:
    """Drains strips that share one GPU in lockstep on one stream: every
    engine's layers, then each exchange (ssla_strip_drain_lockstep)."""
    k = len(engines)
    lib = engines[0].lib
    e_arr = (C.c_void_p * k)(*[e.h.value if isinstance(e.h, C.c_void_p) else e.h for e in engines])
    ev_arr = (C.c_void_p * k)(*[_ptr(x) for x in events])
    n_arr = (C.c_int * k)(*[int(x.shape[0]) for x in events])
    f_arr = (C.c_void_p * k)(*[_ptr(f) for f in flags]) if flags is not None else None
    _check(lib.ssla_strip_drain_lockstep(e_arr, k, ev_arr, n_arr, f_arr, _stream(stream)))
