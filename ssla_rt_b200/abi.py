"""ctypes / numpy mirrors of include/ssla_abi_types.h and include/ssla_b200.h.

The reference's own mirrors are orin/orin/hybrid_common.py:30-122; these
declare the same byte layouts so a reference caller's buffers can be handed
to libssla_b200.so unchanged (tests/test_abi_layout.py pins sizes/offsets).
"""
from __future__ import annotations

import ctypes as C

import numpy as np

MAX_BLOCKS = 16
C1, C2, C3 = 24, 48, 96

INPUT_DTYPE = np.dtype([
    ("seq_done", "<u8"), ("t", "<f4"), ("x", "<u2"), ("y", "<u2"),
    ("feat1", "<f4", (C1,)), ("t_push_ns", "<u8"), ("t_emit_ns", "<u8"),
])
OUTPUT_DTYPE = np.dtype([("pass2", "<i4"), ("pass3", "<i4"), ("s3_feat", "<f4", (C3,))])
TIMING_DTYPE = np.dtype([
    ("t_pop_clk", "<u8"), ("t_done_clk", "<u8"), ("seq", "<u4"), ("owner", "<u4"),
    ("t_push_ns", "<u8"), ("t_emit_ns", "<u8"),
])
EVENT_DTYPE = np.dtype([("t", "<f4"), ("x", "<f4"), ("y", "<f4"), ("p", "<f4")])


class HybridStrip(C.Structure):
    _fields_ = [(n, C.c_int32) for n in (
        "owned_lo", "owned_hi", "s3_owned_lo", "s3_owned_hi",
        "owned_y_lo", "owned_y_hi", "s3_owned_y_lo", "s3_owned_y_hi")]


class LayerWeightsS2S3(C.Structure):
    _fields_ = [(n, C.c_uint64) for n in ("qvgIn", "goW", "input_proj", "ln_gamma", "ln_beta")]


class HybridS2S3Config(C.Structure):
    _fields_ = [
        ("H2", C.c_int32), ("W2", C.c_int32), ("H3", C.c_int32), ("W3", C.c_int32),
        ("tdrop_window", C.c_int32), ("head_out_dim", C.c_int32),
        ("n_blocks", C.c_int32), ("_pad_nblocks", C.c_int32),
        ("strip", HybridStrip * MAX_BLOCKS),
        ("layers", (LayerWeightsS2S3 * 4) * MAX_BLOCKS),
        ("hidden", (C.c_uint64 * 4) * MAX_BLOCKS),
        ("tdrop_s2", C.c_uint64 * MAX_BLOCKS),
        ("tdrop_s3", C.c_uint64 * MAX_BLOCKS),
        ("head_W", C.c_uint64), ("head_b", C.c_uint64),
        ("head_cls_conv_W", C.c_uint64), ("head_cls_conv_b", C.c_uint64),
        ("head_cls_pred_W", C.c_uint64), ("head_cls_pred_b", C.c_uint64),
        ("head_reg_conv_W", C.c_uint64), ("head_reg_conv_b", C.c_uint64),
        ("head_reg_pred_W", C.c_uint64), ("head_reg_pred_b", C.c_uint64),
        ("head_obj_pred_W", C.c_uint64), ("head_obj_pred_b", C.c_uint64),
        ("preds", C.c_uint64 * MAX_BLOCKS),
        ("version", C.c_uint64 * MAX_BLOCKS),
        ("timing", C.c_uint64 * MAX_BLOCKS),
        ("timing_mask", C.c_uint32), ("_pad_timing", C.c_uint32),
        ("kernel_start_clk", C.c_uint64 * MAX_BLOCKS),
        ("kernel_end_clk", C.c_uint64 * MAX_BLOCKS),
    ]


class SslaEngineConfig(C.Structure):
    _fields_ = [("n_partitions", C.c_int), ("max_events", C.c_int), ("layout", C.c_int),
                ("device", C.c_int), ("record_stage_outputs", C.c_int),
                ("max_events_per_partition", C.c_int)]


class SslaEngineInfo(C.Structure):
    _fields_ = [("H", C.c_int), ("W", C.c_int), ("ncls", C.c_int), ("tdrop_window", C.c_int),
                ("layout", C.c_int), ("n_partitions", C.c_int), ("max_events", C.c_int),
                ("device", C.c_int), ("stage_events", C.c_longlong * 5),
                ("launches", C.c_int), ("_pad", C.c_int)]


class SslaLiveRing(C.Structure):
    """include/ssla_b200.h SslaLiveRing: every pointer pinned host memory."""
    _fields_ = [("events", C.c_void_p), ("capacity", C.c_uint64), ("head", C.c_void_p),
                ("tail", C.c_void_p), ("events_done", C.c_void_p), ("flags", C.c_void_p),
                ("preds", C.c_void_p), ("stop_flag", C.c_void_p)]


class SslaServeLog(C.Structure):
    """include/ssla_b200.h SslaServeLog: per-drain record of ssla_engine_serve_rings."""
    _fields_ = [("done_ns", C.c_void_p), ("taken", C.c_void_p), ("cap", C.c_int), ("n", C.c_int),
                ("drains", C.c_int), ("flags_hist", C.c_void_p), ("hist_len", C.c_uint64)]


class SslaReplayStats(C.Structure):
    """include/ssla_b200.h SslaReplayStats."""
    _fields_ = [("published", C.c_uint64), ("start_ns", C.c_uint64), ("max_lag_ns", C.c_int64),
                ("full_waits", C.c_uint64)]


# SSLA_LIVE_* status bits
LIVE_ERR_WEIGHTS, LIVE_ERR_INPUT, LIVE_ERR_CONTRIB, LIVE_ERR_EVENT, LIVE_ERR_DONE = 1, 2, 4, 8, 16
LIVE_EXIT_STOP, LIVE_EXIT_IDLE = 0x100, 0x200


class SslaPhaseTime(C.Structure):
    _fields_ = [("name", C.c_char * 40), ("ms", C.c_float), ("launches", C.c_int)]


SSLA_OK, SSLA_ERR_ARG, SSLA_ERR_CUDA, SSLA_ERR_LOAD, SSLA_ERR_CAPACITY, SSLA_ERR_NO_DEVICE = range(6)
LAYOUT_DECOMP, LAYOUT_HYBRID = 0, 1
HEAD_EXACT, HEAD_TENSOR = 0, 1
F_VALID, F_R1, F_R2, F_R3, F_R4 = 1, 2, 4, 8, 16
(STATE_HIDDEN, STATE_COUNTER, STATE_LAST_T, STATE_PREDS_DEC, STATE_PREDS_RAW,
 STATE_VERSION, STATE_STAGE_OUT, STATE_FLAGS) = range(8)

# Every symbol include/ssla_b200.h declares (tests check the .so exports them).
EXPORTED = (
    "ssla_engine_create", "ssla_engine_destroy", "ssla_engine_reset",
    "ssla_engine_drain_device", "ssla_engine_drain_host", "ssla_engine_drain_host_async",
    "ssla_engine_state_bytes",
    "ssla_engine_read_state", "ssla_engine_write_state", "ssla_engine_state_ptr",
    "ssla_engine_info", "ssla_s2s3_drain_n_multi", "ssla_s2s3_drain_n",
    "ssla_engine_set_profiling", "ssla_engine_phase_times", "ssla_measure_fp32_peak", "ssla_selftest_reciprocal",
    "ssla_selftest_sigmoid_pair",
    "ssla_expf_host", "ssla_sigmoidf_host", "ssla_last_error", "ssla_version", "ssla_s2s3_gate_codes_noalloc",
    "ssla_engine_drain_records", "ssla_engine_step", "ssla_engine_step_latency",
    "ssla_engine_live_start", "ssla_engine_live_join", "ssla_engine_live_latency",
    "ssla_engine_live_withhold_completion", "ssla_engine_fill_s2s3_config",
    "ssla_engine_set_head_mode", "ssla_engine_head_status",
    "ssla_engine_set_owned", "ssla_write_oracle_dump", "ssla_engine_oracle_dump",
    "ssla_engine_strip_init", "ssla_engine_strip_recv_buffer", "ssla_engine_strip_connect",
    "ssla_engine_strip_drain", "ssla_strip_drain_lockstep", "ssla_engine_strip_status",
    "ssla_engine_rings_attach", "ssla_engine_drain_rings", "ssla_engine_serve_rings",
    "ssla_replay_start", "ssla_replay_stop", "ssla_replay_join",
)
# SSLA_STRIP_ERR_* bits
STRIP_ERR_CAPACITY, STRIP_ERR_TIMEOUT, STRIP_ERR_MISMATCH = 1, 2, 4
# Every symbol include/stage01_to_gpu.h declares (the libstage01_to_gpu ABI).
S01G_EXPORTED = (
    "s01g_init", "s01g_init_full", "s01g_attach_gpu_rings", "s01g_attach_gpu_rings_multi",
    "s01g_submit_batch", "s01g_snapshot_stats", "s01g_reset_stats", "s01g_start_synthetic",
    "s01g_stop_synthetic", "s01g_synthetic_n_pushed", "s01g_shutdown", "s01g_flush",
)
NOALLOC_MAX_RECORDS = 65536
NOALLOC_MAX_CELLS = 65535
