"""TEST INFRASTRUCTURE ONLY -- ctypes front ends for the two CPU checkers.

``Oracle``     : the plain-C restatement (oracle/ssla_oracle.c,
                 libssla_oracle.so).
``RefPipeline``: the reference's own SslaSPipeline built from its sources
                 (oracle/_ref/libssla_ref.so, see oracle/Makefile).

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
arm may use this module; the product never does.
"""
from __future__ import annotations

import ctypes as C
import os
from typing import Dict, Optional

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "libssla_oracle.so")
REF_SO = os.path.join(HERE, "_ref", "libssla_ref.so")

LAYOUT_DECOMP = 0
LAYOUT_HYBRID = 1
CHANS = (12, 24, 48, 96)
F_VALID, F_R1, F_R2, F_R3, F_R4 = 1, 2, 4, 8, 16

_fp = C.POINTER(C.c_float)


class _RawLayer(C.Structure):
    _fields_ = [("in_dim", C.c_int), ("out_dim", C.c_int),
                ("n_pos_in", C.c_int), ("n_pos_out", C.c_int),
                ("W_in_cat", _fp), ("W_out_cat", _fp), ("q", _fp), ("v", _fp),
                ("g", _fp), ("o", _fp), ("ip", _fp), ("norm_w", _fp),
                ("norm_b", _fp)]


class _RawHead(C.Structure):
    _fields_ = [("c_in", C.c_int), ("c_hid", C.c_int), ("ncls", C.c_int)] + [
        (n, _fp) for n in (
            "cls_conv_w", "cls_conv_b", "cls_bn_w", "cls_bn_b", "cls_bn_mean",
            "cls_bn_var", "reg_conv_w", "reg_conv_b", "reg_bn_w", "reg_bn_b",
            "reg_bn_mean", "reg_bn_var", "cls_pred_w", "cls_pred_b",
            "reg_pred_w", "reg_pred_b", "obj_pred_w", "obj_pred_b")]


class _OrState(C.Structure):
    _fields_ = [("layout", C.c_int), ("cnt_len", C.c_int * 4),
                ("hidden", _fp * 8), ("cnt", C.POINTER(C.c_uint8) * 4),
                ("last_t", C.POINTER(C.c_double)), ("preds_dec", _fp),
                ("preds_raw", _fp), ("version", C.POINTER(C.c_uint32))]


def _ptr(a: Optional[np.ndarray]):
    if a is None:
        return None
    return a.ctypes.data_as(C.c_void_p)


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def load_npz(weights_dir: str) -> Dict[str, np.ndarray]:
    with np.load(os.path.join(weights_dir, "weights.npz")) as z:
        return {k: np.asarray(z[k]) for k in z.files}


class Oracle:
    """C restatement with one state (one stream)."""

    def __init__(self, tensors: Dict[str, np.ndarray], h: int, w: int,
                 tdrop: int = 4, layout: int = LAYOUT_HYBRID, ncls: int = 2):
        lib = C.CDLL(ORACLE_SO)
        lib.or_model_create.restype = C.c_void_p
        lib.or_model_create.argtypes = [C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p]
        lib.or_state_create.restype = C.POINTER(_OrState)
        lib.or_state_create.argtypes = [C.c_void_p, C.c_int]
        lib.or_state_reset.argtypes = [C.c_void_p, C.c_void_p]
        lib.or_state_free.argtypes = [C.c_void_p]
        lib.or_model_free.argtypes = [C.c_void_p]
        lib.or_run_events.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int] + [C.c_void_p] * 5
        lib.or_run_s2_records.argtypes = [C.c_void_p, C.c_void_p] + [C.c_void_p] * 4 + [C.c_int] + [C.c_void_p] * 3
        lib.or_head_raw.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p]
        lib.or_expf.restype = C.c_float
        lib.or_expf.argtypes = [C.c_float]
        lib.or_sigmoidf.restype = C.c_float
        lib.or_sigmoidf.argtypes = [C.c_float]
        self.lib = lib
        self.h, self.w, self.ncls, self.layout = h, w, ncls, layout
        self._keep = []
        raws = (_RawLayer * 8)()
        dims = [(2, 12)] + [(12, 12), (12, 24), (24, 24), (24, 48), (48, 48),
                            (48, 96), (96, 96)]
        for li, (i_d, o_d) in enumerate(dims):
            p = f"layers/{li}"
            arrs = {k: _f32(tensors[f"{p}/{k}"]) for k in
                    ("W_in_cat", "W_out_cat", "q_proj/weight", "v_proj/weight",
                     "g_proj/weight", "o_proj/weight", "norm/weight", "norm/bias")}
            ip = tensors.get(f"{p}/input_proj/weight")
            ip = None if ip is None else _f32(ip)
            self._keep += list(arrs.values()) + [ip]
            r = raws[li]
            r.in_dim, r.out_dim = i_d, o_d
            r.n_pos_in = arrs["W_in_cat"].shape[1] // o_d
            r.n_pos_out = arrs["W_out_cat"].shape[0] // o_d
            r.W_in_cat = arrs["W_in_cat"].ctypes.data_as(_fp)
            r.W_out_cat = arrs["W_out_cat"].ctypes.data_as(_fp)
            r.q = arrs["q_proj/weight"].ctypes.data_as(_fp)
            r.v = arrs["v_proj/weight"].ctypes.data_as(_fp)
            r.g = arrs["g_proj/weight"].ctypes.data_as(_fp)
            r.o = arrs["o_proj/weight"].ctypes.data_as(_fp)
            r.ip = ip.ctypes.data_as(_fp) if ip is not None else _fp()
            r.norm_w = arrs["norm/weight"].ctypes.data_as(_fp)
            r.norm_b = arrs["norm/bias"].ctypes.data_as(_fp)
        hd = _RawHead()
        hd.c_in, hd.c_hid, hd.ncls = 96, 96, ncls

        def setf(name, key, optional=False):
            a = tensors.get(key)
            if a is None:
                if not optional:
                    raise KeyError(key)
                setattr(hd, name, _fp())
                return
            a = _f32(a).reshape(-1)
            self._keep.append(a)
            setattr(hd, name, a.ctypes.data_as(_fp))
        for br, pre in (("cls", "cls_convs"), ("reg", "reg_convs")):
            setf(f"{br}_conv_w", f"head/{pre}/0/0/weight")
            setf(f"{br}_conv_b", f"head/{pre}/0/0/bias", optional=True)
            setf(f"{br}_bn_w", f"head/{pre}/0/1/weight")
            setf(f"{br}_bn_b", f"head/{pre}/0/1/bias")
            setf(f"{br}_bn_mean", f"head/{pre}/0/1/running_mean")
            setf(f"{br}_bn_var", f"head/{pre}/0/1/running_var")
        for br in ("cls", "reg", "obj"):
            setf(f"{br}_pred_w", f"head/{br}_preds/0/weight")
            setf(f"{br}_pred_b", f"head/{br}_preds/0/bias")
        self.model = lib.or_model_create(h, w, tdrop, C.cast(raws, C.c_void_p),
                                         C.cast(C.pointer(hd), C.c_void_p))
        if not self.model:
            raise RuntimeError("or_model_create failed")
        self.state = lib.or_state_create(self.model, layout)
        self.s = self.state.contents

    def __del__(self):
        try:
            self.lib.or_state_free(self.state)
            self.lib.or_model_free(self.model)
        except Exception:
            pass

    def reset(self):
        self.lib.or_state_reset(self.model, self.state)

    def run_events(self, ev: np.ndarray, want_stage_out: bool = True):
        ev = _f32(ev).reshape(-1, 4)
        n = ev.shape[0]
        flags = np.zeros(n, np.uint8)
        so = [np.zeros((n, c), np.float32) if want_stage_out else None for c in CHANS]
        self.lib.or_run_events(self.model, self.state, _ptr(ev), n, _ptr(flags),
                               *[_ptr(a) for a in so])
        return flags, so

    def run_s2_records(self, x2, y2, feat1, owner):
        x2 = np.ascontiguousarray(x2, np.int32)
        y2 = np.ascontiguousarray(y2, np.int32)
        owner = np.ascontiguousarray(owner, np.int32)
        feat1 = _f32(feat1).reshape(-1, 24)
        n = x2.size
        p2 = np.zeros(n, np.int32)
        p3 = np.zeros(n, np.int32)
        s3 = np.zeros((n, 96), np.float32)
        self.lib.or_run_s2_records(self.model, self.state, _ptr(x2), _ptr(y2),
                                   _ptr(feat1), _ptr(owner), n, _ptr(p2),
                                   _ptr(p3), _ptr(s3))
        return p2, p3, s3

    # state views (copies)
    def hidden(self, layer: int) -> np.ndarray:
        st = layer // 2
        n = (self.h >> st) * (self.w >> st) * CHANS[st]
        return np.ctypeslib.as_array(self.s.hidden[layer], shape=(n,)).copy()

    def set_hidden(self, layer: int, values: np.ndarray) -> None:
        st = layer // 2
        n = (self.h >> st) * (self.w >> st) * CHANS[st]
        dst = np.ctypeslib.as_array(self.s.hidden[layer], shape=(n,))
        dst[:] = _f32(values).reshape(-1)

    def counters(self, g: int) -> np.ndarray:
        return np.ctypeslib.as_array(self.s.cnt[g], shape=(self.s.cnt_len[g],)).copy()

    def last_t(self) -> np.ndarray:
        return np.ctypeslib.as_array(self.s.last_t, shape=(self.h * self.w,)).copy()

    def preds_dec(self) -> np.ndarray:
        n3 = (self.h >> 3) * (self.w >> 3)
        return np.ctypeslib.as_array(self.s.preds_dec, shape=(n3 * (5 + self.ncls),)).reshape(n3, -1).copy()

    def preds_raw(self) -> np.ndarray:
        n3 = (self.h >> 3) * (self.w >> 3)
        return np.ctypeslib.as_array(self.s.preds_raw, shape=(n3 * (5 + self.ncls),)).reshape(n3, -1).copy()

    def version(self) -> np.ndarray:
        n3 = (self.h >> 3) * (self.w >> 3)
        return np.ctypeslib.as_array(self.s.version, shape=(n3,)).copy()

    def expf(self, x: float) -> float:
        return self.lib.or_expf(x)

    def head_raw(self, feat: np.ndarray) -> np.ndarray:
        """Raw head outputs [reg 4, obj, cls...] of one 96-float stage-3 feature."""
        f = _f32(feat).reshape(96)
        out = np.zeros(5 + self.ncls, np.float32)
        self.lib.or_head_raw(self.model, _ptr(f), _ptr(out))
        return out


class RefPipeline:
    """The reference's own SslaSPipeline (oracle/_ref) for one stream."""

    def __init__(self, weights_dir: str, layout: int = LAYOUT_HYBRID):
        if not os.path.exists(REF_SO):
            raise FileNotFoundError(REF_SO)
        lib = C.CDLL(REF_SO)
        lib.ref_create.restype = C.c_void_p
        lib.ref_create.argtypes = [C.c_char_p]
        lib.ref_destroy.argtypes = [C.c_void_p]
        lib.ref_reset.argtypes = [C.c_void_p]
        lib.ref_num_anchors.argtypes = [C.c_void_p]
        lib.ref_cols.argtypes = [C.c_void_p]
        lib.ref_run_events.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_int] + [C.c_void_p] * 5
        lib.ref_run_s2_records.argtypes = [C.c_void_p] + [C.c_void_p] * 4 + [C.c_int] + [C.c_void_p] * 3
        lib.ref_get_hidden.argtypes = [C.c_void_p, C.c_int, C.c_void_p]
        lib.ref_get_predictions.argtypes = [C.c_void_p, C.c_void_p]
        lib.ref_time_streams.restype = C.c_double
        lib.ref_time_streams.argtypes = [C.c_char_p, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_int]
        self.lib = lib
        self.weights_dir = weights_dir
        self.layout = layout
        self.h = lib.ref_create(weights_dir.encode())
        if not self.h:
            raise RuntimeError(f"reference SslaSPipeline failed to load {weights_dir}")
        import json
        with open(os.path.join(weights_dir, "meta.json")) as f:
            meta = json.load(f)
        self.H, self.W = int(meta["height"]), int(meta["width"])

    def __del__(self):
        try:
            self.lib.ref_destroy(self.h)
        except Exception:
            pass

    def reset(self):
        self.lib.ref_reset(self.h)

    def run_events(self, ev: np.ndarray, want_stage_out: bool = True):
        ev = _f32(ev).reshape(-1, 4)
        n = ev.shape[0]
        flags = np.zeros(n, np.uint8)
        so = [np.zeros((n, c), np.float32) if want_stage_out else None for c in CHANS]
        self.lib.ref_run_events(self.h, self.layout, _ptr(ev), n, _ptr(flags),
                                *[_ptr(a) for a in so])
        return flags, so

    def run_s2_records(self, x2, y2, feat1, owner):
        x2 = np.ascontiguousarray(x2, np.int32)
        y2 = np.ascontiguousarray(y2, np.int32)
        owner = np.ascontiguousarray(owner, np.int32)
        feat1 = _f32(feat1).reshape(-1, 24)
        n = x2.size
        p2 = np.zeros(n, np.int32)
        p3 = np.zeros(n, np.int32)
        s3 = np.zeros((n, 96), np.float32)
        self.lib.ref_run_s2_records(self.h, _ptr(x2), _ptr(y2), _ptr(feat1),
                                    _ptr(owner), n, _ptr(p2), _ptr(p3), _ptr(s3))
        return p2, p3, s3

    def hidden(self, layer: int) -> np.ndarray:
        st = layer // 2
        n = (self.H >> st) * (self.W >> st) * CHANS[st]
        out = np.zeros(n, np.float32)
        self.lib.ref_get_hidden(self.h, layer, _ptr(out))
        return out

    def predictions(self) -> np.ndarray:
        na, co = self.lib.ref_num_anchors(self.h), self.lib.ref_cols(self.h)
        out = np.zeros(na * co, np.float32)
        self.lib.ref_get_predictions(self.h, _ptr(out))
        return out.reshape(na, co)

    def time_streams(self, streams, n_threads: int) -> float:
        """Wall seconds for independent reference pipelines over `streams`."""
        arrs = [_f32(s).reshape(-1, 4) for s in streams]
        ptrs = (C.c_void_p * len(arrs))(*[a.ctypes.data for a in arrs])
        ns = (C.c_int * len(arrs))(*[a.shape[0] for a in arrs])
        return self.lib.ref_time_streams(self.weights_dir.encode(), self.layout,
                                         len(arrs), ptrs, ns, n_threads)
