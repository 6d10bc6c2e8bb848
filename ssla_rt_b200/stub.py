"""Seeded SSLA-S stub weights (random, schema-valid) -- the BASELINE model.

Writes ``weights.npz`` + ``meta.json`` with the key schema, shapes, value
distributions and draw order of the reference's stub generator
(tools/make_ssla_stub.py:29-153), so ``write_stub(dir, h=64, w=80, seed=1)``
yields the same tensors as ``make_ssla_stub.py dir --h 64 --w 80 --seed 1``
(tests/test_stub_weights.py checks this against a committed digest).

Schema (per layer ``layers/<i>/``):
  W_in_cat (IN, A*OUT), W_out_cat (A*OUT, OUT), {q,v,g,o}_proj/weight (OUT, OUT),
  input_proj/weight (OUT, IN) iff IN != OUT, norm/{weight,bias} (OUT,)
Head level 0 (``head/``): {cls,reg}_convs/0/{0/weight, 1/{weight,bias,
  running_mean,running_var}}, {cls,reg,obj}_preds/0/{weight,bias}.
"""
from __future__ import annotations

import json
import os
from typing import Dict

import numpy as np

IN_DIM = 2
CHANS = (12, 24, 48, 96)
# (in, out, kernel) per layer: L0 is K=1, every other layer K=3.
LAYER_SPECS = ((2, 12, 1), (12, 12, 3), (12, 24, 3), (24, 24, 3),
               (24, 48, 3), (48, 48, 3), (48, 96, 3), (96, 96, 3))


def stub_tensors(seed: int = 1, num_classes: int = 2,
                 num_head_levels: int = 1) -> Dict[str, np.ndarray]:
    """All stub tensors, drawn from ``np.random.default_rng(seed)`` in the
    reference generator's order."""
    rng = np.random.default_rng(seed)
    f32 = np.float32
    out: Dict[str, np.ndarray] = {}
    for li, (i_d, o_d, k) in enumerate(LAYER_SPECS):
        a = k * k
        p = f"layers/{li}"
        out[f"{p}/W_in_cat"] = rng.normal(scale=0.3, size=(i_d, a * o_d)).astype(f32)
        out[f"{p}/W_out_cat"] = rng.normal(scale=0.3, size=(a * o_d, o_d)).astype(f32)
        for proj in ("q_proj", "v_proj", "g_proj", "o_proj"):
            out[f"{p}/{proj}/weight"] = rng.normal(scale=0.3, size=(o_d, o_d)).astype(f32)
        if i_d != o_d:
            out[f"{p}/input_proj/weight"] = rng.normal(scale=0.3, size=(o_d, i_d)).astype(f32)
        out[f"{p}/norm/weight"] = (rng.normal(scale=0.1, size=(o_d,)) + 1.0).astype(f32)
        out[f"{p}/norm/bias"] = rng.normal(scale=0.1, size=(o_d,)).astype(f32)
    c_hid = CHANS[-1]
    for lvl in range(num_head_levels):
        c_in = CHANS[len(CHANS) - num_head_levels + lvl]
        k = str(lvl)
        for branch in ("cls_convs", "reg_convs"):
            out[f"head/{branch}/{k}/0/weight"] = rng.normal(scale=0.1, size=(c_hid, c_in)).astype(f32)
            out[f"head/{branch}/{k}/1/weight"] = (rng.normal(scale=0.05, size=(c_hid,)) + 1.0).astype(f32)
            out[f"head/{branch}/{k}/1/bias"] = rng.normal(scale=0.05, size=(c_hid,)).astype(f32)
            out[f"head/{branch}/{k}/1/running_mean"] = np.zeros((c_hid,), dtype=f32)
            out[f"head/{branch}/{k}/1/running_var"] = np.ones((c_hid,), dtype=f32)
        out[f"head/cls_preds/{k}/weight"] = rng.normal(scale=0.05, size=(num_classes, c_hid)).astype(f32)
        out[f"head/cls_preds/{k}/bias"] = rng.normal(scale=0.05, size=(num_classes,)).astype(f32)
        out[f"head/reg_preds/{k}/weight"] = rng.normal(scale=0.05, size=(4, c_hid)).astype(f32)
        out[f"head/reg_preds/{k}/bias"] = rng.normal(scale=0.05, size=(4,)).astype(f32)
        out[f"head/obj_preds/{k}/weight"] = rng.normal(scale=0.05, size=(1, c_hid)).astype(f32)
        out[f"head/obj_preds/{k}/bias"] = rng.normal(scale=0.05, size=(1,)).astype(f32)
    return out


def write_stub(out_dir: str, h: int = 64, w: int = 80, seed: int = 1,
               num_classes: int = 2, tdrop: int = 4) -> str:
    """Write weights.npz (uncompressed, as the C++ loaders require) and
    meta.json into ``out_dir``; returns ``out_dir``."""
    os.makedirs(out_dir, exist_ok=True)
    t = stub_tensors(seed=seed, num_classes=num_classes)
    np.savez(os.path.join(out_dir, "weights.npz"), **t)
    meta = {
        "schema_version": 1,
        "model": "ssla_s_yolox_det",
        "method": "ssla",
        "height": int(h),
        "width": int(w),
        "num_classes": int(num_classes),
        "num_anchors": 1,
        "ssla_tdrop_window": int(tdrop),
        "dtype": "float32",
        "layout": "C_order_row_major",
        "key_separator": "/",
        "checkpoint": "stub_random",
        "total_params": int(sum(int(np.prod(v.shape)) for v in t.values())),
    }
    with open(os.path.join(out_dir, "meta.json"), "w") as f:
        json.dump(meta, f, indent=2)
    return out_dir


def tensors_digest(t: Dict[str, np.ndarray]) -> str:
    """Order-independent sha256 over (key, shape, bytes) of every tensor."""
    import hashlib
    hsh = hashlib.sha256()
    for k in sorted(t):
        a = np.ascontiguousarray(t[k], dtype=np.float32)
        hsh.update(k.encode())
        hsh.update(str(a.shape).encode())
        hsh.update(a.tobytes())
    return hsh.hexdigest()
