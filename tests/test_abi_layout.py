"""The drop-in byte layouts (include/ssla_abi_types.h) match the reference's
structs: HybridInputRec 128 B (src/lib_stage01_to_gpu.cpp:51-60),
HybridS2S3OutputSlot (ssla_s2_s3_head_celled.cuh:139-143), GpuTimingSlot 40 B
(:66-76) and the HybridS2S3Config field offsets of
orin/orin/hybrid_common.py:76-111."""
import ctypes as C

from ssla_rt_b200 import abi


def test_record_layouts():
    assert abi.INPUT_DTYPE.itemsize == 128
    assert abi.INPUT_DTYPE.fields["t"][1] == 8
    assert abi.INPUT_DTYPE.fields["x"][1] == 12
    assert abi.INPUT_DTYPE.fields["y"][1] == 14
    assert abi.INPUT_DTYPE.fields["feat1"][1] == 16
    assert abi.INPUT_DTYPE.fields["t_push_ns"][1] == 112
    assert abi.INPUT_DTYPE.fields["t_emit_ns"][1] == 120
    assert abi.OUTPUT_DTYPE.itemsize == 392
    assert abi.TIMING_DTYPE.itemsize == 40
    assert abi.EVENT_DTYPE.itemsize == 16


def test_config_layout():
    cfg = abi.HybridS2S3Config
    assert C.sizeof(abi.HybridStrip) == 32
    assert C.sizeof(abi.LayerWeightsS2S3) == 40
    assert cfg.strip.offset == 32
    assert cfg.layers.offset == 32 + 16 * 32
    assert cfg.hidden.offset == cfg.layers.offset + 16 * 4 * 40
    assert cfg.tdrop_s2.offset == cfg.hidden.offset + 16 * 4 * 8
    assert cfg.head_W.offset == cfg.tdrop_s3.offset + 16 * 8
    assert cfg.preds.offset == cfg.head_obj_pred_b.offset + 8
    assert cfg.timing_mask.offset == cfg.timing.offset + 16 * 8
    assert cfg.kernel_end_clk.offset + 16 * 8 == C.sizeof(cfg)


def test_header_asserts_match():
    """The C header pins the same numbers with static_assert."""
    import os
    import re
    here = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    txt = open(os.path.join(here, "include", "ssla_abi_types.h")).read()
    assert "sizeof(HybridInputRec) == 128" in txt
    assert "sizeof(HybridS2S3OutputSlot) == 392" in txt
    assert "sizeof(GpuTimingSlot) == 40" in txt
    assert re.search(r"offsetof\(HybridS2S3Config, layers\) == 32 \+ 16 \* 32", txt)
