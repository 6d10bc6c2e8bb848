/* ssla_abi_types.h -- data layouts shared with haohq19/ssla-rt callers.
 *
 * These structs are byte-for-byte the reference's ring record, drain_n
 * output slot, timing slot and s2/s3 kernel configuration, so existing
 * callers (the C++ host library and the orin/ cuda-python runners, whose
 * ctypes mirrors are orin/orin/hybrid_common.py:30-122) can hand their
 * buffers to this library unchanged.  Sizes and offsets are pinned by
 * static asserts here and by tests/test_abi_layout.py.
 */
#ifndef SSLA_ABI_TYPES_H
#define SSLA_ABI_TYPES_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SSLA_MAX_BLOCKS 16   /* MAX_BLOCKS, ssla_s2_s3_head_celled.cuh:82 */

/* GPU ring record, 128 B (src/lib_stage01_to_gpu.cpp:51-60,
 * ssla_s2_s3_head_celled.cuh:129-137).  seq_done = slot + 1 once published. */
typedef struct {
    uint64_t seq_done;
    float    t;
    uint16_t x;              /* s2-grid x */
    uint16_t y;              /* s2-grid y */
    float    feat1[24];      /* stage-1 output (C1 = 24) */
    uint64_t t_push_ns;
    uint64_t t_emit_ns;
} HybridInputRec;

/* drain_n per-record output (ssla_s2_s3_head_celled.cuh:139-143).
 * pass2 / pass3: 1 owner-passed, 0 owner-dropped, -1 halo. */
typedef struct {
    int   pass2;
    int   pass3;
    float s3_feat[96];
} HybridS2S3OutputSlot;

/* Per-event timing slot, 40 B (ssla_s2_s3_head_celled.cuh:66-76). */
typedef struct {
    uint64_t t_pop_clk;
    uint64_t t_done_clk;
    uint32_t seq;
    uint32_t owner;
    uint64_t t_push_ns;
    uint64_t t_emit_ns;
} GpuTimingSlot;

/* Strip ownership in s2 / s3 coordinates (ssla_s2_s3_head_celled.cuh:53-64). */
typedef struct {
    int owned_lo, owned_hi;
    int s3_owned_lo, s3_owned_hi;
    int owned_y_lo, owned_y_hi;
    int s3_owned_y_lo, s3_owned_y_hi;
} HybridStrip;

/* Device pointers of one s2/s3 layer in the reference's GPU layouts
 * (orin/orin/hybrid_common.py:192-199): qvgIn (A, IN, 3*OUT), goW
 * (A, OUT_in, OUT_out), input_proj (IN, OUT) or NULL. */
typedef struct {
    const float* qvgIn;
    const float* goW;
    const float* input_proj;
    const float* ln_gamma;
    const float* ln_beta;
} LayerWeightsS2S3;

/* ssla_s2_s3_head_celled.cuh:84-127 */
typedef struct {
    int H2, W2;
    int H3, W3;
    int tdrop_window;
    int head_out_dim;
    int n_blocks;
    int _pad_nblocks;
    HybridStrip      strip[SSLA_MAX_BLOCKS];
    LayerWeightsS2S3 layers[SSLA_MAX_BLOCKS][4];
    float*           hidden[SSLA_MAX_BLOCKS][4];
    unsigned char*   tdrop_s2[SSLA_MAX_BLOCKS];
    unsigned char*   tdrop_s3[SSLA_MAX_BLOCKS];
    const float*     head_W;
    const float*     head_b;
    const float*     head_cls_conv_W;
    const float*     head_cls_conv_b;
    const float*     head_cls_pred_W;
    const float*     head_cls_pred_b;
    const float*     head_reg_conv_W;
    const float*     head_reg_conv_b;
    const float*     head_reg_pred_W;
    const float*     head_reg_pred_b;
    const float*     head_obj_pred_W;
    const float*     head_obj_pred_b;
    float*           preds[SSLA_MAX_BLOCKS];
    unsigned int*    version[SSLA_MAX_BLOCKS];
    GpuTimingSlot*   timing[SSLA_MAX_BLOCKS];
    unsigned int     timing_mask;
    unsigned int     _pad_timing;
    unsigned long long* kernel_start_clk[SSLA_MAX_BLOCKS];
    unsigned long long* kernel_end_clk[SSLA_MAX_BLOCKS];
} HybridS2S3Config;

#ifdef __cplusplus
}
static_assert(sizeof(HybridInputRec) == 128, "HybridInputRec layout");
static_assert(offsetof(HybridInputRec, t) == 8, "HybridInputRec.t");
static_assert(offsetof(HybridInputRec, x) == 12, "HybridInputRec.x");
static_assert(offsetof(HybridInputRec, feat1) == 16, "HybridInputRec.feat1");
static_assert(offsetof(HybridInputRec, t_push_ns) == 112, "HybridInputRec.t_push_ns");
static_assert(sizeof(HybridS2S3OutputSlot) == 392, "HybridS2S3OutputSlot layout");
static_assert(sizeof(GpuTimingSlot) == 40, "GpuTimingSlot layout");
static_assert(sizeof(HybridStrip) == 32, "HybridStrip layout");
static_assert(sizeof(LayerWeightsS2S3) == 40, "LayerWeightsS2S3 layout");
static_assert(offsetof(HybridS2S3Config, strip) == 32, "cfg.strip");
static_assert(offsetof(HybridS2S3Config, layers) == 32 + 16 * 32, "cfg.layers");
static_assert(offsetof(HybridS2S3Config, hidden) == 3104, "cfg.hidden");
static_assert(offsetof(HybridS2S3Config, head_W) == 3872, "cfg.head_W");
static_assert(offsetof(HybridS2S3Config, preds) == 3968, "cfg.preds");
static_assert(offsetof(HybridS2S3Config, timing_mask) == 4352, "cfg.timing_mask");
static_assert(sizeof(HybridS2S3Config) == 4616, "HybridS2S3Config layout");
#endif
#endif
