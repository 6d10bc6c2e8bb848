/* ssla_oracle.h -- TEST INFRASTRUCTURE ONLY.
 *
 * Plain-C CPU restatement of the reference's SSLA-S per-event path, used as
 * the parity checker for the CUDA engine.  Nothing in the product links,
 * imports or calls this code; only tests/, __graft_entry__.smoke() and the
 * cpu_baseline leg of bench.py do.
 *
 * Parity pins (tests/test_oracle_pins.py):
 *   - the reference's own C++ SslaSPipeline compiled from its sources into
 *     oracle/_ref (oracle/Makefile), on the same seeded inputs;
 *   - golden vectors in tests/golden/ produced from that build and from the
 *     reference's numpy oracle (orin/orin/ssla_ref.py), with the generating
 *     script committed beside them.
 *
 * Arithmetic contract (shared with the CUDA engine so the two can be compared
 * bit for bit): every dot product is an fmaf() chain in the reference's loop
 * order, starting from 0 (or from the bias where the reference does), no
 * other contraction (-ffp-contract=off), LayerNorm reductions sequential in
 * fp64, and exp() is the portable Cody-Waite + degree-7 Taylor restatement in
 * or_expf(), which the engine implements identically.
 */
#ifndef SSLA_ORACLE_H
#define SSLA_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Gate layouts (which counter grid each temporal-dropout gate uses).
 * OR_LAYOUT_DECOMP: src/legacy/schemes/s2_decomp_st.cpp:138-176 -- three
 *   tdrop_and_pool gates after s0/s1/s2 (counters on the s1/s2/s3 grids), the
 *   head runs for every event that finishes s3.
 * OR_LAYOUT_HYBRID: the production chain src/lib_stage01_to_gpu.cpp:228-311
 *   (CPU gates on the s1/s2 grids) followed by
 *   orin/kernels/ssla_s2_s3_head_celled.cuh:1679-1755 (GPU tdrop_s2 on the s2
 *   grid gating stage 3, tdrop_s3 on the s3 grid gating the head). */
enum { OR_LAYOUT_DECOMP = 0, OR_LAYOUT_HYBRID = 1 };

typedef struct {
    int in_dim, out_dim, A;      /* A = number of patch positions (1 or 9)       */
    float* qvg;                  /* [A][3*OUT][IN]  src/ssla_kernels.cpp:126-129 */
    float* goW;                  /* [A][OUT][OUT]   src/ssla_kernels.cpp:130     */
    float* ip;                   /* [OUT][IN] or NULL (input_proj)               */
    float* gamma;                /* [OUT] */
    float* beta;                 /* [OUT] */
} OrLayer;

typedef struct {
    int H, W, ncls, tdrop_window;
    OrLayer L[8];
    /* YOLOX head, BN folded (vendor/openeva/heads/async_yolox.h:98-143),
     * (out, in) row-major like the reference's YoloxLevel.                  */
    int c_in, c_hid, stride_h, stride_w;
    float *cls_conv_W, *cls_conv_b, *reg_conv_W, *reg_conv_b;
    float *cls_pred_W, *cls_pred_b, *reg_pred_W, *reg_pred_b;
    float *obj_pred_W, *obj_pred_b;
} OrModel;

typedef struct {
    int layout;
    int cnt_len[4];
    float*    hidden[8];         /* [Hs*Ws][OUT] per layer                      */
    uint8_t*  cnt[4];            /* gate counters (grid per layout)             */
    double*   last_t;            /* [H*W], -1.0 = never seen                    */
    float*    preds_dec;         /* [H3*W3][5+ncls] decoded (CPU contract)      */
    float*    preds_raw;         /* [H3*W3][5+ncls] raw reg4,obj,cls (GPU)      */
    uint32_t* version;           /* [H3*W3] head writes per cell                */
} OrState;

/* Raw tensors of one SSLA layer as stored in weights.npz
 * (tools/make_ssla_stub.py:29-49). ip may be NULL. */
typedef struct {
    int in_dim, out_dim;
    int n_pos_in, n_pos_out;     /* W_in_cat cols / OUT, W_out_cat rows / OUT */
    const float *W_in_cat, *W_out_cat, *q, *v, *g, *o, *ip, *norm_w, *norm_b;
} OrRawLayer;

/* Raw YOLOX head level 0 tensors (tools/make_ssla_stub.py:52-81). */
typedef struct {
    int c_in, c_hid, ncls;
    const float *cls_conv_w, *cls_conv_b;        /* conv bias may be NULL */
    const float *cls_bn_w, *cls_bn_b, *cls_bn_mean, *cls_bn_var;
    const float *reg_conv_w, *reg_conv_b;
    const float *reg_bn_w, *reg_bn_b, *reg_bn_mean, *reg_bn_var;
    const float *cls_pred_w, *cls_pred_b, *reg_pred_w, *reg_pred_b;
    const float *obj_pred_w, *obj_pred_b;
} OrRawHead;

/* Per-event flag bits written by or_run_events: VALID = in bounds,
 * R1..R4 = reached stage 1 / 2 / 3 / the head. */
enum { OR_F_VALID = 1, OR_F_R1 = 2, OR_F_R2 = 4, OR_F_R3 = 8, OR_F_R4 = 16 };

OrModel* or_model_create(int H, int W, int tdrop_window,
                         const OrRawLayer* raw8, const OrRawHead* head);
void     or_model_free(OrModel* m);
OrState* or_state_create(const OrModel* m, int layout);
void     or_state_free(OrState* s);
void     or_state_reset(const OrModel* m, OrState* s);

/* Runs n raw events (t,x,y,p per event, reference Event layout) in order.
 * flags[n] gets OR_F_* bits; stage_out_s (each may be NULL) [n*C_s] gets the
 * stage-s output of events whose stage-s output was produced (s3 = the L7
 * output of head events). */
void or_run_events(const OrModel* m, OrState* s, const float* ev, int n,
                   uint8_t* flags, float* stage_out0, float* stage_out1,
                   float* stage_out2, float* stage_out3);

/* drain_n contract (orin/kernels/ssla_s2_s3_head_celled.cuh:986-1094) for one
 * block: s2-level records in order.  x2,y2: s2 coords, feat1: n*24.  owner[n]
 * is the strip ownership of each record.  Writes pass2/pass3 codes and the
 * 96-float s3_feat slot as the reference kernel leaves it.  Uses cnt[2]
 * (tdrop_s2, s2 grid) and cnt[3] (tdrop_s3, s3 grid) of a HYBRID state. */
void or_run_s2_records(const OrModel* m, OrState* s, const int* x2,
                       const int* y2, const float* feat1, const int* owner,
                       int n, int* pass2, int* pass3, float* s3_feat);

/* Raw head outputs [reg 4, obj, cls ncls] of one 96-float stage-3 feature. */
void or_head_raw(const OrModel* m, const float* feat, float* raw);

/* Math restatements exposed for tests. */
float or_expf(float x);
float or_sigmoidf(float x);
/* One generic layer forward at stage resolution (layer_forward_ct,
 * src/ssla_kernels.cpp:315-385); want_out = 0 runs the state-only update. */
void or_layer_forward(const OrModel* m, OrState* s, int l, int ex, int ey,
                      const float* in, float* out, int want_out);

#ifdef __cplusplus
}
#endif
#endif
