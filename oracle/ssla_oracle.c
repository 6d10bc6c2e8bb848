/* ssla_oracle.c -- TEST INFRASTRUCTURE ONLY (see ssla_oracle.h).
 *
 * CPU restatement of the reference SSLA-S per-event path.  Each function
 * cites the reference file:line it restates (paths relative to the
 * haohq19/ssla-rt checkout).  Build flags: -O2 -ffp-contract=off (no
 * fast-math), so every rounding step is the one written here.
 */
#include "ssla_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

static const int kChans[4] = {12, 24, 48, 96};

/* ---------------------------------------------------------------------------
 * exp / sigmoid
 *
 * or_expf: Cody-Waite argument reduction x = n*ln2 + r (ln2 split into a
 * 12-bit head and a float tail, so n*ln2_hi is exact for |n| < 2^12) followed
 * by the degree-7 Taylor polynomial of exp(r) on |r| <= ln2/2 (truncation
 * error r^8/8! < 6e-9 relative) evaluated by Horner with fmaf, then an exact
 * power-of-two scaling.  Every step is an IEEE-754 basic operation, so the
 * CUDA engine's copy of this function returns identical bits.  The reference
 * uses std::exp (vendor/openeva/prim/activation.h:17); tests bound the
 * difference to <= 2 ulp.
 * ------------------------------------------------------------------------- */
static float pow2i(int e) {          /* 2^e for -126 <= e <= 127, exact */
    union { uint32_t u; float f; } b;
    b.u = (uint32_t)(e + 127) << 23;
    return b.f;
}

float or_expf(float x) {
    if (x != x) return x;                              /* NaN */
    if (x > 88.8f) return INFINITY;
    if (x < -104.0f) return 0.0f;
    /* n = nearest integer to x*log2(e), ties to even: adding 1.5*2^23 leaves
     * an integer-spaced float (|x*log2e| < 2^22 here), so the sum rounds
     * exactly as rintf would and the subtraction is exact; the integer is
     * read from the sum's low mantissa bits. */
    union { float f; int32_t i; } big;
    big.f = x * 1.44269502f + 12582912.0f;
    const float n = big.f - 12582912.0f;
    float r = fmaf(-n, 0.693115234375f, x);
    r = fmaf(-n, 3.19461833e-05f, r);
    float p = 1.98412701e-04f;                         /* 1/7! */
    p = fmaf(p, r, 1.38888892e-03f);                   /* 1/6! */
    p = fmaf(p, r, 8.33333377e-03f);                   /* 1/5! */
    p = fmaf(p, r, 4.16666679e-02f);                   /* 1/4! */
    p = fmaf(p, r, 1.66666672e-01f);                   /* 1/3! */
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    const int ni = big.i - 0x4B400000;                 /* -150 .. 129 */
    const int n1 = ni / 2;
    const int n2 = ni - n1;
    return (p * pow2i(n1)) * pow2i(n2);
}

/* activation.h:17  sigmoid(x) = 1 / (1 + exp(-x)) */
/* Sigmoid, vendor/openeva/prim/activation.h:17: 1 / (1 + exp(-x)) with an
 * exp of its own for the range the sigmoid needs.  t = -x is clamped to
 * [-17, 87] (for x >= 17 the result is exactly 1, as 1 + exp(-17) rounds to
 * 1; for x <= -87 it is 1 / (1 + e^87) ~ 1.6e-38, the smallest normal
 * result); n and r as in or_expf
 * (with the product-sum for n fused); exp(r) by a degree-6 minimax
 * polynomial on [-ln2/2, ln2/2] (Remez exchange, coefficients rounded to
 * float, 0.87 ulp on the interval) by Horner with fmaf; one exact scaling by
 * 2^n, n in [-25, 126]; IEEE division.  Within 2.3 ulp of the exact
 * sigmoid for x >= -87, as 1 / (1 + or_expf(-x)) is. */
float or_sigmoidf(float x) {
    if (x != x) return x;
    const float t = fminf(fmaxf(-x, -17.0f), 87.0f);
    union { float f; int32_t i; } big;
    big.f = fmaf(t, 1.44269502f, 12582912.0f);
    const float n = big.f - 12582912.0f;
    float r = fmaf(-n, 0.693115234375f, t);
    r = fmaf(-n, 3.19461833e-05f, r);
    float p = 1.38368458e-03f;
    p = fmaf(p, r, 8.37481581e-03f);
    p = fmaf(p, r, 4.16682251e-02f);
    p = fmaf(p, r, 1.66664198e-01f);
    p = fmaf(p, r, 4.99999911e-01f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    return 1.0f / (1.0f + p * pow2i(big.i - 0x4B400000));
}

/* ---------------------------------------------------------------------------
 * Primitive restatements
 * ------------------------------------------------------------------------- */

/* vendor/openeva/prim/linear.h:80-90 matvec_ct: y[o] = bias[o] (or 0) +
 * sum_i W[o][i] x[i], W (OUT, IN) row-major. */
static void matvec(const float* x, int in, const float* W, int out,
                   const float* bias, float* y) {
    for (int o = 0; o < out; ++o) {
        const float* w = W + (size_t)o * in;
        float acc = bias ? bias[o] : 0.0f;
        for (int i = 0; i < in; ++i) acc = fmaf(w[i], x[i], acc);
        y[o] = acc;
    }
}

/* linear.h:92-101 matvec_accum_ct: y[o] += sum_i W[o][i] x[i]. */
static void matvec_accum(const float* x, int in, const float* W, int out,
                         float* y) {
    for (int o = 0; o < out; ++o) {
        const float* w = W + (size_t)o * in;
        float acc = 0.0f;
        for (int i = 0; i < in; ++i) acc = fmaf(w[i], x[i], acc);
        y[o] = y[o] + acc;
    }
}

/* vendor/openeva/prim/layernorm.h:41-62 layernorm_ct: fp64 mean/var,
 * eps = 1e-5f, in place. */
static void layernorm(float* x, int dim, const float* gamma,
                      const float* beta) {
    double sum = 0.0;
    for (int i = 0; i < dim; ++i) sum += (double)x[i];
    const double mean = sum / (double)dim;
    double var = 0.0;
    for (int i = 0; i < dim; ++i) {
        const double d = (double)x[i] - mean;
        var += d * d;
    }
    var /= (double)dim;
    const double inv = 1.0 / sqrt(var + (double)1e-5f);
    for (int i = 0; i < dim; ++i) {
        const double v = ((double)x[i] - mean) * inv;
        x[i] = (float)(v * (double)gamma[i] + (double)beta[i]);
    }
}

/* ---------------------------------------------------------------------------
 * Model construction
 * ------------------------------------------------------------------------- */

/* vendor/openeva/prim/matmul.h:24-41 mm: C = B @ A, k-loop in order. */
static void mm(const float* B, int b_out, int b_in, const float* A, int a_in,
               float* C) {
    for (int o = 0; o < b_out; ++o) {
        float* cr = C + (size_t)o * a_in;
        for (int i = 0; i < a_in; ++i) cr[i] = 0.0f;
        for (int k = 0; k < b_in; ++k) {
            const float bv = B[(size_t)o * b_in + k];
            const float* ar = A + (size_t)k * a_in;
            for (int i = 0; i < a_in; ++i) cr[i] = fmaf(bv, ar[i], cr[i]);
        }
    }
}

/* src/ssla_kernels.cpp:73-153 load_layer: per-position fused tensors
 * qvgIn[p] = vstack(Q,V,G) @ scatter[p], goW[p] = gather[p] @ O. */
static int build_layer(OrLayer* L, const OrRawLayer* r) {
    const int IN = r->in_dim, OUT = r->out_dim;
    const int A = r->n_pos_in > r->n_pos_out ? r->n_pos_in : r->n_pos_out;
    const int win_cols = r->n_pos_in * OUT;
    L->in_dim = IN; L->out_dim = OUT; L->A = A;
    L->qvg = (float*)calloc((size_t)A * 3 * OUT * IN, sizeof(float));
    L->goW = (float*)calloc((size_t)A * OUT * OUT, sizeof(float));
    L->gamma = (float*)malloc(sizeof(float) * OUT);
    L->beta  = (float*)malloc(sizeof(float) * OUT);
    L->ip = NULL;
    float* scatter = (float*)malloc(sizeof(float) * OUT * IN);
    float* gather  = (float*)malloc(sizeof(float) * OUT * OUT);
    if (!L->qvg || !L->goW || !L->gamma || !L->beta || !scatter || !gather)
        return -1;
    for (int p = 0; p < A; ++p) {
        const int pin  = (r->n_pos_in  == 1) ? 0 : p;
        const int pout = (r->n_pos_out == 1) ? 0 : p;
        for (int d = 0; d < OUT; ++d)
            for (int c = 0; c < IN; ++c)
                scatter[(size_t)d * IN + c] =
                    r->W_in_cat[(size_t)c * win_cols + pin * OUT + d];
        for (int i = 0; i < OUT; ++i)
            for (int j = 0; j < OUT; ++j)
                gather[(size_t)i * OUT + j] =
                    r->W_out_cat[(size_t)(pout * OUT + j) * OUT + i];
        float* qvg = L->qvg + (size_t)p * 3 * OUT * IN;
        mm(r->q, OUT, OUT, scatter, IN, qvg);
        mm(r->v, OUT, OUT, scatter, IN, qvg + (size_t)OUT * IN);
        mm(r->g, OUT, OUT, scatter, IN, qvg + (size_t)2 * OUT * IN);
        mm(gather, OUT, OUT, r->o, OUT, L->goW + (size_t)p * OUT * OUT);
    }
    free(scatter);
    free(gather);
    if (r->ip) {
        L->ip = (float*)malloc(sizeof(float) * OUT * IN);
        if (!L->ip) return -1;
        memcpy(L->ip, r->ip, sizeof(float) * OUT * IN);
    }
    memcpy(L->gamma, r->norm_w, sizeof(float) * OUT);
    memcpy(L->beta,  r->norm_b, sizeof(float) * OUT);
    return 0;
}

/* vendor/openeva/prim/bn_fusion.h:19-60 fuse_bn + fold_bn_into_weight_2d. */
static int fold_conv_bn(const float* w, const float* cb, const float* g,
                        const float* b, const float* mu, const float* var,
                        int out_c, int in_c, float** W_out, float** b_out) {
    float* W  = (float*)malloc(sizeof(float) * out_c * in_c);
    float* bo = (float*)malloc(sizeof(float) * out_c);
    if (!W || !bo) return -1;
    for (int o = 0; o < out_c; ++o) {
        const float inv = 1.0f / sqrtf(var[o] + 1e-5f);
        const float s = g[o] * inv;
        const float shift = b[o] - (g[o] * mu[o]) * inv;
        for (int i = 0; i < in_c; ++i)
            W[(size_t)o * in_c + i] = w[(size_t)o * in_c + i] * s;
        const float bc = cb ? cb[o] : 0.0f;
        bo[o] = fmaf(bc, s, shift);
    }
    *W_out = W;
    *b_out = bo;
    return 0;
}

static float* dupf(const float* src, size_t n) {
    float* d = (float*)malloc(sizeof(float) * n);
    if (d) memcpy(d, src, sizeof(float) * n);
    return d;
}

OrModel* or_model_create(int H, int W, int tdrop_window,
                         const OrRawLayer* raw8, const OrRawHead* hd) {
    if (H <= 0 || W <= 0 || (H % 8) || (W % 8)) return NULL;
    OrModel* m = (OrModel*)calloc(1, sizeof(OrModel));
    if (!m) return NULL;
    m->H = H; m->W = W;
    m->tdrop_window = tdrop_window > 0 ? tdrop_window : 4;
    for (int l = 0; l < 8; ++l)
        if (build_layer(&m->L[l], &raw8[l]) != 0) { or_model_free(m); return NULL; }
    m->ncls = hd->ncls; m->c_in = hd->c_in; m->c_hid = hd->c_hid;
    m->stride_h = H / (H / 8);     /* src/ssla_kernels.cpp:231 */
    m->stride_w = W / (W / 8);
    if (fold_conv_bn(hd->cls_conv_w, hd->cls_conv_b, hd->cls_bn_w, hd->cls_bn_b,
                     hd->cls_bn_mean, hd->cls_bn_var, hd->c_hid, hd->c_in,
                     &m->cls_conv_W, &m->cls_conv_b) ||
        fold_conv_bn(hd->reg_conv_w, hd->reg_conv_b, hd->reg_bn_w, hd->reg_bn_b,
                     hd->reg_bn_mean, hd->reg_bn_var, hd->c_hid, hd->c_in,
                     &m->reg_conv_W, &m->reg_conv_b)) {
        or_model_free(m); return NULL;
    }
    m->cls_pred_W = dupf(hd->cls_pred_w, (size_t)hd->ncls * hd->c_hid);
    m->cls_pred_b = dupf(hd->cls_pred_b, (size_t)hd->ncls);
    m->reg_pred_W = dupf(hd->reg_pred_w, (size_t)4 * hd->c_hid);
    m->reg_pred_b = dupf(hd->reg_pred_b, 4);
    m->obj_pred_W = dupf(hd->obj_pred_w, (size_t)hd->c_hid);
    m->obj_pred_b = dupf(hd->obj_pred_b, 1);
    return m;
}

void or_model_free(OrModel* m) {
    if (!m) return;
    for (int l = 0; l < 8; ++l) {
        free(m->L[l].qvg); free(m->L[l].goW); free(m->L[l].ip);
        free(m->L[l].gamma); free(m->L[l].beta);
    }
    free(m->cls_conv_W); free(m->cls_conv_b); free(m->reg_conv_W);
    free(m->reg_conv_b); free(m->cls_pred_W); free(m->cls_pred_b);
    free(m->reg_pred_W); free(m->reg_pred_b); free(m->obj_pred_W);
    free(m->obj_pred_b);
    free(m);
}

/* ---------------------------------------------------------------------------
 * State
 * ------------------------------------------------------------------------- */

static int grid_cells(const OrModel* m, int s) {
    return (m->H >> s) * (m->W >> s);
}

/* Counter grid (stage index) of gate g under a layout. */
static int gate_grid(int layout, int g) {
    if (g == 0) return 1;
    if (g == 1) return 2;
    if (g == 2) return layout == OR_LAYOUT_HYBRID ? 2 : 3;
    return 3;
}

OrState* or_state_create(const OrModel* m, int layout) {
    OrState* s = (OrState*)calloc(1, sizeof(OrState));
    if (!s) return NULL;
    s->layout = layout;
    for (int l = 0; l < 8; ++l)
        s->hidden[l] = (float*)calloc((size_t)grid_cells(m, l / 2) * kChans[l / 2],
                                      sizeof(float));
    for (int g = 0; g < 4; ++g) {
        s->cnt_len[g] = grid_cells(m, gate_grid(layout, g));
        s->cnt[g] = (uint8_t*)calloc((size_t)s->cnt_len[g], 1);
    }
    const int n3 = grid_cells(m, 3), cols = 5 + m->ncls;
    s->last_t = (double*)malloc(sizeof(double) * (size_t)m->H * m->W);
    s->preds_dec = (float*)calloc((size_t)n3 * cols, sizeof(float));
    s->preds_raw = (float*)calloc((size_t)n3 * cols, sizeof(float));
    s->version = (uint32_t*)calloc((size_t)n3, sizeof(uint32_t));
    or_state_reset(m, s);
    return s;
}

void or_state_free(OrState* s) {
    if (!s) return;
    for (int l = 0; l < 8; ++l) free(s->hidden[l]);
    for (int g = 0; g < 4; ++g) free(s->cnt[g]);
    free(s->last_t); free(s->preds_dec); free(s->preds_raw); free(s->version);
    free(s);
}

/* Head decode of one cell (vendor/openeva/heads/async_yolox.h:203-254
 * decode_yolox_cell_ct).  dec = [cx, cy, w, h, obj, cls...]; raw = the
 * same values before decoding, ordered [reg0..3, obj, cls...] as the GPU
 * head writes them (orin/kernels/ssla_s2_s3_head_celled.cuh:887-898). */
static void head_cell(const OrModel* m, int gx, int gy, const float* feat,
                      float* dec, float* raw) {
    float cls_f[96], reg_f[96], cls[16], reg[4], obj;
    const int C = m->c_hid;
    matvec(feat, m->c_in, m->cls_conv_W, C, m->cls_conv_b, cls_f);
    for (int i = 0; i < C; ++i) cls_f[i] = cls_f[i] * or_sigmoidf(cls_f[i]);
    matvec(cls_f, C, m->cls_pred_W, m->ncls, m->cls_pred_b, cls);
    matvec(feat, m->c_in, m->reg_conv_W, C, m->reg_conv_b, reg_f);
    for (int i = 0; i < C; ++i) reg_f[i] = reg_f[i] * or_sigmoidf(reg_f[i]);
    matvec(reg_f, C, m->reg_pred_W, 4, m->reg_pred_b, reg);
    matvec(reg_f, C, m->obj_pred_W, 1, m->obj_pred_b, &obj);
    dec[0] = (reg[0] + (float)gx) * (float)m->stride_w;
    dec[1] = (reg[1] + (float)gy) * (float)m->stride_h;
    dec[2] = or_expf(reg[2]) * (float)m->stride_w;
    dec[3] = or_expf(reg[3]) * (float)m->stride_h;
    dec[4] = obj;
    for (int c = 0; c < m->ncls; ++c) dec[5 + c] = cls[c];
    for (int k = 0; k < 4; ++k) raw[k] = reg[k];
    raw[4] = obj;
    for (int c = 0; c < m->ncls; ++c) raw[5 + c] = cls[c];
}

/* Raw head outputs [reg0..3, obj, cls...] of one stage-3 feature (the
 * values the reference's GPU head writes, ssla_s2_s3_head_celled.cuh:
 * 841-902), for tests of kernels that write raw predictions. */
void or_head_raw(const OrModel* m, const float* feat, float* raw) {
    float dec[32];
    head_cell(m, 0, 0, feat, dec, raw);
}

/* src/ssla_kernels.cpp:276-286 reset + :969-989 prepopulate_head_zero. */
void or_state_reset(const OrModel* m, OrState* s) {
    for (int l = 0; l < 8; ++l)
        memset(s->hidden[l], 0,
               sizeof(float) * (size_t)grid_cells(m, l / 2) * kChans[l / 2]);
    for (int g = 0; g < 4; ++g) memset(s->cnt[g], 0, (size_t)s->cnt_len[g]);
    for (int i = 0; i < m->H * m->W; ++i) s->last_t[i] = -1.0;
    const int W3 = m->W >> 3, H3 = m->H >> 3, cols = 5 + m->ncls;
    float zero[96];
    memset(zero, 0, sizeof zero);
    for (int gy = 0; gy < H3; ++gy)
        for (int gx = 0; gx < W3; ++gx) {
            float raw[32];
            head_cell(m, gx, gy, zero, s->preds_dec + (size_t)(gy * W3 + gx) * cols, raw);
            memset(s->preds_raw + (size_t)(gy * W3 + gx) * cols, 0, sizeof(float) * cols);
        }
    memset(s->version, 0, sizeof(uint32_t) * (size_t)H3 * W3);
}

/* ---------------------------------------------------------------------------
 * Per-event pieces
 * ------------------------------------------------------------------------- */

/* src/ssla_kernels.cpp:315-385 layer_forward_ct (and the state-only variant
 * ssla_s2_s3_head_celled.cuh:249-290 when want_out == 0: the hidden-state
 * update is identical, the output work is skipped). */
void or_layer_forward(const OrModel* m, OrState* s, int l, int ex, int ey,
                      const float* in, float* out, int want_out) {
    const OrLayer* L = &m->L[l];
    const int stage = l / 2, IN = L->in_dim, OUT = L->out_dim;
    const int Hl = m->H >> stage, Wl = m->W >> stage;
    float* Hall = s->hidden[l];
    float residual[96], qvg[288], qh[96];
    if (want_out) {
        if (L->ip) matvec(in, IN, L->ip, OUT, NULL, residual);
        else memcpy(residual, in, sizeof(float) * OUT);
        for (int o = 0; o < OUT; ++o) out[o] = 0.0f;
    }
    for (int dy = -1; dy <= 1; ++dy) {
        for (int dx = -1; dx <= 1; ++dx) {
            int pos, px, py;
            if (L->A == 1) {
                if (dy != 0 || dx != 0) continue;
                pos = 0; px = ex; py = ey;
            } else {
                py = ey + dy; px = ex + dx;
                if (py < 0 || py >= Hl || px < 0 || px >= Wl) continue;
                pos = (1 - dy) * 3 + (1 - dx);      /* :375 */
            }
            /* process_patch :340-351 */
            matvec(in, IN, L->qvg + (size_t)pos * 3 * OUT * IN, 3 * OUT, NULL, qvg);
            float* h = Hall + (size_t)(py * Wl + px) * OUT;
            for (int c = 0; c < OUT; ++c) {          /* rnn.h:80-91 lru_step */
                const float gc = or_sigmoidf(qvg[2 * OUT + c]);
                const float hc = fmaf(gc, h[c], qvg[OUT + c]);
                h[c] = hc;
                qh[c] = qvg[c] * hc;
            }
            if (want_out)
                matvec_accum(qh, OUT, L->goW + (size_t)pos * OUT * OUT, OUT, out);
        }
    }
    if (want_out) {
        for (int o = 0; o < OUT; ++o) out[o] = out[o] + residual[o];
        layernorm(out, OUT, L->gamma, L->beta);
    }
}

/* src/ssla_kernels.cpp:912-921 tdrop_check_at (uint8 wrap) -- same rule as
 * the GPU parallel_tdrop, ssla_s2_s3_head_celled.cuh:719-747. */
static int gate(const OrModel* m, OrState* s, int g, int cx, int cy) {
    const int grid = gate_grid(s->layout, g);
    const int idx = cy * (m->W >> grid) + cx;
    const uint8_t pre = s->cnt[g][idx];
    s->cnt[g][idx] = (uint8_t)(pre + 1u);
    if (m->tdrop_window <= 1) return 1;
    return (pre % m->tdrop_window) == 0u;
}

static void head_write(const OrModel* m, OrState* s, int gx, int gy,
                       const float* feat) {
    const int W3 = m->W >> 3, cols = 5 + m->ncls;
    const int cell = gy * W3 + gx;
    head_cell(m, gx, gy, feat, s->preds_dec + (size_t)cell * cols,
              s->preds_raw + (size_t)cell * cols);
    s->version[cell] += 1u;
}

void or_run_events(const OrModel* m, OrState* s, const float* ev, int n,
                   uint8_t* flags, float* so0, float* so1, float* so2,
                   float* so3) {
    float f0[2], mid[96], s0o[12], s1o[24], s2o[48], s3o[96];
    const int hyb = s->layout == OR_LAYOUT_HYBRID;
    for (int i = 0; i < n; ++i) {
        const float t = ev[4 * i + 0], x = ev[4 * i + 1];
        const float y = ev[4 * i + 2], p = ev[4 * i + 3];
        uint8_t f = 0;
        /* Bounds rule of the drivers (s2_decomp_st.cpp:140-144,
         * lib_stage01_to_gpu.cpp:210-214): (int) truncation, then range. */
        if (!(x > -1.0f && x < (float)m->W && y > -1.0f && y < (float)m->H)) {
            if (flags) flags[i] = 0;
            continue;
        }
        const int ex = (int)x, ey = (int)y;
        f |= OR_F_VALID;
        /* preprocess, src/ssla_kernels.cpp:288-309 */
        {
            const int pidx = ey * m->W + ex;
            const double prev = s->last_t[pidx];
            float dt;
            if (prev < 0.0) dt = 1.0f;
            else {
                double v = ((double)t - prev) / 1e5;
                if (v < 0.0) v = 0.0;
                if (v > 1.0) v = 1.0;
                dt = (float)v;
            }
            s->last_t[pidx] = (double)t;
            f0[0] = dt;
            f0[1] = p;
        }
        const int x1 = ex >> 1, y1 = ey >> 1, x2 = ex >> 2, y2 = ey >> 2;
        const int x3 = ex >> 3, y3 = ey >> 3;
        /* stage 0 */
        const int r1 = gate(m, s, 0, x1, y1);
        or_layer_forward(m, s, 0, ex, ey, f0, mid, 1);
        or_layer_forward(m, s, 1, ex, ey, mid, s0o, r1);
        if (!r1) { if (flags) flags[i] = f; continue; }
        f |= OR_F_R1;
        if (so0) memcpy(so0 + (size_t)i * 12, s0o, sizeof s0o);
        /* stage 1 */
        const int r2 = gate(m, s, 1, x2, y2);
        or_layer_forward(m, s, 2, x1, y1, s0o, mid, 1);
        or_layer_forward(m, s, 3, x1, y1, mid, s1o, r2);
        if (!r2) { if (flags) flags[i] = f; continue; }
        f |= OR_F_R2;
        if (so1) memcpy(so1 + (size_t)i * 24, s1o, sizeof s1o);
        /* stage 2 */
        const int r3 = hyb ? gate(m, s, 2, x2, y2) : gate(m, s, 2, x3, y3);
        or_layer_forward(m, s, 4, x2, y2, s1o, mid, 1);
        or_layer_forward(m, s, 5, x2, y2, mid, s2o, r3);
        if (!r3) { if (flags) flags[i] = f; continue; }
        f |= OR_F_R3;
        if (so2) memcpy(so2 + (size_t)i * 48, s2o, sizeof s2o);
        /* stage 3 + head */
        const int r4 = hyb ? gate(m, s, 3, x3, y3) : 1;
        or_layer_forward(m, s, 6, x3, y3, s2o, mid, 1);
        or_layer_forward(m, s, 7, x3, y3, mid, s3o, r4);
        if (r4) {
            f |= OR_F_R4;
            if (so3) memcpy(so3 + (size_t)i * 96, s3o, sizeof s3o);
            head_write(m, s, x3, y3, s3o);
        }
        if (flags) flags[i] = f;
    }
}

void or_run_s2_records(const OrModel* m, OrState* s, const int* x2,
                       const int* y2, const float* feat1, const int* owner,
                       int n, int* pass2, int* pass3, float* s3_feat) {
    float l4o[48], s2o[48], l6o[96], s3o[96];
    for (int i = 0; i < n; ++i) {
        const int ex = x2[i], ey = y2[i];
        const int p2 = gate(m, s, 2, ex, ey);
        or_layer_forward(m, s, 4, ex, ey, feat1 + (size_t)i * 24, l4o, 1);
        or_layer_forward(m, s, 5, ex, ey, l4o, s2o, p2);
        const int x3 = ex >> 1, y3 = ey >> 1;
        int p3 = 0;
        if (p2) {
            p3 = gate(m, s, 3, x3, y3);
            or_layer_forward(m, s, 6, x3, y3, s2o, l6o, 1);
            or_layer_forward(m, s, 7, x3, y3, l6o, s3o, p3);
        }
        pass2[i] = owner[i] ? p2 : -1;
        pass3[i] = owner[i] ? (p2 ? p3 : 0) : -1;
        float* slot = s3_feat + (size_t)i * 96;
        if (p3) memcpy(slot, s3o, sizeof s3o);
        else if (p2) memcpy(slot, l6o, sizeof l6o);
        else {
            memcpy(slot, l4o, sizeof l4o);
            memset(slot + 48, 0, sizeof(float) * 48);
        }
    }
}
