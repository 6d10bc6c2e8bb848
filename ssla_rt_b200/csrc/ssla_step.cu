// Single-event step: one event through preprocess, the four tdrop gates,
// stages 0-3 and the head in one launch, for batch-of-1 latency.
//
// A cluster of 9 CTAs; CTA rank d owns patch position d (delta = (1-dy)*3 +
// (1-dx), the reference's numbering).  CTA 0 also runs preprocess and the
// gates, holds the layer input, the residual and the LayerNorm, and runs
// the head.  Per layer: every CTA copies the input row from CTA 0 (DSMEM),
// computes q, v, sigmoid(g) of its patch cell (matvec_ct<IN,3*OUT>,
// linear.h:80-90), updates the cell's state (lru_step, rnn.h:80-91) and,
// when the layer output is used, its goW contribution; after a cluster
// barrier CTA 0 sums the contributions in the reference's patch order
// (delta = 8..0, in-bounds only), adds the residual and normalises
// (layer_forward_ct, src/ssla_kernels.cpp:315-385; layernorm.h:41-62).
// Every value is formed with the same fmaf chains as the chunk engine and
// the C oracle, so a stepped event leaves bit-identical state.
#include <cooperative_groups.h>

#include <atomic>

#include "ssla_kernels.cuh"

namespace cg = cooperative_groups;

namespace ssla {

namespace {

constexpr int kStepNT = 512;
// weight staging buffer (floats): the largest qvg slice + goW slice (layer 7),
// also reused for the residual and head weights
constexpr int kStepW = 96 * 288 + 96 * 96;
constexpr int kStepCTAs = 9;

__device__ __forceinline__ bool step_gate(uint8_t* c, int window) {
    const int pre = *c;
    *c = static_cast<uint8_t>(pre + 1);
    return window <= 1 || ((pre & 255) % window) == 0;
}

struct StepShared {
    float x[96];          // layer input (CTA 0 holds the authoritative copy)
    float qvg[288];       // q | v | g of this CTA's patch cell
    float qh[96];
    float contrib[96];    // goW[delta] * qh
    float res[96];        // CTA 0: residual of the current layer
    float y[96];          // CTA 0: pre-norm output
    float act[192];       // CTA 0: head conv activations (cls | reg)
    float hrow[24];       // CTA 0: head outputs (raw)
    double mean, inv;
    int flags;
    int px, py;           // stage-0 pixel
};

// Copies n floats (n % 4 == 0, 16-byte aligned) into shared memory with
// independent 16-byte loads from every thread.
__device__ __forceinline__ void stage(float* dst, const float* src, int n) {
    for (int t = threadIdx.x; t < n / 4; t += blockDim.x)
        reinterpret_cast<float4*>(dst)[t] = __ldg(reinterpret_cast<const float4*>(src) + t);
}

// Same, as asynchronous 16-byte copies (cp.async); complete after
// async_wait() + __syncthreads().
__device__ __forceinline__ void stage_async(float* dst, const float* src, int n) {
    for (int t = threadIdx.x; t < n / 4; t += blockDim.x) {
        const unsigned sa = static_cast<unsigned>(__cvta_generic_to_shared(dst + 4 * t));
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" :: "r"(sa), "l"(src + 4 * t) : "memory");
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
}

__device__ __forceinline__ void async_wait() {
    asm volatile("cp.async.wait_group 0;" ::: "memory");
}

// One layer of the event's path as seen by one CTA.
struct StepLayer {
    int l, s, half, IN, OUT, A;
    bool used;      // the layer output is consumed (else state-only, last layer)
    bool act;       // this CTA's patch cell is in bounds
    int d, cx, cy;  // patch position and cell
};

__device__ __forceinline__ bool step_layer(int idx, int flags, int px, int py, int rank, const Geo& g,
                                           StepLayer& L) {
    const int s = idx / 2, half = idx % 2;
    if (s > 3) return false;
    if (s > 0 && !(flags & (F_R1 << (s - 1)))) return false;
    if (half == 1) {
        // the first layer of the stage always runs; the second follows it
    }
    L.l = idx;
    L.s = s;
    L.half = half;
    L.OUT = chans(s);
    L.IN = (idx == 0) ? 2 : (half == 0 ? chans(s - 1) : L.OUT);
    L.A = (idx == 0) ? 1 : 9;
    L.used = half == 0 || (s < 3 ? (flags & (F_R1 << s)) != 0 : (flags & F_R4) != 0);
    const int cx0 = px >> s, cy0 = py >> s;
    if (L.A == 1) {
        L.d = 0;
        L.cx = cx0;
        L.cy = cy0;
        L.act = rank == 0;
    } else {
        L.d = rank;
        L.cx = cx0 + 1 - rank % 3;
        L.cy = cy0 + 1 - rank / 3;
        L.act = L.cx >= 0 && L.cx < g.W[s] && L.cy >= 0 && L.cy < g.H[s];
    }
    return true;
}

// Issues the weight copies a CTA needs for layer L into wsm:
// qvg [IN][3*OUT] | goW [OUT][OUT] | (CTA 0, first layers) input_proj [IN][OUT].
__device__ __forceinline__ void issue_layer(const StepLayer& L, const DevLayer* layers, int rank, float* wsm) {
    const int J2 = 3 * L.OUT;
    const DevLayer& W = layers[L.l];
    if (L.act) {
        stage_async(wsm, W.qvgT + static_cast<size_t>(L.d) * L.IN * J2, L.IN * J2);
        if (L.used) stage_async(wsm + L.IN * J2, W.goWT + static_cast<size_t>(L.d) * L.OUT * L.OUT, L.OUT * L.OUT);
    }
    if (rank == 0 && L.used && L.half == 0)
        stage_async(wsm + L.IN * J2 + L.OUT * L.OUT, W.ipT, L.IN * L.OUT);
}

// Head weights for CTA 0: cls conv | reg conv [96][96], reg pred [96][4]
// (obj / cls preds are read directly, they are small).
__device__ __forceinline__ void issue_head(const DevHead& hd, float* wsm) {
    stage_async(wsm, hd.cls_convT, 96 * 96);
    stage_async(wsm + 96 * 96, hd.reg_convT, 96 * 96);
    stage_async(wsm + 2 * 96 * 96, hd.reg_predT, 96 * 4);
}

// LayerNorm of sh.y (OUT values) into sh.x: sequential fp64 statistics by
// one thread (layernorm.h:41-62), then the per-channel normalisation.
__device__ __forceinline__ void step_ln(StepShared& sh, int OUT, const DevLayer& L) {
    const int tid = threadIdx.x;
    if (tid == 0) {
        double sum = 0.0;
        for (int o = 0; o < OUT; ++o) sum += static_cast<double>(sh.y[o]);
        const double mean = sum / static_cast<double>(OUT);
        double var = 0.0;
        for (int o = 0; o < OUT; ++o) {
            const double dd = static_cast<double>(sh.y[o]) - mean;
            var += dd * dd;
        }
        var /= static_cast<double>(OUT);
        sh.mean = mean;
        sh.inv = 1.0 / sqrt(var + static_cast<double>(1e-5f));
    }
    __syncthreads();
    for (int t = tid; t < OUT; t += kStepNT) {
        const double tt = (static_cast<double>(sh.y[t]) - sh.mean) * sh.inv;
        sh.x[t] = static_cast<float>(tt * static_cast<double>(__ldg(L.gamma + t)) +
                                     static_cast<double>(__ldg(L.beta + t)));
    }
}

// One of layers 0-3 of one event by one CTA, every patch position: the
// weights of all positions are staged, then (position, column) items form
// q, v, sigmoid(g), (position, channel) items update the cells and
// (position, output) items form the goW contributions; the ordered sum,
// residual and LayerNorm follow.  Returns false when the layer is the
// event's last (state-only).
template <int IN, int OUT, int A>
__device__ bool small_layer(int l, bool used, const StepArgs& a, int px, int py, StepShared& sh, float* wsm) {
    constexpr int J2 = 3 * OUT;
    const int tid = threadIdx.x;
    const int s = l / 2, half = l % 2;
    const DevLayer& L = a.L[l];
    const Geo& g = a.g;
    const int Ws = g.W[s], Hs = g.H[s], cx0 = px >> s, cy0 = py >> s;
    float* wq = wsm;                              // [A][IN][J2]
    float* wg = wq + A * IN * J2;                 // [A][OUT][OUT]
    float* wi = wg + A * OUT * OUT;               // [IN][OUT]
    float* qvg = wi + IN * OUT;                   // [A][J2]
    float* qh = qvg + A * J2;                     // [A][OUT]
    float* con = qh + A * OUT;                    // [A][OUT]
    auto cell_of = [&](int d, int& cx, int& cy) {
        if (A == 1) { cx = cx0; cy = cy0; return true; }
        cx = cx0 + 1 - d % 3;
        cy = cy0 + 1 - d / 3;
        return cx >= 0 && cx < Ws && cy >= 0 && cy < Hs;
    };
    // this thread's (position, channel) item: its cell state, loaded early
    const int hd = tid / OUT, ht = tid % OUT;
    float* hp = nullptr;
    float h_old = 0.0f;
    if (tid < A * OUT) {
        int cx, cy;
        if (cell_of(hd, cx, cy)) {
            hp = a.ps.hidden[l] + (static_cast<size_t>(cy) * Ws + cx) * OUT + ht;
            h_old = *hp;
        }
    }
    stage(wq, L.qvgT, A * IN * J2);
    if (used) stage(wg, L.goWT, A * OUT * OUT);
    if (used && half == 0) stage(wi, L.ipT, IN * OUT);
    __syncthreads();
    if (used) {
        for (int t = tid; t < OUT; t += kStepNT) {
            float acc;
            if (half == 0) {
                acc = 0.0f;
#pragma unroll
                for (int i = 0; i < IN; ++i) acc = fmaf(wi[i * OUT + t], sh.x[i], acc);
            } else {
                acc = sh.x[t];
            }
            sh.res[t] = acc;
        }
    }
    const int c0 = used ? 0 : OUT;
    for (int it = tid; it < A * (J2 - c0); it += kStepNT) {
        const int d = it / (J2 - c0), col = c0 + it % (J2 - c0);
        int cx, cy;
        if (!cell_of(d, cx, cy)) continue;
        float acc = 0.0f;
        const float* w = wq + d * IN * J2 + col;
#pragma unroll
        for (int i = 0; i < IN; ++i) acc = fmaf(w[i * J2], sh.x[i], acc);
        qvg[d * J2 + col] = acc;
    }
    __syncthreads();
    if (hp) {
        const float* q = qvg + hd * J2;
        const float h = fmaf(ssla_sigmoidf(q[2 * OUT + ht]), h_old, q[OUT + ht]);
        *hp = h;
        if (used) qh[hd * OUT + ht] = q[ht] * h;
    }
    if (!used) return false;                     // state-only second layer: the event ends
    __syncthreads();
    if (tid < A * OUT) {
        int cx, cy;
        if (cell_of(hd, cx, cy)) {
            const float* w = wg + hd * OUT * OUT + ht;
            const float* q = qh + hd * OUT;
            float acc = 0.0f;
#pragma unroll
            for (int i = 0; i < OUT; ++i) acc = fmaf(w[i * OUT], q[i], acc);
            con[hd * OUT + ht] = acc;
        }
    }
    __syncthreads();
    for (int t = tid; t < OUT; t += kStepNT) {
        float v = 0.0f;
#pragma unroll
        for (int d = A - 1; d >= 0; --d) {
            int cx, cy;
            if (!cell_of(d, cx, cy)) continue;
            v = v + con[d * OUT + t];
        }
        sh.y[t] = v + sh.res[t];
    }
    __syncthreads();
    step_ln(sh, OUT, L);
    __syncthreads();
    return true;
}

// Layers 0-3 (the event reaches stage 1 when gate 0 passed).  Leaves the
// stage-2 input in sh.x when the event passes gate 1.
__device__ void small_layers(const StepArgs& a, int flags, int px, int py, StepShared& sh, float* wsm) {
    if (!small_layer<2, 12, 1>(0, true, a, px, py, sh, wsm)) return;
    if (!small_layer<12, 12, 9>(1, (flags & F_R1) != 0, a, px, py, sh, wsm)) return;
    if (!small_layer<12, 24, 9>(2, true, a, px, py, sh, wsm)) return;
    small_layer<24, 24, 9>(3, (flags & F_R2) != 0, a, px, py, sh, wsm);
}

// One CTA's part of layers 4-7: residual (CTA 0), q / v / sigmoid(g) of its
// patch cell, the cell's state update and its goW contribution.
template <int IN, int OUT>
__device__ void cl_compute(const StepLayer& cur, bool rank0, const StepArgs& a, StepShared& sh,
                           const float* wsm, float h_old, float* hp) {
    constexpr int J2 = 3 * OUT;
    const int tid = threadIdx.x;
    const bool used = cur.used;
    const float* wq = wsm;
    const float* wg = wsm + IN * J2;
    const float* wi = wg + OUT * OUT;
    if (rank0 && used) {
        for (int t = tid; t < OUT; t += kStepNT) {
            float acc;
            if (cur.half == 0) {
                acc = 0.0f;
#pragma unroll
                for (int i = 0; i < IN; ++i) acc = fmaf(wi[i * OUT + t], sh.x[i], acc);
            } else {
                acc = sh.x[t];
            }
            sh.res[t] = acc;
        }
    }
    if (cur.act) {
        for (int col = tid + (used ? 0 : OUT); col < J2; col += kStepNT) {
            float acc = 0.0f;
            const float* w = wq + col;
#pragma unroll
            for (int i = 0; i < IN; ++i) acc = fmaf(w[i * J2], sh.x[i], acc);
            sh.qvg[col] = acc;
        }
        __syncthreads();
        if (hp) {
            const float h = fmaf(ssla_sigmoidf(sh.qvg[2 * OUT + tid]), h_old, sh.qvg[OUT + tid]);
            *hp = h;
            if (used) sh.qh[tid] = sh.qvg[tid] * h;
        }
        __syncthreads();
        if (used && tid < OUT) {
            float acc = 0.0f;
#pragma unroll
            for (int i = 0; i < OUT; ++i) acc = fmaf(wg[i * OUT + tid], sh.qh[i], acc);
            sh.contrib[tid] = acc;
        }
    }
}

__global__ void __launch_bounds__(kStepNT) k_step(StepArgs a) {
    cg::cluster_group cluster = cg::this_cluster();
    const int rank = static_cast<int>(cluster.block_rank());
    const int tid = threadIdx.x;
    __shared__ StepShared sh;
    extern __shared__ __align__(16) float wsm[];      // [kStepW] staged weights
    StepShared* sh0 = cluster.map_shared_rank(&sh, 0);
    const PartState& ps = a.ps;
    const Geo& g = a.g;
    const bool hyb = g.layout == LAYOUT_HYBRID;

    // ---- preprocess + gates (CTA 0, one thread) ----
    if (rank == 0 && tid == 0) {
        const float4 e = a.ev;
        int flags = 0;
        if (e.y > -1.0f && e.y < static_cast<float>(g.W[0]) && e.z > -1.0f && e.z < static_cast<float>(g.H[0])) {
            const int x = static_cast<int>(e.y), y = static_cast<int>(e.z);
            double* lt = ps.last_t + y * g.W[0] + x;
            const double prev = *lt;
            float dt;
            if (prev < 0.0) {
                dt = 1.0f;
            } else {
                double v = (static_cast<double>(e.x) - prev) / 1e5;
                if (v < 0.0) v = 0.0;
                if (v > 1.0) v = 1.0;
                dt = static_cast<float>(v);
            }
            *lt = static_cast<double>(e.x);
            flags = F_VALID;
            const int w = g.window;
            const bool pass0 = step_gate(ps.cnt[0] + (y >> 1) * g.W[1] + (x >> 1), w);
            if (pass0) {
                flags |= F_R1;
                const bool pass1 = step_gate(ps.cnt[1] + (y >> 2) * g.W[2] + (x >> 2), w);
                if (pass1) {
                    flags |= F_R2;
                    const bool pass2 = hyb ? step_gate(ps.cnt[2] + (y >> 2) * g.W[2] + (x >> 2), w)
                                           : step_gate(ps.cnt[2] + (y >> 3) * g.W[3] + (x >> 3), w);
                    if (pass2) {
                        flags |= F_R3;
                        const bool pass3 = hyb ? step_gate(ps.cnt[3] + (y >> 3) * g.W[3] + (x >> 3), w) : true;
                        if (pass3) flags |= F_R4;
                    }
                }
            }
            sh.px = x;
            sh.py = y;
            sh.x[0] = dt;
            sh.x[1] = e.w;
        }
        sh.flags = flags;
        if (a.flag_out) *a.flag_out = static_cast<uint8_t>(flags);
    }
    cluster.sync();
    const int flags = sh0->flags;
    const int px = sh0->px, py = sh0->py;

    if (flags & F_VALID) {
        // ---- stages 0-1 (layers 0-3) on CTA 0 alone: all patch positions of
        // these small layers fit one CTA, so no cluster barrier is needed;
        // the other CTAs prefetch their layer-4 weights meanwhile.
        StepLayer cur;
        bool have = (flags & F_R2) && step_layer(4, flags, px, py, rank, g, cur);
        if (have && rank != 0) issue_layer(cur, a.L, rank, wsm);
        if (rank == 0) small_layers(a, flags, px, py, sh, wsm);
        cluster.sync();                    // stage-2 input ready in CTA 0
        if (have && rank == 0) issue_layer(cur, a.L, rank, wsm);
        bool head_issued = false;
        while (have) {
            const int IN = cur.IN, OUT = cur.OUT;
            const int s = cur.s;
            const int Ws = g.W[s], Hs = g.H[s];
            const int cx0 = px >> s, cy0 = py >> s;
            const bool used = cur.used;
            const DevLayer& L = a.L[cur.l];
            // the cell state and the layer input (DSMEM) while the weights arrive
            float* hp = nullptr;
            float h_old = 0.0f;
            if (cur.act && tid < OUT) {
                hp = ps.hidden[cur.l] + (static_cast<size_t>(cur.cy) * Ws + cur.cx) * OUT + tid;
                h_old = *hp;
            }
            if (rank != 0)
                for (int t = tid; t < IN; t += kStepNT) sh.x[t] = sh0->x[t];
            async_wait();
            __syncthreads();
            switch (cur.l) {
                case 4: cl_compute<24, 48>(cur, rank == 0, a, sh, wsm, h_old, hp); break;
                case 5: cl_compute<48, 48>(cur, rank == 0, a, sh, wsm, h_old, hp); break;
                case 6: cl_compute<48, 96>(cur, rank == 0, a, sh, wsm, h_old, hp); break;
                default: cl_compute<96, 96>(cur, rank == 0, a, sh, wsm, h_old, hp); break;
            }
            __syncthreads();               // this layer's weights are consumed
            if (!used) break;              // state-only second layer: the event ends here
            StepLayer nxt;
            have = step_layer(cur.l + 1, flags, px, py, rank, g, nxt);
            if (have) {
                issue_layer(nxt, a.L, rank, wsm);   // lands during the gather / LayerNorm below
            } else if (rank == 0 && (flags & F_R4)) {
                issue_head(a.head, wsm);
                head_issued = true;
            }
            cluster.sync();                // contributions ready, inputs copied
            if (rank == 0) {
                for (int t = tid; t < OUT; t += kStepNT) {
                    float c[9];
#pragma unroll
                    for (int dd = 0; dd < 9; ++dd) {          // all remote loads in flight
                        const int ccx = cx0 + 1 - dd % 3, ccy = cy0 + 1 - dd / 3;
                        const bool in = ccx >= 0 && ccx < Ws && ccy >= 0 && ccy < Hs;
                        c[dd] = in ? cluster.map_shared_rank(&sh, dd)->contrib[t] : 0.0f;
                    }
                    float v = 0.0f;
#pragma unroll
                    for (int dd = 8; dd >= 0; --dd) {
                        const int ccx = cx0 + 1 - dd % 3, ccy = cy0 + 1 - dd / 3;
                        if (ccx < 0 || ccx >= Ws || ccy < 0 || ccy >= Hs) continue;
                        v = v + c[dd];
                    }
                    sh.y[t] = v + sh.res[t];
                }
                __syncthreads();
                step_ln(sh, OUT, L);
            }
            cluster.sync();                // next input ready in CTA 0
            cur = nxt;
        }
        async_wait();
        __syncthreads();
        // ---- head and commit (CTA 0) ----
        if (rank == 0 && (flags & F_R4)) {
            const DevHead& hd = a.head;
            // staged (issue_head): cls conv | reg conv [96][96] each, reg [96][4];
            // obj [96] and cls [96][ncls] follow here
            float* wc = wsm;
            float* wr = wsm + 96 * 96;
            float* wrp = wsm + 2 * 96 * 96;
            float* wob = wrp + 96 * 4;
            float* wcp = wob + 96;
            if (!head_issued) {
                stage(wc, hd.cls_convT, 96 * 96);
                stage(wr, hd.reg_convT, 96 * 96);
                stage(wrp, hd.reg_predT, 96 * 4);
            }
            for (int t = tid; t < 96; t += kStepNT) wob[t] = __ldg(hd.obj_predT + t);
            for (int t = tid; t < 96 * g.ncls; t += kStepNT) wcp[t] = __ldg(hd.cls_predT + t);
            __syncthreads();
            for (int j = tid; j < 192; j += kStepNT) {
                const int jo = j % 96;
                const float* Wt = (j < 96) ? wc : wr;
                float acc = __ldg(((j < 96) ? hd.cls_conv_b : hd.reg_conv_b) + jo);
#pragma unroll 8
                for (int i = 0; i < 96; ++i) acc = fmaf(Wt[i * 96 + jo], sh.x[i], acc);
                sh.act[j] = acc * ssla_sigmoidf(acc);
            }
            __syncthreads();
            const int cols = 5 + g.ncls;
            for (int r = tid; r < cols; r += kStepNT) {
                float acc;
                if (r < 4) {
                    acc = __ldg(hd.reg_pred_b + r);
                    for (int i = 0; i < 96; ++i) acc = fmaf(wrp[i * 4 + r], sh.act[96 + i], acc);
                } else if (r == 4) {
                    acc = __ldg(hd.obj_pred_b);
                    for (int i = 0; i < 96; ++i) acc = fmaf(wob[i], sh.act[96 + i], acc);
                } else {
                    const int c = r - 5;
                    acc = __ldg(hd.cls_pred_b + c);
                    for (int i = 0; i < 96; ++i) acc = fmaf(wcp[i * g.ncls + c], sh.act[i], acc);
                }
                sh.hrow[r] = acc;
            }
            __syncthreads();
            const int c3x = px >> 3, c3y = py >> 3;
            const int x2 = px >> 2, y2 = py >> 2;
            const bool own = x2 >= ps.own_x0 && x2 < ps.own_x1 && y2 >= ps.own_y0 && y2 < ps.own_y1;
            const int cell = c3y * g.W[3] + c3x;
            for (int r = tid; r < cols; r += kStepNT) {
                const float v = sh.hrow[r];
                float dv;
                if (r == 0) dv = (v + static_cast<float>(c3x)) * static_cast<float>(g.stride_w);
                else if (r == 1) dv = (v + static_cast<float>(c3y)) * static_cast<float>(g.stride_h);
                else if (r == 2) dv = ssla_expf(v) * static_cast<float>(g.stride_w);
                else if (r == 3) dv = ssla_expf(v) * static_cast<float>(g.stride_h);
                else dv = v;
                if (own) {
                    ps.preds_dec[static_cast<size_t>(cell) * cols + r] = dv;
                    ps.preds_raw[static_cast<size_t>(cell) * cols + r] = v;
                }
                if (a.pred_out) a.pred_out[r] = dv;
            }
            if (own && tid == 0) ps.version[cell] += 1u;
        }
    }
    cluster.sync();                        // no CTA leaves while its smem may be read
}

}  // namespace

cudaError_t launch_step(cudaStream_t st, const StepArgs& a) {
    constexpr size_t smem = sizeof(float) * kStepW;
    // function attributes are per device: set once for each device used
    static std::atomic<unsigned long long> attr_done{0};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const unsigned long long bit = 1ull << (dev & 63);
    if (!(attr_done.load(std::memory_order_acquire) & bit)) {
        e = cudaFuncSetAttribute(k_step, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(k_step, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        attr_done.fetch_or(bit, std::memory_order_acq_rel);
    }
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(kStepCTAs);
    cfg.blockDim = dim3(kStepNT);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = kStepCTAs;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, k_step, a);
}

}  // namespace ssla
