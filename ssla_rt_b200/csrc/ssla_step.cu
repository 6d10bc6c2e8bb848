// Single-event step: one event through preprocess, the four tdrop gates,
// stages 0-3 and the head in one launch, for batch-of-1 latency.
//
// A cluster of 9 CTAs; CTA rank d owns patch position d (delta = (1-dy)*3 +
// (1-dx), the reference's numbering).  CTA 0 runs preprocess and the gates
// and all of stages 0-1 (their weights fit one CTA), holds the layer input,
// the residual and the LayerNorm, and runs the head.  Layers 4-7: every
// CTA copies the input row from CTA 0 (DSMEM), computes q, v, sigmoid(g) of
// its patch cell (matvec_ct<IN,3*OUT>, linear.h:80-90), updates the cell's
// state (lru_step, rnn.h:80-91) and, when the layer output is used, its goW
// contribution; after a cluster barrier CTA 0 sums the contributions in the
// reference's patch order (delta = 8..0, in-bounds only), adds the residual
// and normalises (layer_forward_ct, src/ssla_kernels.cpp:315-385;
// layernorm.h:41-62).
// Every value is formed with the same fmaf chains as the chunk engine and
// the C oracle, so a stepped event leaves bit-identical state.
// Weights, gamma / beta and the cells' state rows of the next layer are
// copied into shared memory with cp.async while the current layer runs.
#include <cooperative_groups.h>

#include <atomic>

#include "ssla_kernels.cuh"

namespace cg = cooperative_groups;

namespace ssla {

namespace {

constexpr int kStepNT = 512;
constexpr int kStepCTAs = 9;

// ---- shared-memory plan (floats) -------------------------------------------
// Layer buffers: [qvg A*IN*3*OUT][goW A*OUT*OUT][gamma][beta][cell rows A*OUT]
// [input_proj IN*OUT (first layers)], then (layers 0-3) scratch
// [qvg values A*3*OUT][q*h A*OUT][contributions A*OUT].
template <int IN, int OUT, int A>
struct [[maybe_unused]] Lay {
    static constexpr int J2 = 3 * OUT;
    static constexpr int WQ = A * IN * J2, WG = A * OUT * OUT;
    static constexpr int GAM = WQ + WG, BET = GAM + OUT, HR = BET + OUT, WI = HR + A * OUT;
    static constexpr int QV = WI + IN * OUT, QH = QV + A * J2, CON = QH + A * OUT;
    static constexpr int total = CON + A * OUT;
    static constexpr int layer = WI + IN * OUT;      // cluster layers: no scratch
};
// layers 0-3 (CTA 0): even layers at 0, odd layers at kSmallOdd
constexpr int kSmallOdd = Lay<12, 24, 9>::total;
// every CTA's layer-4 buffer, filled while CTA 0 runs layers 0-3
constexpr int kL4Base = kSmallOdd + Lay<24, 24, 9>::total;
// layers 5-7 and the head reuse the low region
constexpr int kSmem = kL4Base + Lay<24, 48, 1>::layer;
static_assert(Lay<2, 12, 1>::total <= kSmallOdd && Lay<12, 12, 9>::total <= kL4Base - kSmallOdd, "small");
static_assert(Lay<48, 48, 1>::layer <= kSmem && Lay<48, 96, 1>::layer <= kSmem &&
              Lay<96, 96, 1>::WI <= kSmem, "layers 5-7");
static_assert(kSmallOdd % 4 == 0 && kL4Base % 4 == 0, "alignment");

__device__ __forceinline__ bool step_gate(int pre, int window) {
    return window <= 1 || ((pre & 255) % window) == 0;
}

struct StepShared {
    float x[96];          // layer input (CTA 0 holds the authoritative copy)
    float qvg[288];       // q | v | g of this CTA's patch cell (layers 4-7)
    float qh[96];
    float contrib[96];    // goW[delta] * qh
    float res[96];        // CTA 0: residual of the current layer
    float y[96];          // CTA 0: pre-norm output
    float gb[192];        // CTA 0: gamma | beta kept aside from the copies
    float act[192];       // CTA 0: head conv activations (cls | reg)
    float hrow[24];       // CTA 0: head outputs (raw)
    double mean, inv;
    double d2[96];        // CTA 0: squared deviations of the LayerNorm
    double lt_prev;       // CTA 0: gate inputs loaded in parallel
    int cnt_in[4];
    int flags;
    int px, py;           // stage-0 pixel
};

// Asynchronous 16-byte copies (cp.async) of n floats (n % 4 == 0, both
// sides 16-byte aligned) by every thread of the CTA; async_commit() closes
// the group, async_wait() + __syncthreads() completes it.
__device__ __forceinline__ void stage_async(float* dst, const float* src, int n) {
    for (int t = threadIdx.x; t < n / 4; t += blockDim.x) {
        const unsigned sa = static_cast<unsigned>(__cvta_generic_to_shared(dst + 4 * t));
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" :: "r"(sa), "l"(src + 4 * t) : "memory");
    }
}
__device__ __forceinline__ void async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void async_wait() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// The patch cell of position d at stage s around (cx0, cy0); A == 1 is the
// event's own cell.
__device__ __forceinline__ bool patch_cell(int A, int d, int cx0, int cy0, int Ws, int Hs, int& cx, int& cy) {
    if (A == 1) { cx = cx0; cy = cy0; return true; }
    cx = cx0 + 1 - d % 3;
    cy = cy0 + 1 - d / 3;
    return cx >= 0 && cx < Ws && cy >= 0 && cy < Hs;
}

// LayerNorm of sh.y (OUT values) into sh.x: the two fp64 sums run
// sequentially in channel order by one thread, the squared deviations
// (the same rounded products) by all threads (layernorm.h:41-62).
__device__ __forceinline__ void step_ln(StepShared& sh, int OUT, const float* gam, const float* bet) {
    const int tid = threadIdx.x;
    if (tid == 0) {
        double sum = 0.0;
        for (int o = 0; o < OUT; ++o) sum += static_cast<double>(sh.y[o]);
        sh.mean = sum / static_cast<double>(OUT);
    }
    __syncthreads();
    const double mean = sh.mean;
    for (int o = tid; o < OUT; o += kStepNT) {
        const double dd = static_cast<double>(sh.y[o]) - mean;
        sh.d2[o] = dd * dd;
    }
    __syncthreads();
    if (tid == 0) {
        double var = 0.0;
        for (int o = 0; o < OUT; ++o) var += sh.d2[o];
        var /= static_cast<double>(OUT);
        sh.inv = 1.0 / sqrt(var + static_cast<double>(1e-5f));
    }
    __syncthreads();
    for (int t = tid; t < OUT; t += kStepNT) {
        const double tt = (static_cast<double>(sh.y[t]) - sh.mean) * sh.inv;
        sh.x[t] = static_cast<float>(tt * static_cast<double>(gam[t]) + static_cast<double>(bet[t]));
    }
}

// ---- layers 0-3 on CTA 0 ---------------------------------------------------
// Issues the copies of small layer l into its buffer: weights of every
// patch position, gamma / beta, the state rows of the in-bounds cells.
template <int IN, int OUT, int A>
__device__ void issue_small(int l, bool used, const StepArgs& a, int px, int py, float* wsm) {
    using Lo = Lay<IN, OUT, A>;
    const DevLayer& L = a.L[l];
    const int s = l / 2;
    float* b = wsm + ((l & 1) ? kSmallOdd : 0);
    stage_async(b, L.qvgT, Lo::WQ);
    if (used) {
        stage_async(b + Lo::WQ, L.goWT, Lo::WG);
        stage_async(b + Lo::GAM, L.gamma, OUT);
        stage_async(b + Lo::BET, L.beta, OUT);
        if ((l & 1) == 0) stage_async(b + Lo::WI, L.ipT, IN * OUT);
    }
    const int Ws = a.g.W[s], Hs = a.g.H[s];
    for (int d = 0; d < A; ++d) {
        int cx, cy;
        if (patch_cell(A, d, px >> s, py >> s, Ws, Hs, cx, cy))
            stage_async(b + Lo::HR + d * OUT, a.ps.hidden[l] + (static_cast<size_t>(cy) * Ws + cx) * OUT, OUT);
    }
    async_commit();
}

// One of layers 0-3 by CTA 0, every patch position: (position, column)
// items form q, v, sigmoid(g), (position, channel) items update the cells
// and (position, output) items form the goW contributions; the ordered
// sum, residual and LayerNorm follow.  Returns false when the layer is the
// event's last (state-only).
template <int IN, int OUT, int A, typename Next>
__device__ bool small_layer(int l, bool used, const StepArgs& a, int px, int py, StepShared& sh, float* wsm,
                            Next next_issue) {
    using Lo = Lay<IN, OUT, A>;
    constexpr int J2 = Lo::J2;
    const int tid = threadIdx.x;
    const int s = l / 2, half = l % 2;
    const int Ws = a.g.W[s], Hs = a.g.H[s], cx0 = px >> s, cy0 = py >> s;
    float* b = wsm + ((l & 1) ? kSmallOdd : 0);
    const float* wq = b;
    const float* wg = b + Lo::WQ;
    const float* wi = b + Lo::WI;
    const float* hr = b + Lo::HR;
    float* qvg = b + Lo::QV;
    float* qh = b + Lo::QH;
    float* con = b + Lo::CON;
    async_wait();                                // this layer's copies (issued earlier)
    __syncthreads();
    next_issue();                                // the next layer's, into the other buffer
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
        if (!patch_cell(A, d, cx0, cy0, Ws, Hs, cx, cy)) continue;
        float acc = 0.0f;
        const float* w = wq + d * IN * J2 + col;
#pragma unroll
        for (int i = 0; i < IN; ++i) acc = fmaf(w[i * J2], sh.x[i], acc);
        qvg[d * J2 + col] = acc;
    }
    __syncthreads();
    const int hd = tid / OUT, ht = tid % OUT;
    int hcx = 0, hcy = 0;
    const bool hact = tid < A * OUT && patch_cell(A, hd, cx0, cy0, Ws, Hs, hcx, hcy);
    if (hact) {
        const float* q = qvg + hd * J2;
        const float h = fmaf(ssla_sigmoidf(q[2 * OUT + ht]), hr[hd * OUT + ht], q[OUT + ht]);
        a.ps.hidden[l][(static_cast<size_t>(hcy) * Ws + hcx) * OUT + ht] = h;
        if (used) qh[hd * OUT + ht] = q[ht] * h;
    }
    if (!used) return false;                     // state-only second layer: the event ends
    __syncthreads();
    if (hact) {
        const float* w = wg + hd * OUT * OUT + ht;
        const float* q = qh + hd * OUT;
        float acc = 0.0f;
#pragma unroll
        for (int i = 0; i < OUT; ++i) acc = fmaf(w[i * OUT], q[i], acc);
        con[hd * OUT + ht] = acc;
    }
    __syncthreads();
    for (int t = tid; t < OUT; t += kStepNT) {
        float v = 0.0f;
#pragma unroll
        for (int d = A - 1; d >= 0; --d) {
            int cx, cy;
            if (!patch_cell(A, d, cx0, cy0, Ws, Hs, cx, cy)) continue;
            v = v + con[d * OUT + t];
        }
        sh.y[t] = v + sh.res[t];
    }
    __syncthreads();
    step_ln(sh, OUT, b + Lo::GAM, b + Lo::BET);
    __syncthreads();
    return true;
}

// Layers 0-3 (layer 0's copies were issued at kernel start).  Leaves the
// stage-2 input in sh.x when the event passes gate 1.
__device__ void small_layers(const StepArgs& a, int flags, int px, int py, StepShared& sh, float* wsm) {
    const bool r1 = (flags & F_R1) != 0, r2 = (flags & F_R2) != 0;
    if (!small_layer<2, 12, 1>(0, true, a, px, py, sh, wsm,
                               [&] { issue_small<12, 12, 9>(1, r1, a, px, py, wsm); }))
        return;
    if (!small_layer<12, 12, 9>(1, r1, a, px, py, sh, wsm,
                                [&] { if (r1) issue_small<12, 24, 9>(2, true, a, px, py, wsm); }))
        return;
    if (!small_layer<12, 24, 9>(2, true, a, px, py, sh, wsm,
                                [&] { issue_small<24, 24, 9>(3, r2, a, px, py, wsm); }))
        return;
    small_layer<24, 24, 9>(3, r2, a, px, py, sh, wsm, [] {});
}

// ---- layers 4-7 on the cluster ---------------------------------------------
struct StepLayer {
    int l, s, half, IN, OUT;
    bool used;      // the layer output is consumed (else state-only, last layer)
    bool act;       // this CTA's patch cell is in bounds
    int cx, cy;     // this CTA's patch cell
};

__device__ __forceinline__ bool step_layer(int l, int flags, int px, int py, int rank, const Geo& g,
                                           StepLayer& L) {
    const int s = l / 2, half = l % 2;
    if (s > 3 || s < 2) return false;
    if (!(flags & (F_R1 << (s - 1)))) return false;
    L.l = l;
    L.s = s;
    L.half = half;
    L.OUT = chans(s);
    L.IN = half == 0 ? chans(s - 1) : L.OUT;
    L.used = half == 0 || (s < 3 ? (flags & (F_R1 << s)) != 0 : (flags & F_R4) != 0);
    L.act = patch_cell(9, rank, px >> s, py >> s, g.W[s], g.H[s], L.cx, L.cy);
    return true;
}

__device__ __forceinline__ float* layer_base(float* wsm, int l) { return wsm + (l == 4 ? kL4Base : 0); }

// Offsets inside a layer-4..7 buffer (Lay<IN, OUT, 1> with runtime sizes).
__device__ __forceinline__ int off_gam(int IN, int OUT) { return IN * 3 * OUT + OUT * OUT; }

// Issues the copies a CTA needs for layer L: its patch position's weights
// and state row; CTA 0 also gamma, beta and input_proj (first layers).
__device__ void issue_layer(const StepLayer& L, const StepArgs& a, int rank, float* wsm) {
    const int IN = L.IN, OUT = L.OUT, J2 = 3 * OUT;
    const DevLayer& W = a.L[L.l];
    float* b = layer_base(wsm, L.l);
    const int gam = off_gam(IN, OUT);
    if (L.act) {
        stage_async(b, W.qvgT + static_cast<size_t>(rank) * IN * J2, IN * J2);
        if (L.used) stage_async(b + IN * J2, W.goWT + static_cast<size_t>(rank) * OUT * OUT, OUT * OUT);
        stage_async(b + gam + 2 * OUT,
                    a.ps.hidden[L.l] + (static_cast<size_t>(L.cy) * a.g.W[L.s] + L.cx) * OUT, OUT);
    }
    if (rank == 0 && L.used) {
        stage_async(b + gam, W.gamma, OUT);
        stage_async(b + gam + OUT, W.beta, OUT);
        if (L.half == 0) stage_async(b + gam + 3 * OUT, W.ipT, IN * OUT);
    }
    async_commit();
}

// One CTA's part of a layer 4-7: residual (CTA 0), q / v / sigmoid(g) of
// its patch cell, the cell's state update and its goW contribution.
template <int IN, int OUT>
__device__ void cl_compute(const StepLayer& cur, bool rank0, const StepArgs& a, StepShared& sh,
                           const float* b) {
    constexpr int J2 = 3 * OUT;
    constexpr int GAM = IN * J2 + OUT * OUT;
    const int tid = threadIdx.x;
    const bool used = cur.used;
    const float* wq = b;
    const float* wg = b + IN * J2;
    const float* wi = b + GAM + 3 * OUT;
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
        if (tid < OUT) {
            const float h = fmaf(ssla_sigmoidf(sh.qvg[2 * OUT + tid]), b[GAM + 2 * OUT + tid], sh.qvg[OUT + tid]);
            a.ps.hidden[cur.l][(static_cast<size_t>(cur.cy) * a.g.W[cur.s] + cur.cx) * OUT + tid] = h;
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
    if (rank0 && used) {
        // gamma / beta aside: the next layer's copies may reuse this buffer
        for (int t = tid; t < OUT; t += kStepNT) {
            sh.gb[t] = b[GAM + t];
            sh.gb[96 + t] = b[GAM + OUT + t];
        }
    }
}

// ---- head (CTA 0) ------------------------------------------------------------
// cls conv | reg conv [96][96], reg pred [96][4], obj pred [96], cls pred
// [96][ncls], cls | reg conv biases [96] each.
constexpr int kHeadRp = 2 * 96 * 96, kHeadOb = kHeadRp + 96 * 4, kHeadCp = kHeadOb + 96;
__device__ __forceinline__ int head_cb(int ncls) { return kHeadCp + ((96 * ncls + 3) & ~3); }

__device__ void issue_head(const DevHead& hd, int ncls, float* wsm) {
    stage_async(wsm, hd.cls_convT, 96 * 96);
    stage_async(wsm + 96 * 96, hd.reg_convT, 96 * 96);
    stage_async(wsm + kHeadRp, hd.reg_predT, 96 * 4);
    stage_async(wsm + kHeadOb, hd.obj_predT, 96);
    stage_async(wsm + kHeadCp, hd.cls_predT, 96 * ncls);
    stage_async(wsm + head_cb(ncls), hd.cls_conv_b, 96);
    stage_async(wsm + head_cb(ncls) + 96, hd.reg_conv_b, 96);
    async_commit();
}

__global__ void __launch_bounds__(kStepNT) k_step(StepArgs a) {
    cg::cluster_group cluster = cg::this_cluster();
    const int rank = static_cast<int>(cluster.block_rank());
    const int tid = threadIdx.x;
    __shared__ StepShared sh;
    extern __shared__ __align__(16) float wsm[];
    StepShared* sh0 = cluster.map_shared_rank(&sh, 0);
    const PartState& ps = a.ps;
    const Geo& g = a.g;
    const bool hyb = g.layout == LAYOUT_HYBRID;

    // ---- preprocess + gates (CTA 0): inputs loaded in parallel, decided by
    // one thread in gate order (each counter advances at most once) ----
    if (rank == 0) {
        const float4 e = a.ev;
        const bool valid = e.y > -1.0f && e.y < static_cast<float>(g.W[0]) && e.z > -1.0f &&
                           e.z < static_cast<float>(g.H[0]);
        const int x = valid ? static_cast<int>(e.y) : 0, y = valid ? static_cast<int>(e.z) : 0;
        const int k0 = (y >> 1) * g.W[1] + (x >> 1), k1 = (y >> 2) * g.W[2] + (x >> 2);
        const int k2 = hyb ? k1 : (y >> 3) * g.W[3] + (x >> 3), k3 = (y >> 3) * g.W[3] + (x >> 3);
        if (valid) {
            issue_small<2, 12, 1>(0, true, a, x, y, wsm);       // layer 0, needed by any valid event
            if (tid == 0) sh.lt_prev = ps.last_t[y * g.W[0] + x];
            else if (tid == 1) sh.cnt_in[0] = ps.cnt[0][k0];
            else if (tid == 2) sh.cnt_in[1] = ps.cnt[1][k1];
            else if (tid == 3) sh.cnt_in[2] = ps.cnt[2][k2];
            else if (tid == 4 && hyb) sh.cnt_in[3] = ps.cnt[3][k3];
        }
        __syncthreads();
        if (tid == 0) {
            int flags = 0;
            if (valid) {
                const double prev = sh.lt_prev;
                float dt;
                if (prev < 0.0) {
                    dt = 1.0f;
                } else {
                    double v = (static_cast<double>(e.x) - prev) / 1e5;
                    if (v < 0.0) v = 0.0;
                    if (v > 1.0) v = 1.0;
                    dt = static_cast<float>(v);
                }
                ps.last_t[y * g.W[0] + x] = static_cast<double>(e.x);
                flags = F_VALID;
                const int w = g.window;
                ps.cnt[0][k0] = static_cast<uint8_t>(sh.cnt_in[0] + 1);
                if (step_gate(sh.cnt_in[0], w)) {
                    flags |= F_R1;
                    ps.cnt[1][k1] = static_cast<uint8_t>(sh.cnt_in[1] + 1);
                    if (step_gate(sh.cnt_in[1], w)) {
                        flags |= F_R2;
                        ps.cnt[2][k2] = static_cast<uint8_t>(sh.cnt_in[2] + 1);
                        if (step_gate(sh.cnt_in[2], w)) {
                            flags |= F_R3;
                            bool pass3 = true;
                            if (hyb) {
                                ps.cnt[3][k3] = static_cast<uint8_t>(sh.cnt_in[3] + 1);
                                pass3 = step_gate(sh.cnt_in[3], w);
                            }
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
    }
    cluster.sync();
    const int flags = sh0->flags;
    const int px = sh0->px, py = sh0->py;

    if (flags & F_VALID) {
        // layer-4 copies of every CTA land while CTA 0 runs layers 0-3
        StepLayer cur;
        bool have = step_layer(4, flags, px, py, rank, g, cur);
        if (have) issue_layer(cur, a, rank, wsm);
        if (rank == 0) small_layers(a, flags, px, py, sh, wsm);
        cluster.sync();                    // stage-2 input ready in CTA 0
        bool head_issued = false;
        while (have) {
            const int OUT = cur.OUT;
            const int s = cur.s;
            const int Ws = g.W[s], Hs = g.H[s];
            const int cx0 = px >> s, cy0 = py >> s;
            const float* b = layer_base(wsm, cur.l);
            if (rank != 0)
                for (int t = tid; t < cur.IN; t += kStepNT) sh.x[t] = sh0->x[t];
            async_wait();
            __syncthreads();
            switch (cur.l) {
                case 4: cl_compute<24, 48>(cur, rank == 0, a, sh, b); break;
                case 5: cl_compute<48, 48>(cur, rank == 0, a, sh, b); break;
                case 6: cl_compute<48, 96>(cur, rank == 0, a, sh, b); break;
                default: cl_compute<96, 96>(cur, rank == 0, a, sh, b); break;
            }
            __syncthreads();               // this layer's weights are consumed
            if (!cur.used) break;          // state-only second layer: the event ends here
            StepLayer nxt;
            have = step_layer(cur.l + 1, flags, px, py, rank, g, nxt);
            if (have) {
                issue_layer(nxt, a, rank, wsm);   // lands during the gather / LayerNorm below
            } else if (rank == 0 && (flags & F_R4)) {
                issue_head(a.head, g.ncls, wsm);
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
                step_ln(sh, OUT, sh.gb, sh.gb + 96);
            }
            cluster.sync();                // next input ready in CTA 0
            cur = nxt;
        }
        async_wait();
        __syncthreads();
        // ---- head and commit (CTA 0) ----
        if (rank == 0 && (flags & F_R4)) {
            const DevHead& hd = a.head;
            const int ncls = g.ncls;
            if (!head_issued) issue_head(hd, ncls, wsm);
            const float obj_b = __ldg(hd.obj_pred_b);
            async_wait();
            __syncthreads();
            const float* wc = wsm;
            const float* wr = wsm + 96 * 96;
            const float* wrp = wsm + kHeadRp;
            const float* wob = wsm + kHeadOb;
            const float* wcp = wsm + kHeadCp;
            const float* cb = wsm + head_cb(ncls);
            for (int j = tid; j < 192; j += kStepNT) {
                const int jo = j % 96;
                const float* Wt = (j < 96) ? wc : wr;
                float acc = cb[j];
#pragma unroll 8
                for (int i = 0; i < 96; ++i) acc = fmaf(Wt[i * 96 + jo], sh.x[i], acc);
                sh.act[j] = acc * ssla_sigmoidf(acc);
            }
            __syncthreads();
            const int cols = 5 + ncls;
            for (int r = tid; r < cols; r += kStepNT) {
                float acc;
                if (r < 4) {
                    acc = __ldg(hd.reg_pred_b + r);
                    for (int i = 0; i < 96; ++i) acc = fmaf(wrp[i * 4 + r], sh.act[96 + i], acc);
                } else if (r == 4) {
                    acc = obj_b;
                    for (int i = 0; i < 96; ++i) acc = fmaf(wob[i], sh.act[96 + i], acc);
                } else {
                    const int c = r - 5;
                    acc = __ldg(hd.cls_pred_b + c);
                    for (int i = 0; i < 96; ++i) acc = fmaf(wcp[i * ncls + c], sh.act[i], acc);
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
    async_wait();                          // no copy in flight at exit
    cluster.sync();                        // no CTA leaves while its smem may be read
}

}  // namespace

cudaError_t launch_step(cudaStream_t st, const StepArgs& a) {
    constexpr size_t smem = sizeof(float) * kSmem;
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
