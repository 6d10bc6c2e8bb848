// Single-event step: one event through preprocess, the four tdrop gates,
// stages 0-3 and the head in one launch, for batch-of-1 latency.
//
// A cluster of 9 CTAs; CTA rank d owns patch position d (delta = (1-dy)*3 +
// (1-dx), the reference's numbering).  Every CTA reads the gate counters and
// derives the event's reach bits itself, so no CTA waits for a decision.
// CTA 0 runs preprocess and all of stages 0-1 (their weights fit one CTA),
// holds the layer input, the residual and the LayerNorm, and runs the head.
// Layers 4-7 are message-passing between CTA 0 and the CTAs whose patch cell
// is in bounds: CTA 0 sends the layer input into their shared memory
// (st.async, completing on the receiver's mbarrier); each computes q, v,
// sigmoid(g) of its cell (matvec_ct<IN,3*OUT>, linear.h:80-90), updates the
// cell's state (lru_step, rnn.h:80-91) and sends its goW contribution back
// the same way; CTA 0 sums the contributions in the reference's patch order
// (delta = 8..0, in-bounds only), adds the residual and normalises
// (layer_forward_ct, src/ssla_kernels.cpp:315-385; layernorm.h:41-62).
// Weights, gamma / beta and the cells' state rows reach shared memory by bulk
// copies issued as soon as their buffer is free, each layer completing on its
// own mbarrier.  Every wait is bounded (cl::kWaitNs); a wait that runs out sets a
// bit in the caller's status word and the kernel carries on to its end.
// Every value is formed with the same fmaf chains as the chunk engine and
// the C oracle, so a stepped event leaves bit-identical state.
#include <atomic>

#include "ssla_cluster.cuh"
#include "ssla_kernels.cuh"

namespace ssla {

namespace {

using namespace cl;

constexpr int kStepNT = 512;
constexpr int kStepCTAs = 9;
constexpr int kIssuer = kStepNT - 32;                         // lane 0 of the last warp issues copies

// ---- shared-memory plan (floats) -------------------------------------------
// A layer buffer: [qvg A*IN*3*OUT][goW A*OUT*OUT][gamma][beta][cell rows A*OUT]
// [input_proj IN*OUT (first layers)], then (layers 0-3) scratch
// [qvg values A*3*OUT][q*h A*OUT][contributions A*OUT].
#pragma nv_diag_suppress 177   // not every layer uses every offset of its plan
template <int IN, int OUT, int A>
struct Lay {
    static constexpr int J2 = 3 * OUT;
    static constexpr int WQ = A * IN * J2, WG = A * OUT * OUT;
    static constexpr int GAM = WQ + WG, BET = GAM + OUT, HR = BET + OUT, WI = HR + A * OUT;
    static constexpr int QV = WI + IN * OUT, QH = QV + A * J2, CON = QH + A * OUT;
    static constexpr int total = CON + A * OUT;
    static constexpr int layer = WI + IN * OUT;      // layers 4-7: no scratch
};
// CTA 0, from kernel start: layers 0-3 back to back, then layer 4.
constexpr int kS1 = Lay<2, 12, 1>::total;
constexpr int kS2 = kS1 + Lay<12, 12, 9>::total;
constexpr int kS3 = kS2 + Lay<12, 24, 9>::total;
constexpr int kR4 = kS3 + Lay<24, 24, 9>::total;
// Layers 5-7 (one patch position each): layer 6 at 0, layer 5 above it; layer
// 7's qvg block over the layer 4/5 buffers, its goW | gamma | beta | row at 0.
// The head (CTA 0) at 0 once layers 6 and 7 no longer need it.
constexpr int kR6 = 0;
constexpr int kR5 = Lay<48, 96, 1>::layer;
constexpr int kR7q = kR5;
constexpr int kR7 = 0;
constexpr int kRH = 0;
constexpr int kDyn = (kR4 + Lay<24, 48, 1>::layer) > (kR7q + 96 * 288) ? (kR4 + Lay<24, 48, 1>::layer)
                                                                       : (kR7q + 96 * 288);
static_assert(kR5 + Lay<48, 48, 1>::WI <= kR4, "layer 5 below layer 4");
static_assert(kR7 + 96 * 96 + 3 * 96 <= kR7q, "layer 7 goW below its qvg block");
static_assert(kS1 % 4 == 0 && kS2 % 4 == 0 && kS3 % 4 == 0 && kR4 % 4 == 0 && kR5 % 4 == 0,
              "16-byte aligned buffers");
// head: cls conv | reg conv [96][96], reg pred [96][4], obj pred [96],
// cls pred [96][ncls], cls | reg conv biases [96] each.
constexpr int kHeadRp = 2 * 96 * 96, kHeadOb = kHeadRp + 96 * 4, kHeadCp = kHeadOb + 96;
__host__ __device__ constexpr int head_cb(int ncls) { return kHeadCp + 96 * ncls; }
__host__ __device__ constexpr int head_floats(int ncls) { return head_cb(ncls) + 192; }

struct StepShared {
    uint64_t bar_w[10];   // copies: layers 0-7, head (8), layer-7 qvg block (9)
    uint64_t bar_x[8];    // layer input received (layers 4-7)
    uint64_t bar_c[8];    // CTA 0: contributions received (layers 4-7)
    double ln_mean, ln_inv;
    double lnbuf[96];     // CTA 0: LayerNorm operands
    float x[96];          // layer input
    float qvg[288];       // q | v | g of this CTA's patch cell (layers 4-7)
    float qh[96];
    float res[96];        // CTA 0: residual of the current layer
    float gb[192];        // CTA 0: gamma | beta of layers 4-7, kept aside from the copies
    float con[9][96];     // CTA 0: goW contributions by patch position; head activations
    unsigned wmask;       // copy barriers the issuing thread has armed (bit i: bar_w[i])
};
static_assert(sizeof(StepShared) + sizeof(float) * kDyn <= kMaxBlockSmem, "shared memory");

// status bits: a wait for copies, for the layer input, for contributions ran out
constexpr unsigned kErrWeights = 1u, kErrInput = 2u, kErrContrib = 4u;

__device__ __forceinline__ int cl_in(int l) { return l == 4 ? 24 : l == 7 ? 96 : 48; }
__device__ __forceinline__ int cl_out(int l) { return l < 6 ? 48 : 96; }
__device__ __forceinline__ float* cl_wq(float* wsm, int l) {
    return wsm + (l == 4 ? kR4 : l == 5 ? kR5 : l == 6 ? kR6 : kR7q);
}
// goW | gamma | beta | cell row | input_proj of a layer 4-7 buffer
__device__ __forceinline__ float* cl_rest(float* wsm, int l) {
    return l == 7 ? wsm + kR7 : cl_wq(wsm, l) + cl_in(l) * 3 * cl_out(l);
}
// This CTA takes part in layer l (4-7): its cell is in bounds, or it is CTA 0
// and the layer's output is used (residual, gather, LayerNorm).
__device__ __forceinline__ bool cl_part(const Plan& P, int l, int rank) {
    return P.runs(l) && (((P.inb(l) >> rank) & 1u) || (rank == 0 && P.used(l)));
}

// ---- copies (issuer thread) -----------------------------------------------------
// The issuing thread's arrival on a copy barrier, recorded so that the CTA
// can wait for every copy it issued before it exits.
__device__ __forceinline__ void arrive_w(StepShared& sh, uint64_t* bar) {
    sh.wmask |= 1u << static_cast<unsigned>(bar - sh.bar_w);
    mbar_arrive(bar);
}

template <int IN, int OUT, int A>
__device__ void issue_small(int l, const Plan& P, const StepArgs& a, float* b, uint64_t* bar, StepShared& sh) {
    using Lo = Lay<IN, OUT, A>;
    const DevLayer& L = a.L[l];
    const int s = l / 2;
    bulk(b, L.qvgT, Lo::WQ, bar);
    if (P.used(l)) {
        bulk(b + Lo::WQ, L.goWT, Lo::WG, bar);
        bulk(b + Lo::GAM, L.gamma, OUT, bar);
        bulk(b + Lo::BET, L.beta, OUT, bar);
        if ((l & 1) == 0) bulk(b + Lo::WI, L.ipT, IN * OUT, bar);
    }
    const int Ws = a.g.W[s], Hs = a.g.H[s];
    for (int d = 0; d < A; ++d) {
        int cx, cy;
        if (patch_cell(A, d, P.px >> s, P.py >> s, Ws, Hs, cx, cy))
            bulk(b + Lo::HR + d * OUT, a.ps.hidden[l] + (static_cast<size_t>(cy) * Ws + cx) * OUT, OUT, bar);
    }
    arrive_w(sh, bar);
}

// Layer l (4-7) copies of CTA `rank`: part 1 = its qvg block, part 2 = the
// rest (goW, cell row; CTA 0 also gamma, beta, input_proj), 3 = both.
// Layer 7's qvg block completes on its own barrier.
__device__ void issue_cl(int l, int part, const Plan& P, int rank, const StepArgs& a, float* wsm,
                         StepShared& sh) {
    const int IN = cl_in(l), OUT = cl_out(l), J2 = 3 * OUT, s = l / 2;
    const bool act = (P.inb(l) >> rank) & 1u;
    const DevLayer& W = a.L[l];
    if ((part & 1) && act) {
        uint64_t* bar = l == 7 ? &sh.bar_w[9] : &sh.bar_w[l];
        bulk(cl_wq(wsm, l), W.qvgT + static_cast<size_t>(rank) * IN * J2, IN * J2, bar);
        if (l == 7) arrive_w(sh, bar);
    }
    if (part & 2) {
        uint64_t* bar = &sh.bar_w[l];
        float* r = cl_rest(wsm, l);
        if (act) {
            if (P.used(l)) bulk(r, W.goWT + static_cast<size_t>(rank) * OUT * OUT, OUT * OUT, bar);
            int cx, cy;
            patch_cell(9, rank, P.px >> s, P.py >> s, a.g.W[s], a.g.H[s], cx, cy);
            bulk(r + OUT * OUT + 2 * OUT, a.ps.hidden[l] + (static_cast<size_t>(cy) * a.g.W[s] + cx) * OUT, OUT,
                 bar);
        }
        if (rank == 0 && P.used(l)) {
            bulk(r + OUT * OUT, W.gamma, OUT, bar);
            bulk(r + OUT * OUT + OUT, W.beta, OUT, bar);
            if ((l & 1) == 0) bulk(r + OUT * OUT + 3 * OUT, W.ipT, IN * OUT, bar);
        }
        arrive_w(sh, bar);
    }
}

__device__ void issue_head(const DevHead& hd, int ncls, float* wsm, uint64_t* bar, StepShared& sh) {
    float* h = wsm + kRH;
    bulk(h, hd.cls_convT, 96 * 96, bar);
    bulk(h + 96 * 96, hd.reg_convT, 96 * 96, bar);
    bulk(h + kHeadRp, hd.reg_predT, 96 * 4, bar);
    bulk(h + kHeadOb, hd.obj_predT, 96, bar);
    bulk(h + kHeadCp, hd.cls_predT, 96 * ncls, bar);
    bulk(h + head_cb(ncls), hd.cls_conv_b, 96, bar);
    bulk(h + head_cb(ncls) + 96, hd.reg_conv_b, 96, bar);
    arrive_w(sh, bar);
}

// Copies that wait for a buffer to be consumed, issued at point p: p = 3
// when layers 0-3 are done (CTA 0) or at the start (other CTAs), p = l
// after layer l's compute.  Layer 7's qvg block needs the layer 4/5 buffers
// free, its rest and the head need the layer 6 (and 7) buffers free.
struct Deferred {
    bool q7, r7, head;
};

__device__ void issue_deferred(int p, Deferred& D, const Plan& P, int rank, const StepArgs& a, float* wsm,
                               StepShared& sh) {
    const bool u4 = cl_part(P, 4, rank), u5 = cl_part(P, 5, rank), u6 = cl_part(P, 6, rank),
               u7 = cl_part(P, 7, rank);
    if (!D.q7 && u7 && (!u4 || p >= 4) && (!u5 || p >= 5)) {
        issue_cl(7, 1, P, rank, a, wsm, sh);
        D.q7 = true;
    }
    if (!D.r7 && u7 && (!u6 || p >= 6)) {
        issue_cl(7, 2, P, rank, a, wsm, sh);
        D.r7 = true;
    }
    if (!D.head && rank == 0 && (P.flags & F_R4) && (!u6 || p >= 6) && (!u7 || p >= 7)) {
        issue_head(a.head, a.g.ncls, wsm, &sh.bar_w[8], sh);
        D.head = true;
    }
}

// ---- LayerNorm (warp 0 of CTA 0) --------------------------------------------
// y[t] = (sum over in-bounds positions d = A-1..0 of con[d][t]) + res[t];
// x = LN(y) into sh.x, also sent to the CTAs of `bmask` (layer nl's input).
// The two fp64 sums run sequentially in channel order on lane 0; the
// deviations and the normalisation are per lane (layernorm.h:41-62).
template <int OUT, int A>
__device__ void gather_ln(StepShared& sh, const float* con, int cstride, unsigned inb, const float* gam,
                          const float* bet, int nl, unsigned bmask) {
    constexpr int KP = (OUT + 31) / 32;
    const int lane = threadIdx.x;
    float yv[KP];
#pragma unroll
    for (int k = 0; k < KP; ++k) {
        const int t = lane + 32 * k;
        if (t < OUT) {
            float v = 0.0f;
#pragma unroll
            for (int d = A - 1; d >= 0; --d)
                if ((inb >> d) & 1u) v = v + con[d * cstride + t];
            yv[k] = v + sh.res[t];
            sh.lnbuf[t] = static_cast<double>(yv[k]);
        }
    }
    __syncwarp();
    if (lane == 0) {
        double sum = 0.0;
#pragma unroll
        for (int o = 0; o < OUT; ++o) sum += sh.lnbuf[o];
        sh.ln_mean = sum / static_cast<double>(OUT);
    }
    __syncwarp();
    const double mean = sh.ln_mean;
#pragma unroll
    for (int k = 0; k < KP; ++k) {
        const int t = lane + 32 * k;
        if (t < OUT) {
            const double dd = static_cast<double>(yv[k]) - mean;
            sh.lnbuf[t] = dd * dd;
        }
    }
    __syncwarp();
    if (lane == 0) {
        double var = 0.0;
#pragma unroll
        for (int o = 0; o < OUT; ++o) var += sh.lnbuf[o];
        var /= static_cast<double>(OUT);
        sh.ln_inv = 1.0 / sqrt(var + static_cast<double>(1e-5f));
    }
    __syncwarp();
    const double inv = sh.ln_inv;
#pragma unroll
    for (int k = 0; k < KP; ++k) {
        const int t = lane + 32 * k;
        if (t < OUT) {
            const double tt = (static_cast<double>(yv[k]) - mean) * inv;
            const float xv = static_cast<float>(tt * static_cast<double>(gam[t]) + static_cast<double>(bet[t]));
            sh.x[t] = xv;
            for (int r = 1; r < kStepCTAs; ++r)
                if ((bmask >> r) & 1u) send(&sh.x[t], &sh.bar_x[nl], r, xv);
        }
    }
}

// ---- layers 0-3 (CTA 0) -----------------------------------------------------------
// Every patch position: (position, column) items form q, v, sigmoid(g),
// (position, channel) items update the cells and (position, output) items
// form the goW contributions; warp 0 sums, adds the residual and
// normalises.  Returns false when the layer is the event's last.
template <int IN, int OUT, int A>
__device__ bool small_layer(int l, const Plan& P, const StepArgs& a, StepShared& sh, float* b, unsigned bmask) {
    using Lo = Lay<IN, OUT, A>;
    constexpr int J2 = Lo::J2;
    const int tid = threadIdx.x;
    const int s = l / 2, half = l % 2;
    const bool used = P.used(l);
    const int Ws = a.g.W[s], Hs = a.g.H[s], cx0 = P.px >> s, cy0 = P.py >> s;
    const float* wq = b;
    const float* wg = b + Lo::WQ;
    const float* wi = b + Lo::WI;
    const float* hr = b + Lo::HR;
    float* qvg = b + Lo::QV;
    float* qh = b + Lo::QH;
    float* con = b + Lo::CON;
    mbar_wait(&sh.bar_w[l], 0, a.err, kErrWeights);
    if (used && tid < OUT) {
        float acc;
        if (half == 0) {
            acc = 0.0f;
#pragma unroll
            for (int i = 0; i < IN; ++i) acc = fmaf(wi[i * OUT + tid], sh.x[i], acc);
        } else {
            acc = sh.x[tid];
        }
        sh.res[tid] = acc;
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
    float h = 0.0f;
    if (hact) {
        const float* q = qvg + hd * J2;
        h = fmaf(ssla_sigmoidf(q[2 * OUT + ht]), hr[hd * OUT + ht], q[OUT + ht]);
        if (used) qh[hd * OUT + ht] = q[ht] * h;
    }
    if (used) {
        __syncthreads();
        if (hact) {
            const float* w = wg + hd * OUT * OUT + ht;
            const float* q = qh + hd * OUT;
            float acc = 0.0f;
#pragma unroll
            for (int i = 0; i < OUT; ++i) acc = fmaf(w[i * OUT], q[i], acc);
            con[hd * OUT + ht] = acc;
        }
    }
    if (hact) a.ps.hidden[l][(static_cast<size_t>(hcy) * Ws + hcx) * OUT + ht] = h;
    if (!used) return false;                     // state-only second layer: the event ends
    __syncthreads();
    if (tid < 32) {
        unsigned inb = 1u;
        if (A > 1) {
            inb = 0;
            for (int d = 0; d < A; ++d) {
                int cx, cy;
                if (patch_cell(A, d, cx0, cy0, Ws, Hs, cx, cy)) inb |= 1u << d;
            }
        }
        gather_ln<OUT, A>(sh, con, OUT, inb, b + Lo::GAM, b + Lo::BET, l + 1, bmask);
    }
    __syncthreads();
    return true;
}

// ---- layers 4-7 -----------------------------------------------------------------
// One CTA's part: residual (CTA 0), q / v / sigmoid(g) of its patch cell,
// the cell's state update and its goW contribution (kept by CTA 0, sent to
// CTA 0 by the others).
template <int IN, int OUT>
__device__ void cl_layer(int l, const Plan& P, int rank, const StepArgs& a, StepShared& sh, float* wsm) {
    constexpr int J2 = 3 * OUT;
    const int tid = threadIdx.x;
    const int s = l / 2;
    const bool used = P.used(l);
    const bool act = (P.inb(l) >> rank) & 1u;
    const float* wq = cl_wq(wsm, l);
    const float* rest = cl_rest(wsm, l);
    const float* wg = rest;
    const float* hr = rest + OUT * OUT + 2 * OUT;
    const float* wi = rest + OUT * OUT + 3 * OUT;
    if (rank != 0) mbar_wait(&sh.bar_x[l], 0, a.err, kErrInput);
    mbar_wait(&sh.bar_w[l], 0, a.err, kErrWeights);
    if (l == 7 && act) mbar_wait(&sh.bar_w[9], 0, a.err, kErrWeights);
    if (rank == 0 && used && tid < OUT) {
        float acc;
        if ((l & 1) == 0) {
            acc = 0.0f;
#pragma unroll
            for (int i = 0; i < IN; ++i) acc = fmaf(wi[i * OUT + tid], sh.x[i], acc);
        } else {
            acc = sh.x[tid];
        }
        sh.res[tid] = acc;
    }
    if (rank == 0 && used && tid < 2 * OUT) sh.gb[tid] = rest[OUT * OUT + tid];
    if (act) {
        for (int col = tid + (used ? 0 : OUT); col < J2; col += kStepNT) {
            float acc = 0.0f;
            const float* w = wq + col;
#pragma unroll
            for (int i = 0; i < IN; ++i) acc = fmaf(w[i * J2], sh.x[i], acc);
            sh.qvg[col] = acc;
        }
        __syncthreads();
        float h = 0.0f;
        if (tid < OUT) {
            h = fmaf(ssla_sigmoidf(sh.qvg[2 * OUT + tid]), hr[tid], sh.qvg[OUT + tid]);
            if (used) sh.qh[tid] = sh.qvg[tid] * h;
        }
        if (used) {
            __syncthreads();
            if (tid < OUT) {
                float acc = 0.0f;
#pragma unroll
                for (int i = 0; i < OUT; ++i) acc = fmaf(wg[i * OUT + tid], sh.qh[i], acc);
                if (rank == 0) sh.con[0][tid] = acc;
                else send(&sh.con[rank][tid], &sh.bar_c[l], 0, acc);
            }
        }
        if (tid < OUT) {
            int cx, cy;
            patch_cell(9, rank, P.px >> s, P.py >> s, a.g.W[s], a.g.H[s], cx, cy);
            a.ps.hidden[l][(static_cast<size_t>(cy) * a.g.W[s] + cx) * OUT + tid] = h;
        }
    }
    __syncthreads();                   // buffers consumed; CTA 0: residual and own contribution visible
}

__device__ void run_cl(int l, const Plan& P, int rank, const StepArgs& a, StepShared& sh, float* wsm) {
    switch (l) {
        case 4: cl_layer<24, 48>(l, P, rank, a, sh, wsm); break;
        case 5: cl_layer<48, 48>(l, P, rank, a, sh, wsm); break;
        case 6: cl_layer<48, 96>(l, P, rank, a, sh, wsm); break;
        default: cl_layer<96, 96>(l, P, rank, a, sh, wsm); break;
    }
}

// CTA 0 after layer l's compute: the gathered, normalised output, sent on as
// layer l+1's input.
__device__ void cl_gather(int l, const Plan& P, const StepArgs& a, StepShared& sh, float* wsm) {
    if (threadIdx.x < 32) {
        mbar_wait(&sh.bar_c[l], 0, a.err, kErrContrib);
        const unsigned bmask = (l < 7 && P.runs(l + 1)) ? (P.inb(l + 1) & ~1u) : 0u;
        if (cl_out(l) == 48) gather_ln<48, 9>(sh, &sh.con[0][0], 96, P.inb(l), sh.gb, sh.gb + 48, l + 1, bmask);
        else gather_ln<96, 9>(sh, &sh.con[0][0], 96, P.inb(l), sh.gb, sh.gb + 96, l + 1, bmask);
    }
    __syncthreads();
}

// ---- head and commit (CTA 0) -----------------------------------------------------
// async_yolox.h:203-254: cls / reg convs with SiLU, then the 2 + 4 + 1
// predictions; decoded row written to the owned cell, raw row beside it.
__device__ void run_head(const Plan& P, const StepArgs& a, StepShared& sh, float* wsm, float pbias) {
    const int tid = threadIdx.x;
    const Geo& g = a.g;
    const PartState& ps = a.ps;
    const int ncls = g.ncls, cols = 5 + ncls;
    mbar_wait(&sh.bar_w[8], 0, a.err, kErrWeights);
    const float* h = wsm + kRH;
    float* act = &sh.con[0][0];
    if (tid < 192) {
        const int jo = tid % 96;
        const float* Wt = h + (tid < 96 ? 0 : 96 * 96) + jo;
        float acc = h[head_cb(ncls) + tid];
#pragma unroll
        for (int i = 0; i < 96; ++i) acc = fmaf(Wt[i * 96], sh.x[i], acc);
        act[tid] = acc * ssla_sigmoidf(acc);
    }
    __syncthreads();
    float v = 0.0f;
    if (tid < cols) {
        float acc = pbias;
        if (tid < 4) {
            const float* w = h + kHeadRp + tid;
#pragma unroll
            for (int i = 0; i < 96; ++i) acc = fmaf(w[i * 4], act[96 + i], acc);
        } else if (tid == 4) {
            const float* w = h + kHeadOb;
#pragma unroll
            for (int i = 0; i < 96; ++i) acc = fmaf(w[i], act[96 + i], acc);
        } else {
            const float* w = h + kHeadCp + (tid - 5);
#pragma unroll 16
            for (int i = 0; i < 96; ++i) acc = fmaf(w[i * ncls], act[i], acc);
        }
        v = acc;
    }
    const int c3x = P.px >> 3, c3y = P.py >> 3;
    const int x2 = P.px >> 2, y2 = P.py >> 2;
    const bool own = x2 >= ps.own_x0 && x2 < ps.own_x1 && y2 >= ps.own_y0 && y2 < ps.own_y1;
    const int cell = c3y * g.W[3] + c3x;
    if (tid < cols) {
        const int r = tid;
        float dv;
        if (r == 0) dv = (v + static_cast<float>(c3x)) * static_cast<float>(g.stride_w);
        else if (r == 1) dv = (v + static_cast<float>(c3y)) * static_cast<float>(g.stride_h);
        else if (r == 2) dv = ssla_expf(v) * static_cast<float>(g.stride_w);
        else if (r == 3) dv = ssla_expf(v) * static_cast<float>(g.stride_h);
        else dv = v;
        if (a.pred_out) a.pred_out[r] = dv;
        if (own) {
            ps.preds_dec[static_cast<size_t>(cell) * cols + r] = dv;
            ps.preds_raw[static_cast<size_t>(cell) * cols + r] = v;
        }
    }
    if (own && tid == 0) ps.version[cell] += 1u;
}

__global__ void __launch_bounds__(kStepNT, 1) k_step(StepArgs a) {
    __shared__ __align__(16) StepShared sh;
    extern __shared__ __align__(128) float wsm[];
    const int rank = static_cast<int>(cta_rank());
    const int tid = threadIdx.x;
    const PartState& ps = a.ps;
    const Geo& g = a.g;
    const bool hyb = g.layout == LAYOUT_HYBRID;

    // ---- gate inputs (every CTA), preprocess inputs and head biases (CTA 0) ----
    const float4 e = a.ev;
    const bool valid = e.y > -1.0f && e.y < static_cast<float>(g.W[0]) && e.z > -1.0f &&
                       e.z < static_cast<float>(g.H[0]);
    const int px = valid ? static_cast<int>(e.y) : 0, py = valid ? static_cast<int>(e.z) : 0;
    int k[4];
    gate_cells(g, px, py, k);
    int c[4] = {0, 0, 0, 0};
    if (valid) {
        c[0] = ps.cnt[0][k[0]];
        c[1] = ps.cnt[1][k[1]];
        c[2] = ps.cnt[2][k[2]];
        if (hyb) c[3] = ps.cnt[3][k[3]];
    }
    double lt_prev = 0.0;
    if (rank == 0 && tid == 0 && valid) lt_prev = ps.last_t[py * g.W[0] + px];
    float pbias = 0.0f;
    if (rank == 0 && tid < 5 + g.ncls)
        pbias = tid < 4 ? __ldg(a.head.reg_pred_b + tid)
                        : tid == 4 ? __ldg(a.head.obj_pred_b) : __ldg(a.head.cls_pred_b + (tid - 5));
    const int flags = gate_flags(valid, c, g.window, hyb);
    Plan P;
    make_plan(P, flags, px, py, g);

    // ---- barriers, expected messages, first copies ----
    if (tid == 0) {
        for (int i = 0; i < 10; ++i) mbar_init(&sh.bar_w[i], 1);
        sh.wmask = 0u;
        for (int i = 0; i < 8; ++i) {
            mbar_init(&sh.bar_x[i], 1);
            mbar_init(&sh.bar_c[i], 1);
        }
        fence_mbar_init();
        for (int l = 4; l < 8; ++l) {
            if (rank != 0 && P.runs(l) && ((P.inb(l) >> rank) & 1u)) mbar_arrive_tx(&sh.bar_x[l], 4u * cl_in(l));
            if (rank == 0 && P.used(l))
                mbar_arrive_tx(&sh.bar_c[l], 4u * cl_out(l) * __popc(P.inb(l) & ~1u));
        }
    }
    __syncthreads();
    Deferred D{false, false, false};
    if (tid == kIssuer) {
        if (rank == 0) {
            if (P.runs(0)) issue_small<2, 12, 1>(0, P, a, wsm, &sh.bar_w[0], sh);
            if (P.runs(1)) issue_small<12, 12, 9>(1, P, a, wsm + kS1, &sh.bar_w[1], sh);
            if (P.runs(2)) issue_small<12, 24, 9>(2, P, a, wsm + kS2, &sh.bar_w[2], sh);
            if (P.runs(3)) issue_small<24, 24, 9>(3, P, a, wsm + kS3, &sh.bar_w[3], sh);
            if (cl_part(P, 4, 0)) issue_cl(4, 3, P, 0, a, wsm, sh);
        } else {
            for (int l = 4; l < 7; ++l)
                if (cl_part(P, l, rank)) issue_cl(l, 3, P, rank, a, wsm, sh);
            issue_deferred(3, D, P, rank, a, wsm, sh);
        }
    }
    cluster_arrive();                  // every CTA has read the counters and set up its barriers

    if (rank == 0) {
        if (valid) {
            if (tid == 0) {
                sh.x[0] = dt_norm(lt_prev, e.x);
                sh.x[1] = e.w;
            }
            __syncthreads();
            small_layer<2, 12, 1>(0, P, a, sh, wsm, 0u);
        }
        cluster_wait();
        if (valid && tid == 0) {       // the counters may change now that every CTA has read them
            ps.last_t[py * g.W[0] + px] = static_cast<double>(e.x);
            ps.cnt[0][k[0]] = static_cast<uint8_t>(c[0] + 1);
            if (flags & F_R1) ps.cnt[1][k[1]] = static_cast<uint8_t>(c[1] + 1);
            if (flags & F_R2) ps.cnt[2][k[2]] = static_cast<uint8_t>(c[2] + 1);
            if (hyb && (flags & F_R3)) ps.cnt[3][k[3]] = static_cast<uint8_t>(c[3] + 1);
        }
        if (P.runs(1) && small_layer<12, 12, 9>(1, P, a, sh, wsm + kS1, 0u) &&
            small_layer<12, 24, 9>(2, P, a, sh, wsm + kS2, 0u)) {
            const unsigned b4 = P.runs(4) ? (P.inb(4) & ~1u) : 0u;
            if (small_layer<24, 24, 9>(3, P, a, sh, wsm + kS3, b4) && tid == kIssuer) {
                // layers 0-3 are done: their buffers take layers 5 and 6
                for (int l = 5; l < 7; ++l)
                    if (cl_part(P, l, 0)) issue_cl(l, 3, P, 0, a, wsm, sh);
                issue_deferred(3, D, P, 0, a, wsm, sh);
            }
        }
    } else {
        cluster_wait();
    }

    // ---- layers 4-7 ----
    for (int l = 4; l < 8; ++l) {
        if (!P.runs(l)) break;
        if (cl_part(P, l, rank)) run_cl(l, P, rank, a, sh, wsm);
        if (tid == kIssuer) issue_deferred(l, D, P, rank, a, wsm, sh);
        if (!P.used(l)) break;         // state-only second layer: the event ends here
        if (rank == 0) cl_gather(l, P, a, sh, wsm);
    }

    if (rank == 0) {
        if (P.flags & F_R4) run_head(P, a, sh, wsm, pbias);
        if (tid == 0 && a.flag_out) *a.flag_out = static_cast<uint8_t>(flags);
    }

    // ---- exit: no copy of this CTA still writing its shared memory (bounded
    // waits: a copy whose wait ran out above may still be in flight), and no
    // CTA leaves while a peer could still send into it ----
    __syncthreads();
    if (tid == 0)
        for (int i = 0; i < 10; ++i)
            if ((sh.wmask >> i) & 1u) mbar_wait(&sh.bar_w[i], 0, nullptr, 0u);
    __syncthreads();
    cluster_arrive();
    cluster_wait();
}

}  // namespace

cudaError_t launch_step(cudaStream_t st, const StepArgs& a) {
    constexpr size_t smem = sizeof(float) * kDyn;
    if (head_floats(a.g.ncls) > kDyn) return cudaErrorInvalidValue;
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
