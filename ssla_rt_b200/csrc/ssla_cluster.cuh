// ssla_cluster.cuh -- thread-block-cluster plumbing shared by the single-event
// kernels (k_step, k_live): mbarriers, bulk copies into shared memory,
// st.async messages into a peer CTA's shared memory, cluster barriers, and
// the patch / gate helpers of one event.
#pragma once

#include <cstdint>

#include "ssla_device.cuh"

namespace ssla {
namespace cl {

constexpr int kMaxBlockSmem = 232448;                              // 227 KB per CTA on sm_100
constexpr unsigned long long kWaitNs = 20ull * 1000ull * 1000ull;  // bound of a message / copy wait (20 ms)

__device__ __forceinline__ uint32_t su32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint32_t cta_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ unsigned long long gtime() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ---- mbarriers ---------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(bar)) : "memory");
}
// Arrival that also raises the phase's expected byte count.
__device__ __forceinline__ void mbar_arrive_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(bar)), "r"(bytes) : "memory");
}
// Arrival on the barrier at the same address in CTA `rank` (release at
// cluster scope: this CTA's earlier writes are visible to whoever acquires).
__device__ __forceinline__ void mbar_arrive_remote(const uint64_t* bar, int rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(su32(bar)), "r"(rank));
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(r) : "memory");
}
// The same without ordering this CTA's earlier writes (an acknowledgement
// that inputs have been read; it does not wait for outstanding stores).
__device__ __forceinline__ void mbar_arrive_remote_relaxed(const uint64_t* bar, int rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(su32(bar)), "r"(rank));
    asm volatile("mbarrier.arrive.relaxed.cluster.shared::cluster.b64 _, [%0];" ::"r"(r) : "memory");
}
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n"
        " mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(su32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Waits for the phase of `bar` with the given parity, at most `limit_ns`;
// returns false (and ORs `code` into *err when err is set) if it ran out.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned* err, unsigned code,
                                          unsigned long long limit_ns = kWaitNs) {
    if (mbar_test(bar, parity)) return true;
    const unsigned long long t0 = gtime();
    while (!mbar_test(bar, parity)) {
        if (gtime() - t0 > limit_ns) {
            if (err) atomicOr_system(err, code);
            return false;
        }
    }
    return true;
}

// ---- copies and messages --------------------------------------------------------
// n floats global -> this CTA's shared memory (n % 4 == 0, both addresses
// 16-byte aligned), completing on `bar`; the issuing thread also raises the
// barrier's expected byte count.
__device__ __forceinline__ void bulk(float* dst, const float* src, int n, uint64_t* bar) {
    const uint32_t bytes = static_cast<uint32_t>(n) * 4u;
    asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(su32(bar)), "r"(bytes) : "memory");
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(su32(dst)),
        "l"(src), "r"(bytes), "r"(su32(bar))
        : "memory");
}
__device__ __forceinline__ uint32_t peer(uint32_t addr, int rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}
// One 32-bit word into CTA `rank`'s shared memory at the address of `dst` in
// this CTA, completing 4 bytes on that CTA's barrier at the address of `bar`.
__device__ __forceinline__ void send(const void* dst, const uint64_t* bar, int rank, float v) {
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];" ::"r"(
                     peer(su32(dst), rank)),
                 "r"(__float_as_uint(v)), "r"(peer(su32(bar), rank))
                 : "memory");
}
// Four words (16-byte aligned) in one message.
__device__ __forceinline__ void send4(const void* dst, const uint64_t* bar, int rank, float4 v) {
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.b32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(
                     peer(su32(dst), rank)),
                 "r"(__float_as_uint(v.x)), "r"(__float_as_uint(v.y)), "r"(__float_as_uint(v.z)),
                 "r"(__float_as_uint(v.w)), "r"(peer(su32(bar), rank))
                 : "memory");
}
__device__ __forceinline__ void cluster_arrive() {
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// ---- one event's patch and gates ------------------------------------------------------
__device__ __forceinline__ bool step_gate(int pre, int window) {
    return window <= 1 || ((pre & 255) % window) == 0;
}

// The patch cell of position d at stage s around (cx0, cy0); A == 1 is the
// event's own cell.  delta = (1-dy)*3 + (1-dx), the reference's numbering.
__device__ __forceinline__ bool patch_cell(int A, int d, int cx0, int cy0, int Ws, int Hs, int& cx, int& cy) {
    if (A == 1) { cx = cx0; cy = cy0; return true; }
    cx = cx0 + 1 - d % 3;
    cy = cy0 + 1 - d / 3;
    return cx >= 0 && cx < Ws && cy >= 0 && cy < Hs;
}

// What the event does, as register bitmasks.
struct Plan {
    int flags, px, py;
    unsigned runs_m;            // bit l: layer l runs (its stage is reached)
    unsigned used_m;            // bit l: its output is consumed (else state-only: the event ends there)
    unsigned long long inb_m;   // 9 bits per stage: patch position d's cell is in bounds
    __device__ __forceinline__ bool runs(int l) const { return (runs_m >> l) & 1u; }
    __device__ __forceinline__ bool used(int l) const { return (used_m >> l) & 1u; }
    __device__ __forceinline__ unsigned inb(int l) const {
        return static_cast<unsigned>(inb_m >> (9 * (l >> 1))) & 0x1FFu;
    }
};

// Positions d = (1-dy)*3 + (1-dx): column d%3 = 0, 1, 2 is dx = +1, 0, -1,
// row d/3 likewise for dy.
__device__ __forceinline__ unsigned patch_mask(int cx0, int cy0, int Ws, int Hs) {
    const unsigned cols = (cx0 + 1 < Ws ? 1u : 0u) | 2u | (cx0 >= 1 ? 4u : 0u);
    return (cy0 + 1 < Hs ? cols : 0u) | (cols << 3) | (cy0 >= 1 ? cols << 6 : 0u);
}

__device__ __forceinline__ void make_plan(Plan& P, int flags, int px, int py, const Geo& g) {
    P.flags = flags;
    P.px = px;
    P.py = py;
    unsigned runs = 0, used = 0;
    if (flags & F_VALID) {
        runs = 0x3u;                                   // stage 0
        if (flags & F_R1) runs |= 0xCu;
        if (flags & F_R2) runs |= 0x30u;
        if (flags & F_R3) runs |= 0xC0u;
        // first layers of reached stages; second layers when the next stage (head) is reached
        used = runs & 0x55u;
        if (flags & F_R1) used |= 0x2u;
        if (flags & F_R2) used |= 0x8u;
        if (flags & F_R3) used |= 0x20u;
        if (flags & F_R4) used |= 0x80u;
    }
    P.runs_m = runs;
    P.used_m = used;
    unsigned long long m = 0;
#pragma unroll
    for (int s = 0; s < 4; ++s)
        m |= static_cast<unsigned long long>(patch_mask(px >> s, py >> s, g.W[s], g.H[s])) << (9 * s);
    P.inb_m = m;
}

// Preprocess input and the four gate decisions in gate order from the
// counters' values before the event (src/ssla_kernels.cpp:288-309,
// :903-921; ssla_s2_s3_head_celled.cuh:719-747 for the HYBRID s3 gate).
__device__ __forceinline__ int gate_flags(bool valid, const int c[4], int window, bool hyb) {
    if (!valid) return 0;
    int flags = F_VALID;
    if (step_gate(c[0], window)) {
        flags |= F_R1;
        if (step_gate(c[1], window)) {
            flags |= F_R2;
            if (step_gate(c[2], window)) {
                flags |= F_R3;
                if (!hyb || step_gate(c[3], window)) flags |= F_R4;
            }
        }
    }
    return flags;
}

// Counter cells of the four gates for pixel (px, py).
__device__ __forceinline__ void gate_cells(const Geo& g, int px, int py, int k[4]) {
    const bool hyb = g.layout == LAYOUT_HYBRID;
    k[0] = (py >> 1) * g.W[1] + (px >> 1);
    k[1] = (py >> 2) * g.W[2] + (px >> 2);
    k[3] = (py >> 3) * g.W[3] + (px >> 3);
    k[2] = hyb ? k[1] : k[3];
}

__device__ __forceinline__ float dt_norm(double prev, float t) {
    if (prev < 0.0) return 1.0f;
    double v = (static_cast<double>(t) - prev) / 1e5;
    if (v < 0.0) v = 0.0;
    if (v > 1.0) v = 1.0;
    return static_cast<float>(v);
}

// ---- arithmetic of one event -----------------------------------------------------
// Four adjacent output columns c..c+3 of x . W (W row-major, row stride ld,
// w = &W[0][c]): acc.j = fmaf(W[i][c+j], x[i], acc.j) for i = 0..N-1 in
// order -- four independent chains, each exactly matvec_ct's
// (linear.h:80-90); weights and inputs are read as float4 (x, w 16-byte
// aligned, ld % 4 == 0).
template <int N>
__device__ __forceinline__ float4 dot4(const float* w, int ld, const float* x, float4 acc) {
#pragma unroll
    for (int i = 0; i + 4 <= N; i += 4) {
        const float4 xv = *reinterpret_cast<const float4*>(x + i);
        const float4 a = *reinterpret_cast<const float4*>(w + (i + 0) * ld);
        const float4 b = *reinterpret_cast<const float4*>(w + (i + 1) * ld);
        const float4 c = *reinterpret_cast<const float4*>(w + (i + 2) * ld);
        const float4 d = *reinterpret_cast<const float4*>(w + (i + 3) * ld);
        acc.x = fmaf(a.x, xv.x, acc.x); acc.y = fmaf(a.y, xv.x, acc.y);
        acc.z = fmaf(a.z, xv.x, acc.z); acc.w = fmaf(a.w, xv.x, acc.w);
        acc.x = fmaf(b.x, xv.y, acc.x); acc.y = fmaf(b.y, xv.y, acc.y);
        acc.z = fmaf(b.z, xv.y, acc.z); acc.w = fmaf(b.w, xv.y, acc.w);
        acc.x = fmaf(c.x, xv.z, acc.x); acc.y = fmaf(c.y, xv.z, acc.y);
        acc.z = fmaf(c.z, xv.z, acc.z); acc.w = fmaf(c.w, xv.z, acc.w);
        acc.x = fmaf(d.x, xv.w, acc.x); acc.y = fmaf(d.y, xv.w, acc.y);
        acc.z = fmaf(d.z, xv.w, acc.z); acc.w = fmaf(d.w, xv.w, acc.w);
    }
#pragma unroll
    for (int i = N & ~3; i < N; ++i) {
        const float xv = x[i];
        const float4 a = *reinterpret_cast<const float4*>(w + i * ld);
        acc.x = fmaf(a.x, xv, acc.x); acc.y = fmaf(a.y, xv, acc.y);
        acc.z = fmaf(a.z, xv, acc.z); acc.w = fmaf(a.w, xv, acc.w);
    }
    return acc;
}
// One column with row stride ld: acc = fmaf(w[i*ld], x[i], acc), i in order.
template <int N>
__device__ __forceinline__ float dot1(const float* w, int ld, const float* x, float acc) {
#pragma unroll
    for (int i = 0; i < N; i += 4) {
        const float4 xv = *reinterpret_cast<const float4*>(x + i);
        const float a = w[(i + 0) * ld], b = w[(i + 1) * ld], c = w[(i + 2) * ld], d = w[(i + 3) * ld];
        acc = fmaf(a, xv.x, acc);
        acc = fmaf(b, xv.y, acc);
        acc = fmaf(c, xv.z, acc);
        acc = fmaf(d, xv.w, acc);
    }
    return acc;
}

__host__ __device__ constexpr int ceil_log2(int v) { return v <= 1 ? 0 : 1 + ceil_log2((v + 1) / 2); }

// LayerNorm over OUT channels held by one warp, lane g holding channels
// 4g..4g+3 (lanes g >= OUT/4 hold nothing); returns the normalised values
// of the lane's channels (layernorm.h:41-62, with the reference's fp64
// arithmetic and summation order):
//   mean = (sum_o y_o) / OUT -- the sum in channel order, or as a tree when
//     the values' exponents prove every partial sum exact (then every order
//     gives the same double);
//   var  = (sum_o (y_o - mean)^2) / OUT, summed in channel order;
//   x_o  = float(((y_o - mean) * inv) * gamma_o + beta_o), inv = 1/sqrt(var + eps).
template <int OUT>
__device__ __forceinline__ float4 ln4(float4 y, const float* gam, const float* bet) {
    constexpr int G = OUT / 4;
    constexpr unsigned kAll = 0xFFFFFFFFu;
    const int lane = threadIdx.x & 31;
    const bool act = lane < G;
    unsigned emax = 0, emin = 255;
    if (act) {
        const float v[4] = {y.x, y.y, y.z, y.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const unsigned u = __float_as_uint(v[j]);
            if (u & 0x7FFFFFFFu) {
                unsigned e = (u >> 23) & 0xFFu;
                e = e < 1u ? 1u : e;                 // subnormals: the ulp of exponent 1
                emax = e > emax ? e : emax;
                emin = e < emin ? e : emin;
            }
        }
    }
    emax = __reduce_max_sync(kAll, emax);
    emin = __reduce_min_sync(kAll, emin);
    double mean;
    if (emax == 0 || (emax < 255u && static_cast<int>(emax - emin) + ceil_log2(OUT) <= 29)) {
        // |partial sums| < 2^53 * (smallest ulp): every addition is exact
        double s = act ? (static_cast<double>(y.x) + static_cast<double>(y.y)) +
                             (static_cast<double>(y.z) + static_cast<double>(y.w))
                       : 0.0;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(kAll, s, off);
        mean = s / static_cast<double>(OUT);
    } else {
        double s = 0.0;
#pragma unroll
        for (int g = 0; g < G; ++g) {
            s += static_cast<double>(__shfl_sync(kAll, y.x, g));
            s += static_cast<double>(__shfl_sync(kAll, y.y, g));
            s += static_cast<double>(__shfl_sync(kAll, y.z, g));
            s += static_cast<double>(__shfl_sync(kAll, y.w, g));
        }
        mean = s / static_cast<double>(OUT);
    }
    const double d0 = static_cast<double>(y.x) - mean, d1 = static_cast<double>(y.y) - mean;
    const double d2 = static_cast<double>(y.z) - mean, d3 = static_cast<double>(y.w) - mean;
    const double q0 = d0 * d0, q1 = d1 * d1, q2 = d2 * d2, q3 = d3 * d3;
    double var = 0.0;
#pragma unroll
    for (int g = 0; g < G; ++g) {
        var += __shfl_sync(kAll, q0, g);
        var += __shfl_sync(kAll, q1, g);
        var += __shfl_sync(kAll, q2, g);
        var += __shfl_sync(kAll, q3, g);
    }
    var /= static_cast<double>(OUT);
    const double inv = 1.0 / sqrt(var + static_cast<double>(1e-5f));
    float4 x = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    if (act) {
        const float4 g4 = *reinterpret_cast<const float4*>(gam + 4 * lane);
        const float4 b4 = *reinterpret_cast<const float4*>(bet + 4 * lane);
        x.x = static_cast<float>((d0 * inv) * static_cast<double>(g4.x) + static_cast<double>(b4.x));
        x.y = static_cast<float>((d1 * inv) * static_cast<double>(g4.y) + static_cast<double>(b4.y));
        x.z = static_cast<float>((d2 * inv) * static_cast<double>(g4.z) + static_cast<double>(b4.z));
        x.w = static_cast<float>((d3 * inv) * static_cast<double>(g4.w) + static_cast<double>(b4.w));
    }
    return x;
}

}  // namespace cl
}  // namespace ssla
