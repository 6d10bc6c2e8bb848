// ssla_device.cuh -- device-side types and math shared by the engine kernels.
//
// Engine model (one drain call = one "chunk" of events for P independent
// partitions):
//   - gates are integer-only, so every temporal-dropout decision of the chunk
//     is computed up front (k_gates) and the events entering each stage are
//     compacted in stream order into E_s lists (k_compact_*);
//   - every layer is then run layer-synchronously over the whole chunk:
//       k_scan   -- one warp per grid cell walks, in stream order, the events
//                   whose 3x3 patch covers the cell and applies the LRU update
//                   h = sigmoid(g)*h + v (the cell-owner invariant of
//                   ssla_s2_s3_head_celled.cuh:1-38 taken to its limit: one
//                   owner per cell, no atomics, exact per-cell order);
//       k_event  -- per event (batched 32 per CTA): the 9-owner gather
//                   sum_delta goW[delta]*(q*h_new) in the reference patch
//                   order, residual, fp64 LayerNorm, then the next layer's
//                   fused qvg matvec for all patch positions (or the head).
// Arithmetic follows the oracle contract exactly (fmaf chains in reference
// loop order, no other contraction -- the build uses -fmad=false --,
// sequential fp64 LayerNorm sums, ssla_expf below), so results are
// bit-identical to oracle/ssla_oracle.c.
#pragma once

#include <cstdint>

namespace ssla {

constexpr int kNT = 256;            // threads per CTA (event / filter kernels)
constexpr int kMB = 32;             // events per k_event batch
constexpr int kEPT = 8;             // events per thread in k_event tiles
constexpr int kGroups = kMB / kEPT; // event groups per batch
constexpr int kTile = 8;            // tile side (cells) of tile lists
constexpr int kMaxTileCols = 64;    // tiles per row (stage-0 width <= 512)
constexpr int kMaxParts = 1024;
constexpr uint32_t kInvalidXY = 0xFFFFFFFFu;
constexpr int kCompactTile = 4096;  // events per compaction tile at most (512 at least)

enum : uint8_t { F_VALID = 1, F_R1 = 2, F_R2 = 4, F_R3 = 8, F_R4 = 16, F_FOREIGN = 32 };
enum { LAYOUT_DECOMP = 0, LAYOUT_HYBRID = 1 };

__host__ __device__ constexpr int chans(int s) { return s == 0 ? 12 : s == 1 ? 24 : s == 2 ? 48 : 96; }

struct DevLayer {
    const float* qvgT;   // [A][IN][3*OUT]
    const float* goWT;   // [A][OUT][OUT]  ([p][i][o])
    const float* ipT;    // [IN][OUT] or null
    const float* gamma;  // [OUT]
    const float* beta;   // [OUT]
};

struct DevHead {
    const float *cls_convT, *cls_conv_b, *reg_convT, *reg_conv_b;  // [96][96], [96]
    const float *cls_predT, *cls_pred_b;                            // [96][ncls]
    const float *reg_predT, *reg_pred_b;                            // [96][4]
    const float *obj_predT, *obj_pred_b;                            // [96][1]
    // drains only: non-null selects the tensor-core head (k_head_tc), whose
    // [cls_conv | reg_conv] rows [192][96] these are (TF32 hi terms, then lo)
    const float* tc_w1;
    unsigned* tc_err;                                               // its status bits (host-mapped)
};

// Per-partition state pointers (device memory).
struct PartState {
    float* hidden[8];    // [Hs*Ws][C_s]
    uint8_t* cnt[4];     // gate counters, grid of gate g per layout
    double* last_t;      // [H*W]
    float* preds_dec;    // [H3*W3][5+ncls]
    float* preds_raw;    // [H3*W3][5+ncls]
    uint32_t* version;   // [H3*W3]
    int own_x0, own_x1, own_y0, own_y1;  // owned range, s2 coordinates
};

struct Geo {
    int H[4], W[4];      // grid per stage
    int P;               // partitions
    int layout;
    int window;
    int ncls;
    int stride_h, stride_w;
    int tx[4], ty[4];    // tiles per stage (x, y)
    int seg;             // tile-list segment length
    int nseg[4];         // allocated segments per (partition, tile) per stage
    int cap[5];          // allocated entries of each stage list (E_0 = events)
    int row_lo[4], row_hi[4];   // rows of each stage's grid the scans update (strips: own rows + 1)
};

struct StageEntry {      // one event in a stage list E_s, stream order
    int e;               // chunk-global event / record index
    int kprev;           // index in E_{s-1} (E_0 index == e)
    uint32_t xy0;        // pixel coords x | y << 16
};

__device__ __forceinline__ int gate_grid(int layout, int g) {
    return g == 0 ? 1 : g == 1 ? 2 : g == 2 ? (layout == LAYOUT_HYBRID ? 2 : 3) : 3;
}

// Twin of or_expf (oracle/ssla_oracle.c): Cody-Waite reduction with ln2 split
// into a 12-bit head and a float tail, degree-7 Taylor polynomial by Horner
// with fmaf, exact power-of-two scaling.  IEEE basic operations only, so
// host and device results are identical; accuracy is tested against
// CUDA's expf and libm.
__host__ __device__ __forceinline__ float ssla_pow2i(int e) {
#ifdef __CUDA_ARCH__
    return __int_as_float((e + 127) << 23);
#else
    union { uint32_t u; float f; } b;
    b.u = static_cast<uint32_t>(e + 127) << 23;
    return b.f;
#endif
}

__host__ __device__ __forceinline__ float ssla_expf(float x) {
    if (x != x) return x;
    if (x > 88.8f) return __builtin_huge_valf();
    if (x < -104.0f) return 0.0f;
    // nearest integer, ties to even, without a conversion instruction
    // (1.5 * 2^23 trick; |x * log2e| < 2^22 after the range checks)
    const float big = x * 1.44269502f + 12582912.0f;
    const float n = big - 12582912.0f;
    float r = fmaf(-n, 0.693115234375f, x);
    r = fmaf(-n, 3.19461833e-05f, r);
    float p = 1.98412701e-04f;
    p = fmaf(p, r, 1.38888892e-03f);
    p = fmaf(p, r, 8.33333377e-03f);
    p = fmaf(p, r, 4.16666679e-02f);
    p = fmaf(p, r, 1.66666672e-01f);
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
#ifdef __CUDA_ARCH__
    const int ni = __float_as_int(big) - 0x4B400000;
#else
    union { float f; int32_t i; } bb;
    bb.f = big;
    const int ni = bb.i - 0x4B400000;
#endif
    const int n1 = ni / 2;
    const int n2 = ni - n1;
    return (p * ssla_pow2i(n1)) * ssla_pow2i(n2);
}

// 1 / y rounded to nearest for y in [1, 2^126): the hardware approximation
// (rcp.approx, within an ulp) refined by one Newton-Raphson step with fused
// multiply-adds, e = 1 - y q exactly, q' = q + q e (P. Markstein, "Computation
// of elementary functions on the IBM RISC System/6000 processor", IBM J. Res.
// Dev. 34(1), 1990).  Equal to IEEE round-to-nearest division for every
// float in that range (checked exhaustively, ssla_selftest_reciprocal), with
// no branch, so the sigmoids of a thread interleave.
__device__ __forceinline__ float ssla_rcp_rn(float y) {
    float q;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(q) : "f"(y));
    return fmaf(q, fmaf(-y, q, 1.0f), q);
}

// vendor/openeva/prim/activation.h:17, 1 / (1 + exp(-x)), with an exp of
// its own for the range the sigmoid needs: t = -x clamped to [-17, 87]
// (for x >= 17 the result is exactly 1, as 1 + exp(-17) rounds to 1; for
// x <= -87 it is 1 / (1 + e^87) ~ 1.6e-38, the smallest normal result,
// instead of a smaller value).
// n = nearest integer to t * log2(e) (1.5 * 2^23 trick), r = t - n ln 2 by
// Cody-Waite with ln 2 split into a 12-bit head and a float tail, exp(r)
// by a degree-6 minimax polynomial on [-ln2/2, ln2/2] (Remez exchange,
// coefficients rounded to float, 0.87 ulp), Horner with fused
// multiply-adds, then one exact scaling by 2^n (n in [-25, 126]).  IEEE
// basic operations only, identical on host and device; the reciprocal of
// 1 + e^t (in [1, 2^126)) is rounded to nearest (ssla_rcp_rn on the device,
// exactly 1.0f / y on the host).  Within 2.3 ulp of the exact sigmoid for
// x >= -87, as the general exp route was.
__host__ __device__ __forceinline__ float ssla_sigmoidf(float x) {
    if (x != x) return x;
    const float t = fminf(fmaxf(-x, -17.0f), 87.0f);
    const float big = fmaf(t, 1.44269502f, 12582912.0f);
    const float n = big - 12582912.0f;
    float r = fmaf(-n, 0.693115234375f, t);
    r = fmaf(-n, 3.19461833e-05f, r);
    float p = 1.38368458e-03f;
    p = fmaf(p, r, 8.37481581e-03f);
    p = fmaf(p, r, 4.16682251e-02f);
    p = fmaf(p, r, 1.66664198e-01f);
    p = fmaf(p, r, 4.99999911e-01f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
#ifdef __CUDA_ARCH__
    const int ni = __float_as_int(big) - 0x4B400000;
    return ssla_rcp_rn(1.0f + p * ssla_pow2i(ni));
#else
    union { float f; int32_t i; } bb;
    bb.f = big;
    const int ni = bb.i - 0x4B400000;
    return 1.0f / (1.0f + p * ssla_pow2i(ni));
#endif
}

#ifdef __CUDACC__
// Two ssla_sigmoidf evaluations with packed FP32 operations: every component
// of __ffma2_rn / __fadd2_rn / __fmul2_rn is one IEEE fmaf / fadd / fmul
// rounded to nearest, the operations of ssla_sigmoidf in the same order, so
// the results are bit-identical to two scalar calls (checked over every
// float pair component by ssla_selftest_sigmoid_pair).  fmaf(-n, c, r) is
// written fmaf(n, -c, r), the same product.  The scale 2^n comes from the
// bits of big = 1.5 * 2^23 + n, which are 0x4B400000 + n: shifted left by
// 23 the constant part leaves 32 bits, so (bits << 23) + (127 << 23) is
// (n + 127) << 23 modulo 2^32, one integer multiply-add per component.
__device__ __forceinline__ float2 ssla_sigmoidf2(float2 x) {
    const float2 t = make_float2(fminf(fmaxf(-x.x, -17.0f), 87.0f), fminf(fmaxf(-x.y, -17.0f), 87.0f));
    const float2 big = __ffma2_rn(t, make_float2(1.44269502f, 1.44269502f),
                                  make_float2(12582912.0f, 12582912.0f));
    const float2 n = __fadd2_rn(big, make_float2(-12582912.0f, -12582912.0f));
    float2 r = __ffma2_rn(n, make_float2(-0.693115234375f, -0.693115234375f), t);
    r = __ffma2_rn(n, make_float2(-3.19461833e-05f, -3.19461833e-05f), r);
    float2 p = __ffma2_rn(make_float2(1.38368458e-03f, 1.38368458e-03f), r,
                          make_float2(8.37481581e-03f, 8.37481581e-03f));
    p = __ffma2_rn(p, r, make_float2(4.16682251e-02f, 4.16682251e-02f));
    p = __ffma2_rn(p, r, make_float2(1.66664198e-01f, 1.66664198e-01f));
    p = __ffma2_rn(p, r, make_float2(4.99999911e-01f, 4.99999911e-01f));
    p = __ffma2_rn(p, r, make_float2(1.0f, 1.0f));
    p = __ffma2_rn(p, r, make_float2(1.0f, 1.0f));
    const float2 s = make_float2(__uint_as_float((__float_as_uint(big.x) << 23) + 0x3F800000u),
                                 __uint_as_float((__float_as_uint(big.y) << 23) + 0x3F800000u));
    const float2 y = __fadd2_rn(make_float2(1.0f, 1.0f), __fmul2_rn(p, s));
    float qx, qy;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(qx) : "f"(y.x));
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(qy) : "f"(y.y));
    const float2 q = make_float2(qx, qy);
    const float2 e = __ffma2_rn(make_float2(-y.x, -y.y), q, make_float2(1.0f, 1.0f));
    float2 out = __ffma2_rn(q, e, q);
    if (x.x != x.x) out.x = x.x;
    if (x.y != x.y) out.y = x.y;
    return out;
}
#endif

}  // namespace ssla
