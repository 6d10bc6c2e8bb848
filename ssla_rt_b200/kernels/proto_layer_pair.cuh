// proto_layer_pair.cuh -- exact-arithmetic device primitives of the B200
// stage-2/3 ring consumer (ssla_s2_s3_head_celled.cuh beside it).
//
// The reference's runners NVRTC-compile their kernel module from two files
// read by name from one directory, ssla_s2_s3_head_celled.cuh and this
// header (orin/bench_s2_s3_head_celled.py:195-200,
// orin/hybrid_runner_multi.py:465-473), so the replacement module keeps the
// two names.  Self-contained and NVRTC-safe: no standard headers and no
// instruction newer than sm_80, so it compiles for whatever
// --gpu-architecture the runner passes (compute_87 by default, compute_100a
// for a B200 build) and loads on a B200 either way.
//
// Every operation is written as the IEEE intrinsic it has to be --
// __fmaf_rn for the fused multiply-adds of the reference's dot products and
// LRU update, __fmul_rn / __fadd_rn / __dadd_rn / __dmul_rn / __ddiv_rn /
// __dsqrt_rn elsewhere -- so neither contraction nor the runners'
// --use_fast_math changes a result: the kernels reproduce the CPU oracle's
// arithmetic (fmaf chains in the reference's loop order, fp64 LayerNorm
// sums in channel order, the portable exp below), except that
// --use_fast_math flushes single-precision subnormals to zero.
#pragma once

namespace sslab {

constexpr unsigned kFull = 0xFFFFFFFFu;

__device__ __forceinline__ unsigned lanemask_lt() {
    unsigned m;
    asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
    return m;
}

// 2^e for e in the normal exponent range.
__device__ __forceinline__ float pow2i(int e) { return __int_as_float((e + 127) << 23); }

// exp(x): Cody-Waite argument reduction (W. J. Cody and W. Waite, Software
// Manual for the Elementary Functions, 1980) with ln 2 split into a 12-bit
// head and a float tail, a degree-7 Taylor polynomial (1/k! rounded to
// float) by Horner with fused multiply-adds, and exact power-of-two
// scaling -- the engine's and the oracle's exp, operation for operation.
__device__ __forceinline__ float exp_portable(float x) {
    if (x != x) return x;
    if (x > 88.8f) return __int_as_float(0x7F800000);
    if (x < -104.0f) return 0.0f;
    // nearest integer of x * log2(e), ties to even (1.5 * 2^23 trick)
    const float big = __fadd_rn(__fmul_rn(x, 1.44269502f), 12582912.0f);
    const float n = __fsub_rn(big, 12582912.0f);
    float r = __fmaf_rn(-n, 0.693115234375f, x);
    r = __fmaf_rn(-n, 3.19461833e-05f, r);
    float p = 1.98412701e-04f;
    p = __fmaf_rn(p, r, 1.38888892e-03f);
    p = __fmaf_rn(p, r, 8.33333377e-03f);
    p = __fmaf_rn(p, r, 4.16666679e-02f);
    p = __fmaf_rn(p, r, 1.66666672e-01f);
    p = __fmaf_rn(p, r, 0.5f);
    p = __fmaf_rn(p, r, 1.0f);
    p = __fmaf_rn(p, r, 1.0f);
    const int ni = __float_as_int(big) - 0x4B400000;
    const int n1 = ni / 2;
    const int n2 = ni - n1;
    return __fmul_rn(__fmul_rn(p, pow2i(n1)), pow2i(n2));
}

// 1 / y rounded to nearest for y in [1, 2^126): rcp.approx refined by one
// Newton-Raphson step with fused multiply-adds (P. Markstein, IBM J. Res.
// Dev. 34(1), 1990), equal to IEEE division on that whole range.
__device__ __forceinline__ float rcp_rn(float y) {
    float q;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(q) : "f"(y));
    return __fmaf_rn(q, __fmaf_rn(-y, q, 1.0f), q);
}

// vendor/openeva/prim/activation.h:17, 1 / (1 + exp(-x)), with an exp of
// its own for the range the sigmoid needs -- the engine's and the oracle's
// sigmoid, operation for operation: t = -x clamped to [-17, 87]; n and the
// Cody-Waite reduction as in exp_portable (the product-sum for n fused);
// exp(r) by a degree-6 minimax polynomial on [-ln2/2, ln2/2] (Remez
// exchange, coefficients rounded to float) by Horner; one exact scaling by
// 2^n; the round-to-nearest reciprocal above.
__device__ __forceinline__ float sigmoid_exact(float x) {
    if (x != x) return x;
    const float t = fminf(fmaxf(-x, -17.0f), 87.0f);
    const float big = __fmaf_rn(t, 1.44269502f, 12582912.0f);
    const float n = __fsub_rn(big, 12582912.0f);
    float r = __fmaf_rn(-n, 0.693115234375f, t);
    r = __fmaf_rn(-n, 3.19461833e-05f, r);
    float p = 1.38368458e-03f;
    p = __fmaf_rn(p, r, 8.37481581e-03f);
    p = __fmaf_rn(p, r, 4.16682251e-02f);
    p = __fmaf_rn(p, r, 1.66664198e-01f);
    p = __fmaf_rn(p, r, 4.99999911e-01f);
    p = __fmaf_rn(p, r, 1.0f);
    p = __fmaf_rn(p, r, 1.0f);
    return rcp_rn(__fadd_rn(1.0f, __fmul_rn(p, pow2i(__float_as_int(big) - 0x4B400000))));
}

// fmaf chain of one output column over N inputs, in input order
// (vendor/openeva/prim/linear.h:80-90 matvec_ct): acc = fma(w[i*ld], x[i], acc).
template <int N>
__device__ __forceinline__ float dot_col(const float* __restrict__ w, int ld, const float* __restrict__ x,
                                         float acc) {
#pragma unroll 8
    for (int i = 0; i < N; ++i) acc = __fmaf_rn(w[i * ld], x[i], acc);
    return acc;
}

// LayerNorm of OUT channels held by one warp, lane g holding channels
// 4g..4g+3 (lanes g >= OUT/4 hold nothing), in place in y
// (vendor/openeva/prim/layernorm.h:41-62 with eps 1e-5f):
//   mean = (sum_o y_o) / OUT in fp64, summed in channel order;
//   var  = (sum_o (y_o - mean)^2) / OUT, summed in channel order;
//   y_o  = float(((y_o - mean) * inv) * gamma_o + beta_o), inv = 1 / sqrt(var + eps).
template <int OUT>
__device__ __forceinline__ void layernorm_warp(float (&y)[4], const float* __restrict__ gam,
                                               const float* __restrict__ bet) {
    constexpr int G = OUT / 4;
    const int lane = threadIdx.x & 31;
    double s = 0.0;
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
        for (int j = 0; j < 4; ++j) s = __dadd_rn(s, static_cast<double>(__shfl_sync(kFull, y[j], g)));
    const double mean = __ddiv_rn(s, static_cast<double>(OUT));
    double d[4], q[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        d[j] = __dsub_rn(static_cast<double>(y[j]), mean);
        q[j] = __dmul_rn(d[j], d[j]);
    }
    double var = 0.0;
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
        for (int j = 0; j < 4; ++j) var = __dadd_rn(var, __shfl_sync(kFull, q[j], g));
    var = __ddiv_rn(var, static_cast<double>(OUT));
    const double inv = __ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(var, static_cast<double>(1e-5f))));
    if (lane < G) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const double v = __dmul_rn(d[j], inv);
            y[j] = static_cast<float>(__dadd_rn(__dmul_rn(v, static_cast<double>(gam[4 * lane + j])),
                                                static_cast<double>(bet[4 * lane + j])));
        }
    }
}

// Ordered temporal-dropout gate over the active lanes of one warp, lane
// order = ring order (src/ssla_kernels.cpp:903-921, the uint8 counter
// wraps): a lane's pre-increment count is the counter plus its same-cell
// peers on lower lanes; the last peer of each cell writes the count back.
__device__ __forceinline__ bool gate_lanes(unsigned char* cnt, bool act, int key, int window) {
    const unsigned peers = __match_any_sync(kFull, act ? key : -1 - static_cast<int>(threadIdx.x & 31));
    int base = 0;
    if (act) base = cnt[key];
    const int pre = (base + __popc(peers & lanemask_lt())) & 255;
    const bool pass = window <= 1 || (pre % window) == 0;
    __syncwarp();
    if (act && static_cast<int>(threadIdx.x & 31) == 31 - __clz(peers))
        cnt[key] = static_cast<unsigned char>(base + __popc(peers));
    return act && pass;
}

}  // namespace sslab
