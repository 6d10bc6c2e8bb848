// k_head_tc: the YOLOX head (vendor/openeva/heads/async_yolox.h:203-254)
// with its two 1x1 convolutions -- cls_conv | reg_conv, 96 -> 192 outputs,
// BN folded (:81-143) -- on the 5th-generation tensor cores, batched over
// the drain's head events.
//
// The convolutions are one GEMM, D[m][n] = sum_k X[m][k] W1[n][k], with
// M = head events (128 per CTA, the UMMA M), N = 192 (two halves of 96:
// cls, reg), K = 96.  tcgen05.mma kind::tf32 takes both operands from shared
// memory (K-major, 128-byte swizzle) and accumulates in tensor memory.  To
// keep fp32-level accuracy the GEMM runs in three TF32 terms (the split-TF32
// scheme): every fp32 operand a = a_hi + a_lo with a_hi its nearest TF32
// value and a_lo the TF32 rounding of the remainder, and
// D = X_hi W_hi + X_hi W_lo + X_lo W_hi (the X_lo W_lo term is below fp32
// resolution).  The epilogue reads D from tensor memory (tcgen05.ld), adds
// the conv biases, applies SiLU, and the 2 + 4 + 1 prediction rows and the
// box decode run on the CUDA cores, as k_head does.
//
// Results equal k_head's within fp32 rounding of a differently ordered sum,
// not bit for bit (k_head runs the reference's fmaf order), so this head is
// an engine option (ssla_engine_set_head_mode); tests bound the difference.
//
// One elected thread issues the MMAs; completion reaches the CTA through an
// mbarrier (tcgen05.commit).  Every wait is bounded: a wait that runs out
// sets the error word, the CTA waits (bounded) once more for its MMAs and
// frees its tensor memory before it returns.
#include <cstdint>
#include <mutex>

#include "ssla_device.cuh"
#include "ssla_kernels.cuh"

namespace ssla {

namespace {

constexpr int kTM = 128;                 // head events per CTA (UMMA M)
constexpr int kTK = 96;                  // input channels (K)
constexpr int kKB = 3;                   // K blocks of 32 TF32 values (one 128-byte swizzle row)
constexpr int kHalfN = 96;               // N per MMA: cls half, reg half
constexpr int kTcThreads = 128;          // one warpgroup: 4 warps x 32 TMEM lanes
constexpr int kTmemCols = 256;           // power of two >= 192 accumulator columns
constexpr int kActStride = 193;          // act row stride (floats), conflict-free per-row reads
// dynamic shared memory (bytes from a 1024-byte aligned base)
constexpr int kABlk = kTM * 128;         // one K block of A: 128 rows x 128 B
constexpr int kBBlk = kHalfN * 128;      // one K block of a B half: 96 rows x 128 B
constexpr int kAHi = 0, kALo = kAHi + kKB * kABlk, kBHi = kALo + kKB * kABlk, kBLo = kBHi + kKB * kBBlk;
constexpr int kSmemUsed = kBLo + kKB * kBBlk;                          // 172,032
constexpr int kSmemBytes = kSmemUsed + 1024;                            // + alignment slack
static_assert(kTM * kActStride * 4 <= kSmemUsed, "activations reuse the operand tiles");
static_assert(kABlk % 1024 == 0 && kBBlk % 1024 == 0 && kALo % 1024 == 0 && kBHi % 1024 == 0 &&
                  kBLo % 1024 == 0, "swizzle atoms are 1024-byte aligned");
constexpr unsigned long long kTcWaitNs = 100ull * 1000ull * 1000ull;   // 100 ms

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ unsigned long long gtime_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Nearest TF32 value of x (10-bit mantissa; the tensor core reads the top
// 19 bits of each 32-bit operand), by integer rounding of the low 13 bits.
__device__ __forceinline__ float tf32_round(float x) {
    uint32_t u = __float_as_uint(x);
    if ((u & 0x7F800000u) != 0x7F800000u) u = (u + 0x1000u) & 0xFFFFE000u;
    return __uint_as_float(u);
}

// Byte offset of element (row r, k) in a K-major, 128-byte-swizzled tile of
// 32-wide K blocks (blk bytes per block): the 16-byte chunk index is XORed
// with the row's position in its 8-row swizzle atom.
__device__ __forceinline__ uint32_t sw128(int r, int k, int blk) {
    const int kb = k >> 5, c = (k & 31) >> 2;
    return static_cast<uint32_t>(kb * blk + r * 128 + ((c ^ (r & 7)) << 4) + ((k & 3) << 2));
}

// UMMA shared-memory descriptor (K-major, SWIZZLE_128B): start address,
// leading byte offset 16 (unused by swizzled K-major layouts), stride byte
// offset 1024 (between 8-row groups), version 1, layout type 2.
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>(1u) << 16;
    d |= static_cast<uint64_t>(1024u >> 4) << 32;
    d |= static_cast<uint64_t>(1u) << 46;
    d |= static_cast<uint64_t>(2u) << 61;
    return d;
}

// Instruction descriptor: D f32, A and B tf32, both K-major, N = 96, M = 128.
constexpr uint32_t kIdesc = (1u << 4) | (2u << 7) | (2u << 10) | (static_cast<uint32_t>(kHalfN >> 3) << 17) |
                            (static_cast<uint32_t>(kTM >> 4) << 24);

__device__ __forceinline__ void umma_tf32(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n"
        :
        : "r"(tmem_d), "l"(a), "l"(b), "r"(kIdesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u));
}

__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ bool mbar_wait_ns(uint32_t bar, uint32_t parity, unsigned long long limit) {
    const unsigned long long t0 = gtime_ns();
    while (!mbar_try(bar, parity))
        if (gtime_ns() - t0 > limit) return false;
    return true;
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Stage one B half (96 output channels, hi and lo terms) into its tiles.
__device__ void stage_b(const float* __restrict__ w1, int half, uint8_t* sm) {
    const float* hi = w1 + static_cast<size_t>(half) * kHalfN * kTK;
    const float* lo = w1 + static_cast<size_t>(2 * kHalfN) * kTK + static_cast<size_t>(half) * kHalfN * kTK;
    for (int t = threadIdx.x; t < kHalfN * (kTK / 4); t += kTcThreads) {
        const int r = t / (kTK / 4), k = 4 * (t % (kTK / 4));
        const uint32_t off = sw128(r, k, kBBlk);
        *reinterpret_cast<float4*>(sm + kBHi + off) = __ldg(reinterpret_cast<const float4*>(hi + r * kTK + k));
        *reinterpret_cast<float4*>(sm + kBLo + off) = __ldg(reinterpret_cast<const float4*>(lo + r * kTK + k));
    }
}

__global__ void __launch_bounds__(kTcThreads, 1) k_head_tc(HeadArgs a) {
    pdl_enter();
    extern __shared__ uint8_t tc_dyn[];
    __shared__ __align__(8) uint64_t bar;
    __shared__ uint32_t tmem_base_s;
    __shared__ int abort_s;
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(tc_dyn) + 1023) & ~static_cast<uintptr_t>(1023));
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n = min(a.count[4], a.g.cap[4]);
    const int row0 = blockIdx.x * kTM;
    if (row0 >= n) return;                         // uniform: no TMEM was taken
    const uint32_t bar_a = smem_u32(&bar);
    if (tid == 0) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar_a) : "memory");
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        abort_s = 0;
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base_s)),
                     "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    // ---- A: this CTA's head-event rows, hi and lo TF32 terms ----
    for (int t = tid; t < kTM * (kTK / 4); t += kTcThreads) {
        const int m = t / (kTK / 4), k = 4 * (t % (kTK / 4));
        const int row = row0 + m;
        float4 x = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (row < n) x = __ldg(reinterpret_cast<const float4*>(a.X + static_cast<size_t>(row) * kTK + k));
        const float4 h = make_float4(tf32_round(x.x), tf32_round(x.y), tf32_round(x.z), tf32_round(x.w));
        const float4 l = make_float4(tf32_round(x.x - h.x), tf32_round(x.y - h.y), tf32_round(x.z - h.z),
                                     tf32_round(x.w - h.w));
        const uint32_t off = sw128(m, k, kABlk);
        *reinterpret_cast<float4*>(sm + kAHi + off) = h;
        *reinterpret_cast<float4*>(sm + kALo + off) = l;
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = tmem_base_s;
    const uint32_t sbase = smem_u32(sm);
    // ---- the two N halves: stage W1's half, 3 terms x 3 K blocks x 4 K steps ----
    for (int half = 0; half < 2; ++half) {
        stage_b(a.tc_w1, half, sm);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // generic writes -> tensor core reads
        __syncthreads();
        if (tid == 0) {
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t d = tmem + static_cast<uint32_t>(half * kHalfN);
            const uint32_t a_off[3] = {kAHi, kAHi, kALo};
            const uint32_t b_off[3] = {kBHi, kBLo, kBHi};
            uint32_t acc = 0;
            for (int term = 0; term < 3; ++term)
                for (int kb = 0; kb < kKB; ++kb)
                    for (int ks = 0; ks < 4; ++ks) {
                        const uint64_t da = umma_desc(sbase + a_off[term] + kb * kABlk + ks * 32);
                        const uint64_t db = umma_desc(sbase + b_off[term] + kb * kBBlk + ks * 32);
                        umma_tf32(d, da, db, acc);
                        acc = 1;
                    }
            asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar_a)
                         : "memory");
        }
        // every thread waits for this half's MMAs (phase `half`) before B is restaged
        const bool ok = mbar_wait_ns(bar_a, static_cast<uint32_t>(half), kTcWaitNs);
        if (!ok) atomicExch(&abort_s, 1);
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        __syncthreads();
        if (abort_s) break;
    }
    const bool aborted = abort_s != 0;
    if (aborted) {
        // the MMAs may still be running: wait once more (bounded), then free
        if (tid == 0 && a.err) atomicOr_system(a.err, 1u);
        mbar_wait_ns(bar_a, 0u, kTcWaitNs);
        mbar_wait_ns(bar_a, 1u, kTcWaitNs);
    } else {
        // ---- epilogue: D rows from tensor memory, + bias, SiLU -> act (reuses the tiles) ----
        float* act = reinterpret_cast<float*>(sm);
        const int m = warp * 32 + lane;                        // this thread's TMEM lane = row
        const uint32_t trow = tmem + (static_cast<uint32_t>(warp * 32) << 16);
        for (int c0 = 0; c0 < 2 * kHalfN; c0 += 32) {
            float v[32];
            tmem_ld32(trow + static_cast<uint32_t>(c0), v);
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                const int col = c0 + i;
                const float b = __ldg((col < kHalfN ? a.head.cls_conv_b : a.head.reg_conv_b) + (col % kHalfN));
                const float y = v[i] + b;
                act[m * kActStride + col] = y * ssla_sigmoidf(y);
            }
        }
        __syncwarp();
        // ---- prediction rows and decode (CUDA cores), one head event per thread ----
        const int row = row0 + m;
        if (row < n) {
            const int ncls = a.g.ncls, cols = 5 + ncls;
            const float* ar = act + m * kActStride;
            const uint32_t xy0 = a.E4[row].xy0;
            const int cx = static_cast<int>(xy0 & 0xFFFFu) >> 3, cy = static_cast<int>(xy0 >> 16) >> 3;
            for (int r = 0; r < cols; ++r) {
                float acc;
                if (r < 4) {
                    acc = __ldg(a.head.reg_pred_b + r);
                    for (int i = 0; i < kHalfN; ++i) acc = fmaf(__ldg(a.head.reg_predT + i * 4 + r), ar[kHalfN + i], acc);
                } else if (r == 4) {
                    acc = __ldg(a.head.obj_pred_b);
                    for (int i = 0; i < kHalfN; ++i) acc = fmaf(__ldg(a.head.obj_predT + i), ar[kHalfN + i], acc);
                } else {
                    const int c = r - 5;
                    acc = __ldg(a.head.cls_pred_b + c);
                    for (int i = 0; i < kHalfN; ++i) acc = fmaf(__ldg(a.head.cls_predT + i * ncls + c), ar[i], acc);
                }
                float d;
                if (r == 0) d = (acc + static_cast<float>(cx)) * static_cast<float>(a.g.stride_w);
                else if (r == 1) d = (acc + static_cast<float>(cy)) * static_cast<float>(a.g.stride_h);
                else if (r == 2) d = ssla_expf(acc) * static_cast<float>(a.g.stride_w);
                else if (r == 3) d = ssla_expf(acc) * static_cast<float>(a.g.stride_h);
                else d = acc;
                a.head_dec[static_cast<size_t>(row) * cols + r] = d;
                a.head_raw[static_cast<size_t>(row) * cols + r] = acc;
            }
        }
    }
    // ---- free the tensor memory once every lane's loads are done ----
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
    }
}

}  // namespace

int head_tc_smem_bytes() { return kSmemBytes; }

void launch_head_tc(cudaStream_t st, const HeadArgs& a, long long max_rows) {
    static std::mutex mu;
    static unsigned long long attr_done = 0;          // one bit per device
    int dev = 0;
    cudaGetDevice(&dev);
    {
        std::lock_guard<std::mutex> lk(mu);
        const unsigned long long bit = 1ull << (dev & 63);
        if (!(attr_done & bit)) {
            cudaFuncSetAttribute(k_head_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
            attr_done |= bit;
        }
    }
    const long long tiles = (max_rows + kTM - 1) / kTM;
    const int grid = static_cast<int>(tiles < 1 ? 1 : tiles);
    pdl_launch(k_head_tc, grid, kTcThreads, kSmemBytes, st, a);
}

}  // namespace ssla
