// Allocation-free stage-2 gate pass: ssla_s2s3_gate_codes_noalloc.
//
// Some callers cannot allocate device memory at the point where they need
// the gate decisions of a drain: a per-batch real-time loop (the P1 ring
// drain runs once per batch under a latency budget, and a cudaMalloc or
// cudaFree there may synchronise the whole device and stall for
// milliseconds), or a host that runs the drain inside a memory pool owned by
// another runtime and must not grow the process's device footprint.  This
// entry point therefore takes all of its scratch memory from one file-scope
// __device__ array of fixed size and calls no allocating routine at all: no
// device, pinned or managed allocation, no library call that allocates.
//
// It evaluates the same stage-2 and stage-3 temporal-dropout gates as
// ssla_s2s3_drain_n_multi (k_gates_s2 / k_write_slots in ssla_kernels.cu,
// the tdrop rule of ssla_s2_s3_head_celled.cuh:742-745): records of each
// block in ring order, the uint8 tdrop counters of cfg advanced in place,
// and the pass2 / pass3 codes of every output slot written (1 / 0, -1 for
// records outside the block's owned strip).  It leaves the hidden state and
// the s3_feat words of the slots untouched.
//
// Work per call is linear in the records: the records are first bucketed
// by (block, stage-3 cell) inside the scratch array -- a stable two-pass
// LSD radix sort of (key << 16 | record) words, so each bucket keeps ring
// order -- and each gate warp then walks only its own cell's bucket.
//
// Set-up: the first call on a device (and the first call after the
// device's context changed, e.g. after cudaDeviceReset) looks up the scratch
// array's device address with cudaGetSymbolAddress, with that device
// current, and keeps it for later calls; that call may load the module and
// should therefore come before any stream capture on the device.
// Concurrency: every call on a device shares the one scratch array, so two
// calls whose work overlaps in time on the same device (different streams or
// threads without ordering between them) race and give undefined results.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>
#include <string>

#include "ssla_abi_types.h"
#include "ssla_b200.h"

namespace ssla {
void set_last_error(const std::string& msg);   // ssla_engine.cu
}

namespace {

constexpr int kMaxRecords = SSLA_NOALLOC_MAX_RECORDS;   // record index fits 16 bits
constexpr int kMaxKeys = SSLA_NOALLOC_MAX_CELLS;        // blocks x stage-3 cells; key fits 16 bits
constexpr uint32_t kNoKey = 0xFFFFu;                    // records outside the stage-2 grid
constexpr int kMaxDevices = 64;
constexpr int kNT = 256;
constexpr int kTile = 2048;                             // records per radix-sort tile
constexpr int kMaxTiles = kMaxRecords / kTile;
static_assert(kMaxRecords <= 65536 && kMaxKeys < 65536, "keys and record indices are 16-bit fields");
static_assert(kMaxRecords % kTile == 0 && kTile % kNT == 0, "tiles of whole rounds");

// Per-call scratch.  xy: packed stage-0 coordinates of each record (the
// packing of the drain_n record prologue); sorted: (key << 16 | record)
// words, ping-pong buffers of the radix sort (buffer 0 ends up sorted by
// key, ring order inside each key); hist: per-tile digit counts, then their
// exclusive offsets; flag: gate results, bit 0 = passed gate 2, bit 1 =
// passed gate 3.  Every flag of the call's records must start at zero (a
// record no gate warp visits keeps "did not pass"); k_na_pack clears them at
// the start of each call.
struct NoAllocScratch {
    uint32_t xy[kMaxRecords];
    uint32_t sorted[2][kMaxRecords];
    uint32_t hist[256 * kMaxTiles];
    uint8_t flag[kMaxRecords];
};

static __device__ __align__(256) NoAllocScratch g_scratch;

struct NaParams {
    int P, n, W2, H2, W3, H3, window;
    int off[SSLA_MAX_BLOCKS + 1];
    const HybridInputRec* ring[SSLA_MAX_BLOCKS];
    HybridS2S3OutputSlot* out[SSLA_MAX_BLOCKS];
    uint8_t* cnt2[SSLA_MAX_BLOCKS];
    uint8_t* cnt3[SSLA_MAX_BLOCKS];
    int own_x0[SSLA_MAX_BLOCKS], own_x1[SSLA_MAX_BLOCKS];
    int own_y0[SSLA_MAX_BLOCKS], own_y1[SSLA_MAX_BLOCKS];
};

__device__ __forceinline__ int na_block_of(const NaParams& a, int i) {
    int p = 0;
    while (p + 1 < a.P && i >= a.off[p + 1]) ++p;
    return p;
}

__device__ __forceinline__ unsigned na_lanemask_lt() {
    unsigned m;
    asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
    return m;
}

// tdrop rule: pass iff window <= 1 or the pre-increment uint8 count is a
// multiple of the window (same rule as gate_pass in ssla_kernels.cu).
__device__ __forceinline__ bool na_pass(int pre, int window) {
    return window <= 1 || ((pre & 255) % window) == 0;
}

// Ordered gate over the active lanes of a warp (lane order = ring order);
// `key` picks one of the counters in `cnt`, inactive lanes pass a key of
// their own.
__device__ __forceinline__ bool na_warp_gate(bool active, int key, int* cnt, int window) {
    const unsigned peers = __match_any_sync(0xffffffffu, key);
    bool pass = false;
    if (active) pass = na_pass(cnt[key] + __popc(peers & na_lanemask_lt()), window);
    __syncwarp();
    if (active && (threadIdx.x & 31) == 31 - __clz(peers)) cnt[key] += __popc(peers);
    __syncwarp();
    return pass;
}

// 1) records -> packed coordinates and (key, record) words; clear the gate
// flags.  key = block * (W3 * H3) + stage-3 cell.
__global__ void k_na_pack(NaParams a, NoAllocScratch* sc) {
    const int cells = a.W3 * a.H3;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < a.n; i += gridDim.x * blockDim.x) {
        const int p = na_block_of(a, i);
        const HybridInputRec& r = a.ring[p][i - a.off[p]];
        const uint32_t x2 = r.x, y2 = r.y;
        sc->xy[i] = (x2 << 2) | ((y2 << 2) << 16);
        sc->flag[i] = 0;
        const bool in = x2 < static_cast<uint32_t>(a.W2) && y2 < static_cast<uint32_t>(a.H2);
        const uint32_t key = in ? static_cast<uint32_t>(p * cells) + (y2 >> 1) * a.W3 + (x2 >> 1) : kNoKey;
        sc->sorted[0][i] = (key << 16) | static_cast<uint32_t>(i);
    }
}

// 2) one stable LSD radix pass over the 8-bit digit at `shift` (16 or 24):
// per-tile digit counts, their exclusive offsets in digit-major order, and
// an ordered scatter (records of a tile in rounds of 256, ranks within a
// round from warp matches and per-warp digit counts).
__global__ void __launch_bounds__(kNT) k_na_hist(int n, const uint32_t* src, int shift, uint32_t* hist) {
    __shared__ uint32_t h[256];
    const int t = blockIdx.x, T = gridDim.x;
    h[threadIdx.x] = 0;
    __syncthreads();
    const int i1 = min(n, (t + 1) * kTile);
    for (int i = t * kTile + threadIdx.x; i < i1; i += kNT) atomicAdd(&h[(src[i] >> shift) & 255u], 1u);
    __syncthreads();
    hist[threadIdx.x * T + t] = h[threadIdx.x];
}

__global__ void __launch_bounds__(kNT) k_na_scan(int T, uint32_t* hist) {
    __shared__ uint32_t part[kNT];
    const int d = threadIdx.x;                  // thread d owns entries [d*T, d*T + T)
    uint32_t s = 0;
    for (int t = 0; t < T; ++t) s += hist[d * T + t];
    part[d] = s;
    __syncthreads();
    if (d == 0) {
        uint32_t run = 0;
        for (int k = 0; k < kNT; ++k) {
            const uint32_t v = part[k];
            part[k] = run;
            run += v;
        }
    }
    __syncthreads();
    uint32_t run = part[d];
    for (int t = 0; t < T; ++t) {
        const uint32_t v = hist[d * T + t];
        hist[d * T + t] = run;
        run += v;
    }
}

__global__ void __launch_bounds__(kNT) k_na_scatter(int n, const uint32_t* src, uint32_t* dst, int shift,
                                                    const uint32_t* hist) {
    constexpr int kWarps = kNT / 32;
    __shared__ uint32_t cursor[256];
    __shared__ uint32_t wc[kWarps][256];
    const int t = blockIdx.x, T = gridDim.x;
    const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    cursor[tid] = hist[tid * T + t];
    for (int i0 = t * kTile; i0 < min(n, (t + 1) * kTile); i0 += kNT) {
        for (int k = 0; k < kWarps; ++k) wc[k][tid] = 0;
        __syncthreads();
        const int i = i0 + tid;
        const bool act = i < n;
        const uint32_t v = act ? src[i] : 0u;
        const int d = act ? static_cast<int>((v >> shift) & 255u) : 256 + lane;
        const unsigned peers = __match_any_sync(0xffffffffu, d);
        const int rank = __popc(peers & na_lanemask_lt());
        if (act && rank == 0) wc[w][d] = __popc(peers);
        __syncthreads();
        {   // per digit: offsets of the warps' groups, in warp order
            uint32_t run = cursor[tid];
            for (int k = 0; k < kWarps; ++k) {
                const uint32_t c = wc[k][tid];
                wc[k][tid] = run;
                run += c;
            }
            cursor[tid] = run;
        }
        __syncthreads();
        if (act) dst[wc[w][d] + rank] = v;
        __syncthreads();
    }
}

// 3) one warp per (block, stage-3 cell): the cell's bucket in ring order,
// gate 2 on the record's stage-2 cell counter, gate 3 on the stage-3 cell
// counter for records that passed gate 2 (k_gates_s2 without tile lists).
__device__ __forceinline__ int na_lower_bound(const uint32_t* v, int n, uint32_t x) {
    int lo = 0, hi = n;
    while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (v[mid] < x) lo = mid + 1;
        else hi = mid;
    }
    return lo;
}

__global__ void __launch_bounds__(32) k_na_gates(NaParams a, NoAllocScratch* sc) {
    const int p = blockIdx.x, cell = blockIdx.y;
    const int gx = cell % a.W3, gy = cell / a.W3;
    const int lane = threadIdx.x;
    __shared__ int c2[4], c3[1];
    uint8_t* cnt2 = a.cnt2[p];
    uint8_t* cnt3 = a.cnt3[p];
    const uint32_t key = static_cast<uint32_t>(p * a.W3 * a.H3 + cell);
    const uint32_t* sorted = sc->sorted[0];
    const int lo = na_lower_bound(sorted, a.n, key << 16);
    const int hi = na_lower_bound(sorted, a.n, (key + 1) << 16);
    if (lo == hi) return;                      // no record in this cell: counters unchanged
    if (lane < 4) c2[lane] = cnt2[(gy * 2 + lane / 2) * a.W2 + gx * 2 + (lane % 2)];
    if (lane == 0) c3[0] = cnt3[gy * a.W3 + gx];
    __syncwarp();
    for (int j0 = lo; j0 < hi; j0 += 32) {
        const bool own = j0 + lane < hi;
        const int j = own ? static_cast<int>(sorted[j0 + lane] & 0xFFFFu) : 0;
        const uint32_t xy0 = own ? sc->xy[j] : 0u;
        const int x2 = static_cast<int>(xy0 & 0xFFFFu) >> 2, y2 = static_cast<int>(xy0 >> 16) >> 2;
        const int sub = (y2 & 1) * 2 + (x2 & 1);
        const bool p2 = na_warp_gate(own, own ? sub : 100 + lane, c2, a.window);
        const bool in3 = own && p2;
        const bool p3 = na_warp_gate(in3, in3 ? 0 : 100 + lane, c3, a.window);
        if (own) sc->flag[j] = static_cast<uint8_t>((p2 ? 1u : 0u) | ((in3 && p3) ? 2u : 0u));
    }
    __syncwarp();
    if (lane < 4) cnt2[(gy * 2 + lane / 2) * a.W2 + gx * 2 + (lane % 2)] = static_cast<uint8_t>(c2[lane]);
    if (lane == 0) cnt3[gy * a.W3 + gx] = static_cast<uint8_t>(c3[0]);
}

// 4) pass codes of the output slots (k_write_slots' rule: -1 outside the
// owned strip, pass3 only meaningful after pass2).
__global__ void k_na_codes(NaParams a, const NoAllocScratch* sc) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < a.n; i += gridDim.x * blockDim.x) {
        const int p = na_block_of(a, i);
        if (a.out[p] == nullptr) continue;
        const uint32_t xy0 = sc->xy[i];
        const int x2 = static_cast<int>(xy0 & 0xFFFFu) >> 2, y2 = static_cast<int>(xy0 >> 16) >> 2;
        const bool owner = x2 >= a.own_x0[p] && x2 < a.own_x1[p] && y2 >= a.own_y0[p] && y2 < a.own_y1[p];
        const int f = sc->flag[i];
        const int p2 = f & 1, p3 = (f >> 1) & 1;
        HybridS2S3OutputSlot* o = a.out[p] + (i - a.off[p]);
        o->pass2 = owner ? p2 : -1;
        o->pass3 = owner ? (p2 ? p3 : 0) : -1;
    }
}

// ---- set-up: the scratch array's device address, per device and context ----
using CtxGetCurrentFn = CUresult (*)(CUcontext*);

struct ScratchSlot {
    CUcontext ctx = nullptr;
    NoAllocScratch* ptr = nullptr;
};

std::mutex g_setup_mu;
ScratchSlot g_scratch_slot[kMaxDevices];
CtxGetCurrentFn g_ctx_get_current = nullptr;

// Device address of the scratch array on the current device (looked up once
// per device, and again if the device's current context is a new one).
// Returns nullptr and sets the error text on failure.
NoAllocScratch* scratch_for(int device) {
    std::lock_guard<std::mutex> lk(g_setup_mu);
    if (g_ctx_get_current == nullptr) {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q{};
        const cudaError_t e = cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q);
        if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || fn == nullptr) {
            ssla::set_last_error("ssla_s2s3_gate_codes_noalloc: cuCtxGetCurrent entry point not found");
            return nullptr;
        }
        g_ctx_get_current = reinterpret_cast<CtxGetCurrentFn>(fn);
    }
    // A thread the runtime has not used yet may have no current context;
    // the symbol lookup binds the device's primary context to it.
    CUcontext ctx = nullptr;
    if (g_ctx_get_current(&ctx) != CUDA_SUCCESS) ctx = nullptr;
    ScratchSlot& s = g_scratch_slot[device];
    if (s.ptr == nullptr || ctx == nullptr || s.ctx != ctx) {
        void* ptr = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&ptr, g_scratch);
        if (e != cudaSuccess || ptr == nullptr) {
            ssla::set_last_error(std::string("cudaGetSymbolAddress(scratch): ") + cudaGetErrorString(e));
            return nullptr;
        }
        if (g_ctx_get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) {
            ssla::set_last_error("ssla_s2s3_gate_codes_noalloc: no current CUDA context");
            return nullptr;
        }
        s.ctx = ctx;
        s.ptr = static_cast<NoAllocScratch*>(ptr);
    }
    return s.ptr;
}

int launch_grid(int n) {
    const int g = (n + kNT - 1) / kNT;
    return g < 1 ? 1 : (g > 1184 ? 1184 : g);
}

}  // namespace

extern "C" int ssla_s2s3_gate_codes_noalloc(const HybridS2S3Config* cfg,
                                            const HybridInputRec* const* rings, const int* ns,
                                            HybridS2S3OutputSlot* const* outs, void* stream) {
    auto fail = [](int code, const std::string& msg) { ssla::set_last_error(msg); return code; };
    if (!cfg || !rings || !ns) return fail(SSLA_ERR_ARG, "null argument");
    const int P = cfg->n_blocks;
    if (P < 1 || P > SSLA_MAX_BLOCKS) return fail(SSLA_ERR_ARG, "cfg->n_blocks must be 1..16");
    if (cfg->H2 <= 0 || cfg->W2 <= 0 || (cfg->H2 % 2) || (cfg->W2 % 2) ||
        cfg->H3 != cfg->H2 / 2 || cfg->W3 != cfg->W2 / 2) {
        return fail(SSLA_ERR_ARG, "cfg grid sizes must be even with H3 = H2/2, W3 = W2/2");
    }
    NaParams a{};
    a.P = P; a.W2 = cfg->W2; a.H2 = cfg->H2; a.W3 = cfg->W3; a.H3 = cfg->H3;
    a.window = cfg->tdrop_window;
    if (static_cast<long long>(cfg->W3) * cfg->H3 * P > kMaxKeys) {
        return fail(SSLA_ERR_CAPACITY, "ssla_s2s3_gate_codes_noalloc: blocks x stage-3 cells exceed the "
                                       "allocation-free limit of " + std::to_string(kMaxKeys));
    }
    long long total = 0;
    for (int b = 0; b < P; ++b) {
        if (ns[b] < 0) return fail(SSLA_ERR_ARG, "negative record count");
        total += ns[b];
    }
    if (total > kMaxRecords) {
        return fail(SSLA_ERR_CAPACITY, "ssla_s2s3_gate_codes_noalloc: " + std::to_string(total) +
                                           " records exceed the allocation-free limit of " +
                                           std::to_string(kMaxRecords) + " records per call");
    }
    total = 0;
    for (int b = 0; b < P; ++b) {
        if (ns[b] > 0 && rings[b] == nullptr) return fail(SSLA_ERR_ARG, "null ring with records");
        if (cfg->tdrop_s2[b] == 0 || cfg->tdrop_s3[b] == 0) {
            return fail(SSLA_ERR_ARG, "null tdrop counter buffer");
        }
        a.off[b] = static_cast<int>(total);
        total += ns[b];
        a.ring[b] = rings[b];
        a.out[b] = outs ? outs[b] : nullptr;
        a.cnt2[b] = reinterpret_cast<uint8_t*>(cfg->tdrop_s2[b]);
        a.cnt3[b] = reinterpret_cast<uint8_t*>(cfg->tdrop_s3[b]);
        a.own_x0[b] = cfg->strip[b].owned_lo; a.own_x1[b] = cfg->strip[b].owned_hi;
        a.own_y0[b] = cfg->strip[b].owned_y_lo; a.own_y1[b] = cfg->strip[b].owned_y_hi;
    }
    a.off[P] = static_cast<int>(total);
    a.n = static_cast<int>(total);
    int device = 0;
    cudaError_t e = cudaGetDevice(&device);
    if (e != cudaSuccess) return fail(SSLA_ERR_NO_DEVICE, cudaGetErrorString(e));
    if (device < 0 || device >= kMaxDevices) return fail(SSLA_ERR_ARG, "device ordinal out of range");
    NoAllocScratch* sc = scratch_for(device);
    if (!sc) return SSLA_ERR_CUDA;
    if (a.n == 0) return SSLA_OK;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int T = (a.n + kTile - 1) / kTile;
    k_na_pack<<<launch_grid(a.n), kNT, 0, st>>>(a, sc);
    for (int pass = 0; pass < 2; ++pass) {       // key bits 16-23, then 24-31
        const uint32_t* src = sc->sorted[pass];
        uint32_t* dst = sc->sorted[pass ^ 1];
        k_na_hist<<<T, kNT, 0, st>>>(a.n, src, 16 + 8 * pass, sc->hist);
        k_na_scan<<<1, kNT, 0, st>>>(T, sc->hist);
        k_na_scatter<<<T, kNT, 0, st>>>(a.n, src, dst, 16 + 8 * pass, sc->hist);
    }
    k_na_gates<<<dim3(P, a.W3 * a.H3), 32, 0, st>>>(a, sc);
    k_na_codes<<<launch_grid(a.n), kNT, 0, st>>>(a, sc);
    e = cudaGetLastError();
    if (e != cudaSuccess) {
        return fail(SSLA_ERR_CUDA, std::string("ssla_s2s3_gate_codes_noalloc launch: ") +
                                       cudaGetErrorString(e));
    }
    return SSLA_OK;
}
