// Exact strip sharding of one sensor across GPUs: exchange of boundary
// layer inputs between neighbouring strips.
//
// A strip engine drains its own events plus a band of its neighbours' events
// (the rows within `band` of each boundary, whole stage-3 block rows).  Gates
// and preprocess of every band event are exact locally (complete blocks and
// pixels), but a band event's layer outputs depend on cells beyond the band.
// So after each of layers 1-6, every strip sends the next-layer input rows
// of ITS events in each neighbour's band to that neighbour, which overwrites
// the rows of those (foreign) events before the next layer reads them: every
// cell an owned event reads is then updated by exactly the events and inputs
// of the single-sensor run, and owned outputs are bit-identical to it.
//
// Both sides walk the same stage list in stream order with identical flags,
// so "my events in the neighbour's band" and "the neighbour's foreign events"
// correspond row for row.  Transport: the exporter writes the rows and a
// count into the receiver's buffer (peer memory over NVLink, or local memory
// when both strips share a GPU), then publishes the exchange's sequence
// number in the receiver's flag word; the importer waits (bounded) for the
// flag, checks the count against its own list and scatters.  Buffers are
// double-buffered by sequence parity; each side both sends and receives at
// every exchange, which keeps a fast strip at most one exchange ahead.
#include "ssla_b200.h"
#include "ssla_cluster.cuh"
#include "ssla_kernels.cuh"

namespace ssla {

namespace {

constexpr int kSelNT = 1024;

__device__ __forceinline__ unsigned lanemask_lt_() {
    unsigned m;
    asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
    return m;
}

// One CTA per stage list k = 1..3: order-preserving selection of the list's
// entries into four index lists -- [side][kind], side 0 = up (rows < lo),
// 1 = down (rows >= hi); kind 0 = mine in that neighbour's band (send), 1 =
// foreign from that neighbour (receive).
__global__ void __launch_bounds__(kSelNT) k_band_select(StripSelectArgs a) {
    const int k = blockIdx.x + 1;
    const StageEntry* E = a.E[k];
    const int n = min(a.count[k], a.g_cap[k]);
    __shared__ int wsum[kSelNT / 32][4];
    __shared__ int run[4];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (threadIdx.x < 4) run[threadIdx.x] = 0;
    __syncthreads();
    int* out = a.idx + static_cast<size_t>(k - 1) * 4 * a.cap;
    for (int j0 = 0; j0 < n; j0 += kSelNT) {
        const int i = j0 + static_cast<int>(threadIdx.x);
        bool p[4] = {false, false, false, false};
        if (i < n) {
            const int y = static_cast<int>(E[i].xy0 >> 16);
            p[0] = a.has[0] && y >= a.lo && y < a.lo + a.band;       // up: mine, in its band
            p[1] = a.has[0] && y < a.lo;                              // up: foreign
            p[2] = a.has[1] && y >= a.hi - a.band && y < a.hi;       // down: mine, in its band
            p[3] = a.has[1] && y >= a.hi;                             // down: foreign
        }
        unsigned m[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            m[q] = __ballot_sync(0xffffffffu, p[q]);
            if (lane == 0) wsum[warp][q] = __popc(m[q]);
        }
        __syncthreads();
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            if (!p[q]) continue;
            int wo = 0;
            for (int w = 0; w < warp; ++w) wo += wsum[w][q];
            const int pos = run[q] + wo + __popc(m[q] & lanemask_lt_());
            if (pos < a.cap) out[static_cast<size_t>(q) * a.cap + pos] = i;
        }
        __syncthreads();
        if (threadIdx.x < 4) {
            int tot = 0;
            for (int w = 0; w < kSelNT / 32; ++w) tot += wsum[w][threadIdx.x];
            run[threadIdx.x] += tot;
        }
        __syncthreads();
    }
    if (threadIdx.x < 4) {
        const int c = run[threadIdx.x];
        a.cnt[(k - 1) * 4 + threadIdx.x] = c;
        if (c > a.cap && a.err) atomicOr_system(a.err, SSLA_STRIP_ERR_CAPACITY);
    }
}

// Rows idx[0..cnt) of X (C floats each) -> dst data (packed), then the count
// and the sequence number into the receiver's header; the last CTA to finish
// publishes (every CTA fences its stores first).
__global__ void __launch_bounds__(256) k_strip_export(StripXferArgs a) {
    const int n = min(*a.cnt, a.cap);
    const int C = a.C;
    for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < n * C; t += gridDim.x * blockDim.x) {
        const int r = t / C, c = t % C;
        a.data[t] = a.X[static_cast<size_t>(a.idx[r]) * C + c];
    }
    __threadfence_system();
    __syncthreads();
    __shared__ bool last;
    if (threadIdx.x == 0) last = atomicAdd(a.done_ctr, 1u) == gridDim.x - 1;
    __syncthreads();
    if (last && threadIdx.x == 0) {
        *a.done_ctr = 0u;
        volatile unsigned long long* hdr = a.header;
        hdr[1 + a.parity] = static_cast<unsigned long long>(n);
        __threadfence_system();
        asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(a.header), "l"(a.seq) : "memory");
    }
}

// Waits (bounded, when `wait`) for the sender's sequence number, checks its
// row count against this strip's foreign list and scatters the rows into X.
__global__ void __launch_bounds__(256) k_strip_import(StripXferArgs a) {
    __shared__ int ok;
    if (threadIdx.x == 0) {
        int good = 1;
        const unsigned long long t0 = cl::gtime();
        for (;;) {
            unsigned long long v;
            asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(a.header) : "memory");
            if (v >= a.seq) break;
            if (!a.wait || cl::gtime() - t0 > a.wait_ns) {
                good = 0;
                if (a.err) atomicOr_system(a.err, SSLA_STRIP_ERR_TIMEOUT);
                break;
            }
        }
        if (good) {
            const unsigned long long sent = reinterpret_cast<volatile unsigned long long*>(a.header)[1 + a.parity];
            if (sent != static_cast<unsigned long long>(min(*a.cnt, a.cap))) {
                good = 0;
                if (a.err) atomicOr_system(a.err, SSLA_STRIP_ERR_MISMATCH);
            }
        }
        ok = good;
    }
    __syncthreads();
    if (!ok) return;
    const int n = min(*a.cnt, a.cap);
    const int C = a.C;
    for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < n * C; t += gridDim.x * blockDim.x) {
        const int r = t / C, c = t % C;
        a.X[static_cast<size_t>(a.idx[r]) * C + c] = a.data[t];
    }
}

// Events outside the strip's own rows (its neighbours' band events): their
// outputs are the neighbours' to compute, so contributions and LayerNorm
// skip them.
__global__ void k_mark_foreign(int n, const uint32_t* __restrict__ ev_xy, uint8_t* __restrict__ rflags, int lo,
                               int hi) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const int y = static_cast<int>(ev_xy[i] >> 16);
        if ((rflags[i] & F_VALID) && (y < lo || y >= hi)) rflags[i] |= F_FOREIGN;
    }
}

}  // namespace

void launch_mark_foreign(cudaStream_t st, int n, const uint32_t* ev_xy, uint8_t* rflags, int lo, int hi) {
    if (n > 0) k_mark_foreign<<<(n + 255) / 256 < 1184 ? (n + 255) / 256 : 1184, 256, 0, st>>>(n, ev_xy, rflags, lo, hi);
}

void launch_band_select(cudaStream_t st, const StripSelectArgs& a) {
    k_band_select<<<3, kSelNT, 0, st>>>(a);
}

void launch_strip_export(cudaStream_t st, const StripXferArgs& a) {
    k_strip_export<<<148, 256, 0, st>>>(a);
}

void launch_strip_import(cudaStream_t st, const StripXferArgs& a) {
    k_strip_import<<<148, 256, 0, st>>>(a);
}

}  // namespace ssla
