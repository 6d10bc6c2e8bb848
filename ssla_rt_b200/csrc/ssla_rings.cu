// Ring drains: many independent event streams, each fed through its own
// pinned host ring (the SslaLiveRing head / tail / events_done protocol of
// include/spsc.h:9-11 and orin/orin/ring.py:34-152), drained together by the
// chunk engine, one ring per partition.
//
// Per drain the host reads every ring's head (acquire) and takes up to a
// per-ring budget of the published events.  k_ring_gather copies them from
// the rings' slots (device-mapped pinned memory, read once over PCIe with
// coalesced 16-byte loads) into the chunk's event rows, partition-major, and
// releases each ring's tail once every CTA's copies are done, so the
// producer may reuse the slots while the drain runs.  After the drain,
// k_ring_scatter writes each event's flags and each head event's decoded
// prediction row into the ring's per-slot outputs and then releases the
// ring's events_done -- the persistent kernel's per-record output slots and
// events_done words (ssla_s2_s3_head_celled.cuh:1547-1784,
// orin/hybrid_runner_multi.py:445-462).
#include "ssla_b200.h"
#include "ssla_kernels.cuh"

namespace ssla {

namespace {

constexpr int kRingNT = 256;

// Partition of chunk row i: the last p with off[p] <= i (empty partitions
// have off[p] == off[p + 1] and are skipped).
__device__ __forceinline__ int ring_of(const int* so, int P, int i) {
    int lo = 0, hi = P;                  // so[lo] <= i < so[hi]
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (so[mid] <= i) lo = mid;
        else hi = mid;
    }
    return lo;
}

__device__ __forceinline__ void load_offsets(const RingArgs& a, int* so) {
    for (int t = threadIdx.x; t < a.P; t += blockDim.x) so[t] = a.take[t].off;
    if (threadIdx.x == 0) so[a.P] = a.n_total;
    __syncthreads();
}

// True in the last CTA to finish (after every CTA's stores are fenced at
// system scope); that CTA also re-arms the counter.
__device__ __forceinline__ bool last_cta(unsigned* ctr) {
    __shared__ bool last;
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
        last = atomicAdd(ctr, 1u) == gridDim.x - 1;
        if (last) *ctr = 0u;
    }
    __syncthreads();
    return last;
}

__device__ __forceinline__ void release_sys(unsigned long long* p, unsigned long long v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__global__ void __launch_bounds__(kRingNT) k_ring_gather(RingArgs a) {
    extern __shared__ int so[];
    load_offsets(a, so);
    for (int i = blockIdx.x * kRingNT + threadIdx.x; i < a.n_total; i += gridDim.x * kRingNT) {
        const int p = ring_of(so, a.P, i);
        const RingTake& t = a.take[p];
        a.ev[i] = t.events[(t.base + static_cast<unsigned long long>(i - so[p])) & t.mask];
    }
    if (!last_cta(a.ctr)) return;
    for (int p = threadIdx.x; p < a.P; p += kRingNT) {
        const RingTake& t = a.take[p];
        if (t.n > 0) release_sys(t.tail, t.base + static_cast<unsigned long long>(t.n));
    }
}

__global__ void __launch_bounds__(kRingNT) k_ring_scatter(RingArgs a) {
    extern __shared__ int so[];
    load_offsets(a, so);
    const int stride = gridDim.x * kRingNT;
    for (int i = blockIdx.x * kRingNT + threadIdx.x; i < a.n_total; i += stride) {
        const int p = ring_of(so, a.P, i);
        const RingTake& t = a.take[p];
        if (t.flags) t.flags[(t.base + static_cast<unsigned long long>(i - so[p])) & t.mask] = a.rflags[i];
    }
    const int n4 = min(*a.count4, a.cap4);
    const int cols = a.cols;
    for (int k = blockIdx.x * kRingNT + threadIdx.x; k < n4 * cols; k += stride) {
        const int j = k / cols, r = k % cols;
        const int e = a.E4[j].e;
        const int p = ring_of(so, a.P, e);
        const RingTake& t = a.take[p];
        if (t.preds) {
            const unsigned long long slot = (t.base + static_cast<unsigned long long>(e - so[p])) & t.mask;
            t.preds[slot * cols + r] = a.head_dec[static_cast<size_t>(j) * cols + r];
        }
    }
    if (!last_cta(a.ctr)) return;
    for (int p = threadIdx.x; p < a.P; p += kRingNT) {
        const RingTake& t = a.take[p];
        if (t.n > 0) release_sys(t.done, t.base + static_cast<unsigned long long>(t.n));
    }
}

int ring_grid(int n) {
    const int g = (n + kRingNT - 1) / kRingNT;
    return g < 1 ? 1 : (g > 148 * 4 ? 148 * 4 : g);
}

}  // namespace

void launch_ring_gather(cudaStream_t st, const RingArgs& a) {
    k_ring_gather<<<ring_grid(a.n_total), kRingNT, sizeof(int) * (a.P + 1), st>>>(a);
}

void launch_ring_scatter(cudaStream_t st, const RingArgs& a) {
    k_ring_scatter<<<ring_grid(a.n_total), kRingNT, sizeof(int) * (a.P + 1), st>>>(a);
}

}  // namespace ssla
