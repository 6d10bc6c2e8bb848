// ssla_kernels.cu -- sm_100a kernels of the SSLA-S per-event hot path.
//
// One drain call processes a chunk of events for P independent partitions
// (ring partitions / camera streams).  Kernel sequence (ssla_engine.cu):
//   k_prep        validity + packed pixel coords per event
//   k_filter(s0)  ordered tile lists of the events around each 8x8 tile
//   k_gates       preprocess (dt_norm) + all four temporal-dropout gates +
//                 layer-0 qvg/residual, one warp per (partition, s3 block)
//   k_compact_*   stream-ordered stage lists E_1..E_4
//   k_filter(s1..s3)
//   per layer l:  k_scan (cell-major LRU update), k_contrib (the 9-owner goW
//                 contributions as a tiled FP32 GEMM per patch position),
//                 k_ln (ordered contribution sum + residual + LayerNorm),
//                 then k_gemm (the next layer's qvg) or k_head
//   k_commit      last head write per s3 cell -> predictions + version
// Reference behaviour each kernel reproduces is cited inline.
#include "ssla_kernels.cuh"

#include <cuda_runtime.h>

#include <algorithm>
#include <stdexcept>

#include "ssla_abi_types.h"

namespace ssla {

namespace {

__device__ __forceinline__ unsigned lanemask_lt() {
    unsigned m;
    asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
    return m;
}

__device__ __forceinline__ int hi_lane(unsigned m) { return 31 - __clz(m); }


// uint8 counter rule of tdrop_check_at (src/ssla_kernels.cpp:912-921) and
// parallel_tdrop (ssla_s2_s3_head_celled.cuh:742-745): pass iff window <= 1
// or the pre-increment count (mod 256) is a multiple of the window.
__device__ __forceinline__ bool gate_pass(int pre_count, int window) {
    if (window <= 1) return true;
    return ((pre_count & 255) % window) == 0;
}

// Warp-cooperative ordered gate over the lanes in `active` (stream order ==
// lane order).  `key` selects a counter in smem `cnt`; lanes not in `active`
// must pass a key unique to themselves.  Returns this lane's pass bit and
// advances the counters.
__device__ __forceinline__ bool warp_gate(bool active, int key, int* cnt, int window) {
    const unsigned peers = __match_any_sync(0xffffffffu, key);
    bool pass = false;
    if (active) pass = gate_pass(cnt[key] + __popc(peers & lanemask_lt()), window);
    __syncwarp();
    if (active && (threadIdx.x & 31) == hi_lane(peers)) cnt[key] += __popc(peers);
    __syncwarp();
    return pass;
}

}  // namespace

// ---------------------------------------------------------------------------
// k_prep: bounds rule of the drivers (s2_decomp_st.cpp:140-144,
// lib_stage01_to_gpu.cpp:210-214): int truncation then range check; written
// as float comparisons so NaN / huge values are rejected like on the host.
// ---------------------------------------------------------------------------
__global__ void k_prep(const float4* __restrict__ ev, int n, int W0, int H0,
                       uint32_t* __restrict__ ev_xy, uint8_t* __restrict__ rflags) {
    pdl_enter();
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const float4 e = ev[i];
        uint32_t xy = kInvalidXY;
        if (e.y > -1.0f && e.y < static_cast<float>(W0) && e.z > -1.0f && e.z < static_cast<float>(H0)) {
            const int x = static_cast<int>(e.y), y = static_cast<int>(e.z);
            xy = static_cast<uint32_t>(x) | (static_cast<uint32_t>(y) << 16);
        }
        ev_xy[i] = xy;
        rflags[i] = 0;
    }
}

// Stage-2 entry (drain_n): records -> E_2 identity list + packed coords.
__global__ void k_prep_records(const HybridInputRec* __restrict__ rec, int n,
                               StageEntry* __restrict__ E2, uint32_t* __restrict__ ev_xy,
                               uint8_t* __restrict__ rflags, float* __restrict__ feat) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const uint32_t x2 = rec[i].x, y2 = rec[i].y;
        const uint32_t xy0 = (x2 << 2) | ((y2 << 2) << 16);
        E2[i] = StageEntry{i, i, xy0};
        ev_xy[i] = xy0;
        rflags[i] = F_VALID | F_R1 | F_R2;
        for (int c = 0; c < 24; ++c) feat[static_cast<size_t>(i) * 24 + c] = rec[i].feat1[c];
    }
}

// ---------------------------------------------------------------------------
// k_filter (stage 0): for (partition, row of tiles, segment) compact, in
// stream order,
// the stage entries whose stage cell lies in each tile of the row grown by
// one cell (the entries whose 3x3 patch touches the tile).  Each entry is
// read once; it touches at most two tiles of the row, and its position in
// each tile's list is its rank among this chunk's hits of that tile (one
// ballot per tile).  grid (P, tile rows, segments).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kNT) k_filter(FilterArgs a) {
    pdl_enter();
    const int p = blockIdx.x, trow = a.trow0 + blockIdx.y, seg = blockIdx.z;
    const int s = a.stage;
    const int tx = a.g.tx[s];
    const int ntiles = tx * a.g.ty[s];
    const int lo = a.range[p], hi = a.range[p + 1];
    const int seg_lo = lo + seg * a.g.seg;
    if (seg_lo >= hi || seg >= a.g.nseg[s]) return;
    const int seg_hi = min(hi, seg_lo + a.g.seg);
    const int ty0 = trow * kTile;
    __shared__ int wc[kNT / 32][kMaxTileCols];
    __shared__ int run[kMaxTileCols];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (int t = tid; t < tx; t += kNT) run[t] = 0;
    for (int j0 = seg_lo; j0 < seg_hi; j0 += kNT) {
        const int j = j0 + tid;
        int t_lo = 1, t_hi = 0;                  // empty tile range
        int2 ent = make_int2(0, 0);
        if (j < seg_hi) {
            uint32_t xy0;
            uint32_t flag = 0;
            if (s == 0) {
                xy0 = a.ev_xy[j];
            } else {
                const StageEntry se = a.E[j];
                xy0 = se.xy0;
                flag = (a.rflags[se.e] & a.out_bit) ? 1u : 0u;
            }
            if (xy0 != kInvalidXY) {
                const int cx = static_cast<int>(xy0 & 0xFFFFu) >> s;
                const int cy = static_cast<int>(xy0 >> 16) >> s;
                if (cy >= ty0 - 1 && cy <= ty0 + kTile) {
                    t_lo = max(0, (cx - 1) >> 3);
                    t_hi = min(tx - 1, (cx + 1) >> 3);
                }
                ent = make_int2(j, static_cast<int>(static_cast<uint32_t>(cx) |
                                                    (static_cast<uint32_t>(cy) << 16) | (flag << 31)));
            }
        }
        int r_lo = 0, r_hi = 0;
        for (int t = 0; t < tx; ++t) {
            const unsigned m = __ballot_sync(0xffffffffu, t_lo <= t && t <= t_hi);
            if (lane == 0) wc[warp][t] = __popc(m);
            const int r = __popc(m & lanemask_lt());
            if (t == t_lo) r_lo = r;
            if (t == t_hi) r_hi = r;
        }
        __syncthreads();
        if (t_lo <= t_hi) {
#pragma unroll 2
            for (int q = 0; q < 2; ++q) {
                const int t = q ? t_hi : t_lo;
                if (q && t_hi == t_lo) break;
                int woff = 0;
                for (int w = 0; w < warp; ++w) woff += wc[w][t];
                const size_t slot = (static_cast<size_t>(p) * ntiles + trow * tx + t) * a.g.nseg[s] + seg;
                a.tl[slot * a.g.seg + run[t] + woff + (q ? r_hi : r_lo)] = ent;
            }
        }
        __syncthreads();
        for (int t = tid; t < tx; t += kNT) {
            int tot = 0;
#pragma unroll
            for (int w = 0; w < kNT / 32; ++w) tot += wc[w][t];
            run[t] += tot;
        }
    }
    __syncthreads();
    for (int t = tid; t < tx; t += kNT) {
        const size_t slot = (static_cast<size_t>(p) * ntiles + trow * tx + t) * a.g.nseg[s] + seg;
        a.tl_cnt[slot] = run[t];
    }
}

// ---------------------------------------------------------------------------
// k_filter_tiles: one CTA per (partition, tile, segment) -- the form for the
// small later stages, where a CTA per tile keeps enough CTAs busy: compacts,
// in stream order, the stage entries whose stage cell lies in the tile
// grown by one cell.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kNT) k_filter_tiles(FilterArgs a) {
    pdl_enter();
    const int p = blockIdx.x, tile = a.trow0 * a.g.tx[a.stage] + blockIdx.y, seg = blockIdx.z;
    const int s = a.stage;
    const int ntiles = a.g.tx[s] * a.g.ty[s];
    const int lo = a.range[p], hi = a.range[p + 1];
    const int seg_lo = lo + seg * a.g.seg;
    if (seg_lo >= hi || seg >= a.g.nseg[s]) return;
    const int seg_hi = min(hi, seg_lo + a.g.seg);
    const int tx0 = (tile % a.g.tx[s]) * kTile, ty0 = (tile / a.g.tx[s]) * kTile;
    const size_t slot = (static_cast<size_t>(p) * ntiles + tile) * a.g.nseg[s] + seg;
    int2* out = a.tl + slot * a.g.seg;
    __shared__ int warp_tot[kNT / 32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int running = 0;
    for (int j0 = seg_lo; j0 < seg_hi; j0 += kNT) {
        const int j = j0 + threadIdx.x;
        bool hit = false;
        int2 ent = make_int2(0, 0);
        if (j < seg_hi) {
            uint32_t xy0;
            uint32_t flag = 0;
            if (s == 0) {
                xy0 = a.ev_xy[j];
            } else {
                const StageEntry se = a.E[j];
                xy0 = se.xy0;
                flag = (a.rflags[se.e] & a.out_bit) ? 1u : 0u;
            }
            if (xy0 != kInvalidXY) {
                const int cx = static_cast<int>(xy0 & 0xFFFFu) >> s;
                const int cy = static_cast<int>(xy0 >> 16) >> s;
                hit = cx >= tx0 - 1 && cx <= tx0 + kTile && cy >= ty0 - 1 && cy <= ty0 + kTile;
                ent = make_int2(j, static_cast<int>(static_cast<uint32_t>(cx) |
                                                    (static_cast<uint32_t>(cy) << 16) | (flag << 31)));
            }
        }
        const unsigned m = __ballot_sync(0xffffffffu, hit);
        if (lane == 0) warp_tot[warp] = __popc(m);
        __syncthreads();
        int woff = 0, tot = 0;
#pragma unroll
        for (int w = 0; w < kNT / 32; ++w) {
            const int c = warp_tot[w];
            woff += (w < warp) ? c : 0;
            tot += c;
        }
        if (hit) out[running + woff + __popc(m & lanemask_lt())] = ent;
        running += tot;
        __syncthreads();
    }
    if (threadIdx.x == 0) a.tl_cnt[slot] = running;
}

// ---------------------------------------------------------------------------
// k_flag_s0: after the gates, sets bit 31 of every stage-0 tile-list entry
// whose event reaches stage 1 (its layer-1 output is consumed), so the
// layer-1 scan reads the flag with the entry instead of loading the event's
// flag byte behind it.  k_filter leaves the bit clear at stage 0.  One warp
// per (partition, tile, segment) slot, grid-stride.  Also zeroes the
// stage-0/1 scans' work counters (no memset node in the launch chain).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kNT) k_flag_s0(FilterArgs a) {
    pdl_enter();
    // the drain's layer-1..3 scans take work items from these counters
    if (a.zero_work && blockIdx.x == 0 && threadIdx.x < 8) a.zero_work[threadIdx.x] = 0;
    const int lane = threadIdx.x & 31;
    const int ntiles = a.g.tx[0] * a.g.ty[0];
    const long long per_p = static_cast<long long>(ntiles) * a.g.nseg[0];
    const long long slots = per_p * a.g.P;
    const long long wstride = (static_cast<long long>(gridDim.x) * blockDim.x) >> 5;
    for (long long w = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; w < slots; w += wstride) {
        const int p = static_cast<int>(w / per_p);
        const int seg = static_cast<int>(w % a.g.nseg[0]);
        const int n_p = a.range[p + 1] - a.range[p];
        if (seg >= (n_p + a.g.seg - 1) / a.g.seg) continue;        // segment not written this drain
        const int cnt = a.tl_cnt[w];
        int2* lst = a.tl + w * a.g.seg;
        for (int j = lane; j < cnt; j += 32) {
            const int2 e = lst[j];
            if (a.rflags[e.x] & F_R1) lst[j].y = e.y | static_cast<int>(0x80000000u);
        }
    }
}

// ---------------------------------------------------------------------------
// k_gates: one 4-warp CTA per (partition, s3 block).
//   Phase 1 (warp 0): walks the block's own events in stream order (the
//     stage-0 tile list of the block, two windows in flight) and computes
//       the previous timestamp of the event's pixel (preprocess,
//         src/ssla_kernels.cpp:288-309; the pixel's last_t advances),
//       gate 0 / 1 / 2 / 3 on the layout's grids (all cells of an event's
//         gates lie inside its s3 block, so the block owns every counter
//         it touches; same-key order inside a window from peer masks),
//     writing the event's flags and buffering (entry, pixel, rank among
//     the buffer's events at that pixel, previous t, t, p, pass0) of up to
//     kGateBuf events.
//   Phase 2 (all threads), layer 0 (K = 1: the event's own pixel,
//     layer_forward_ct, src/ssla_kernels.cpp:315-385):
//     a) per event: dt_norm, v and sigmoid(g) (matvec_ct<2,36> rows);
//     b) per (pixel, channel): the pixel's lru_step over its buffered
//        events in stream order, h after each event;
//     c) per event: q * h, goW contribution, residual, LayerNorm; writes
//        the output row and, for events entering stage 1, the layer-1
//        residual.
// ---------------------------------------------------------------------------
constexpr int kGateBuf = 256;
constexpr int kGateNT = 128;

__global__ void __launch_bounds__(kGateNT, 5) k_gates(GateArgs a) {
    const int p = blockIdx.x, blk = blockIdx.y;
    const int W3 = a.g.W[3];
    const int bx = blk % W3, by = blk / W3;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const PartState ps = a.parts[p];
    const bool hyb = a.g.layout == LAYOUT_HYBRID;
    // 16-byte stores of the layer-0 rows when both output arrays allow them
    const bool v16 = ((reinterpret_cast<uintptr_t>(a.X1) | reinterpret_cast<uintptr_t>(a.Rcopy)) & 15u) == 0;
    __shared__ double lt[64];
    __shared__ int c0[16], c1[4], c2[4], c3[1];
    __shared__ unsigned char passtab[256];
    // layer-0 weights: qvgT [2][36] | ipT [2][12] | goWT [12][12] | gamma | beta
    __shared__ float w0[264];
    __shared__ float h0[64 * 12];
    __shared__ double b_prev[kGateBuf];
    __shared__ float b_t[kGateBuf], b_p[kGateBuf], b_dt[kGateBuf];
    __shared__ int b_k[kGateBuf];
    __shared__ unsigned char b_pix[kGateBuf], b_rank[kGateBuf], b_pass0[kGateBuf];
    __shared__ float b_v[kGateBuf * 12], b_h[kGateBuf * 12];   // v; sigmoid(g) then h after
    __shared__ int pc[64], po[64];
    __shared__ unsigned char pl[kGateBuf];
    __shared__ int b_n, b_done;
    const int W0 = a.g.W[0], W1 = a.g.W[1], W2 = a.g.W[2];
    // The layer-0 weights are constant: loaded before the wait for the
    // previous kernel.  Every load of the set-up is issued before any store,
    // so the set-up costs one round trip, not one per array.
    {
        constexpr int NW = (264 + kGateNT - 1) / kGateNT;
        float wv[NW];
#pragma unroll
        for (int q = 0; q < NW; ++q) {
            const int t = tid + q * kGateNT;
            wv[q] = (t < 72) ? a.L0.qvgT[t] : (t < 96) ? a.L0.ipT[t - 72] : (t < 240) ? a.L0.goWT[t - 96]
                  : (t < 252) ? a.L0.gamma[t - 240] : (t < 264) ? a.L0.beta[t - 252] : 0.0f;
        }
#pragma unroll
        for (int q = 0; q < NW; ++q) {
            const int t = tid + q * kGateNT;
            if (t < 264) w0[t] = wv[q];
        }
    }
    for (int i = tid; i < 256; i += kGateNT) passtab[i] = gate_pass(i, a.g.window) ? 1 : 0;
    pdl_enter();
    {
        constexpr int NH = 64 * 12 / kGateNT;
        static_assert(64 * 12 % kGateNT == 0 && kGateNT >= 64, "gate set-up shape");
        float hv[NH];
#pragma unroll
        for (int q = 0; q < NH; ++q) {
            const int i = tid + q * kGateNT, px = i / 12, c = i % 12;
            hv[q] = ps.hidden[0][(static_cast<size_t>(by * 8 + px / 8) * W0 + bx * 8 + (px % 8)) * 12 + c];
        }
        double ltv = 0.0;
        if (tid < 64) ltv = ps.last_t[(by * 8 + tid / 8) * W0 + bx * 8 + (tid % 8)];
        int cv0 = 0, cv1 = 0, cv2 = 0, cv3 = 0;
        if (tid < 16) cv0 = ps.cnt[0][(by * 4 + tid / 4) * W1 + bx * 4 + (tid % 4)];
        if (tid < 4) cv1 = ps.cnt[1][(by * 2 + tid / 2) * W2 + bx * 2 + (tid % 2)];
        if (hyb) {
            if (tid < 4) cv2 = ps.cnt[2][(by * 2 + tid / 2) * W2 + bx * 2 + (tid % 2)];
            if (tid == 0) cv3 = ps.cnt[3][by * W3 + bx];
        } else if (tid == 0) {
            cv2 = ps.cnt[2][by * W3 + bx];
        }
#pragma unroll
        for (int q = 0; q < NH; ++q) h0[tid + q * kGateNT] = hv[q];
        if (tid < 64) { lt[tid] = ltv; pc[tid] = 0; }
        if (tid < 16) c0[tid] = cv0;
        if (tid < 4) c1[tid] = cv1;
        if (hyb) {
            if (tid < 4) c2[tid] = cv2;
            if (tid == 0) c3[0] = cv3;
        } else if (tid == 0) {
            c2[0] = cv2;
        }
    }
    __syncthreads();

    // Ordered gate over the active lanes of warp 0 (table lookup of the
    // tdrop rule; the counter advances by the number of active peers).
    // Peers = active lanes with the same BITS-bit key, from one ballot per
    // key bit.
    auto peers_of = [&](bool active, int key, int bits) {
        unsigned m = __ballot_sync(0xffffffffu, active);
        for (int b = 0; b < bits; ++b) {
            const bool bit = (key >> b) & 1;
            const unsigned bb = __ballot_sync(0xffffffffu, active && bit);
            m &= bit ? bb : ~bb;
        }
        return m;
    };
    auto gate = [&](bool active, int key, int bits, int* cnt) {
        const unsigned peers = peers_of(active, key, bits);
        bool pass = false;
        if (active) pass = passtab[(cnt[key] + __popc(peers & lanemask_lt())) & 255] != 0;
        __syncwarp();
        if (active && lane == hi_lane(peers)) cnt[key] += __popc(peers);
        __syncwarp();
        return pass;
    };

    const int ntiles = a.g.tx[0] * a.g.ty[0];
    const int tile = by * a.g.tx[0] + bx;     // s0 tiles are the s3 blocks
    const int n_p = a.ev_off[p + 1] - a.ev_off[p];
    const int nseg = min((n_p + a.g.seg - 1) / a.g.seg, a.g.nseg[0]);
    // Phase 1 reads the block's tile list in chunks of kGateChunk entries,
    // loaded by the whole CTA together with the events of the block's own
    // entries (one round trip for the entries, one for the events); warp 0
    // stages the own entries and runs the ordered gate windows from shared
    // memory.  The list arrives as segments; their counts are read
    // kGateChunk at a time and each chunk entry finds its segment by binary
    // search over their prefix.
    constexpr int kGateChunk = kGateNT;
    __shared__ int2 ch_ent[kGateChunk];
    __shared__ float4 ch_ev[kGateChunk];
    __shared__ int sw_pre[kGateChunk + 1];   // exclusive prefix of the window's segment counts
    __shared__ int sw_wsum[kGateNT / 32];
    __shared__ int ch_n, ch_pos, ph1_act;
    __shared__ int2 o_ent[64];               // own entries staged for the next gate windows
    __shared__ float4 o_ev[64];
    const size_t slot0 = (static_cast<size_t>(p) * ntiles + tile) * a.g.nseg[0];
    int sw0 = -kGateChunk, sw_tot = 0, gp = 0;   // CTA-uniform walk state
    bool list_done = false;
    auto is_own = [&](int2 ent) {
        const int x0 = ent.y & 0xFFFF, y0 = (ent.y >> 16) & 0x7FFF;
        return (x0 >> 3) == bx && (y0 >> 3) == by;
    };
    // all threads: the next chunk into ch_ent / ch_ev (ch_n = 0 once the list is done)
    auto load_chunk = [&]() {
        while (!list_done && gp >= sw_tot) {
            sw0 += kGateChunk;
            if (sw0 >= nseg) {
                list_done = true;
                break;
            }
            const int sg = sw0 + tid;
            int v = (sg < nseg) ? a.tl0_cnt[slot0 + sg] : 0;
            const int c = v;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, v, o);
                if (lane >= o) v += y;
            }
            if (lane == 31) sw_wsum[warp] = v;
            __syncthreads();
            int wo = 0, tot = 0;
#pragma unroll
            for (int w = 0; w < kGateNT / 32; ++w) {
                wo += (w < warp) ? sw_wsum[w] : 0;
                tot += sw_wsum[w];
            }
            sw_pre[tid] = wo + v - c;
            if (tid == 0) sw_pre[kGateChunk] = tot;
            __syncthreads();
            sw_tot = tot;
            gp = 0;
        }
        const int nld = list_done ? 0 : min(kGateChunk, sw_tot - gp);
        if (tid < nld) {
            const int q = gp + tid;
            int lo = 0, hi = kGateChunk;          // sw_pre[lo] <= q < sw_pre[hi]
            while (hi - lo > 1) {
                const int mid = (lo + hi) >> 1;
                if (sw_pre[mid] <= q) lo = mid;
                else hi = mid;
            }
            const int2 ent = a.tl0[(slot0 + sw0 + lo) * a.g.seg + (q - sw_pre[lo])];
            ch_ent[tid] = ent;
            ch_ev[tid] = is_own(ent) ? a.ev[ent.x] : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        gp += nld;
        if (tid == 0) {
            ch_n = nld;
            ch_pos = 0;
        }
        __syncthreads();
    };
    int o_n = 0;                             // warp 0: staged own entries
    enum { kNeedChunk = 0, kBufFull = 1, kListDone = 2 };
    load_chunk();

    for (;;) {
        // ---- phase 1: gates and previous timestamps, buffer the own events
        int nb = 0;                          // warp 0: events buffered for phase 2
        int act = kListDone;
        for (;;) {
          if (warp == 0) {
            int cp = ch_pos;
            const int cn = ch_n;
            for (;;) {
                // stage the chunk's own entries until a full window is ready
                while (o_n < 32 && cp < cn) {
                    const int j = cp + lane;
                    const int2 ce = (j < cn) ? ch_ent[j] : make_int2(0, 0);
                    const bool co = j < cn && is_own(ce);
                    const float4 cv = co ? ch_ev[j] : make_float4(0.f, 0.f, 0.f, 0.f);
                    const unsigned cm = __ballot_sync(0xffffffffu, co);
                    if (co) {
                        const int pos = o_n + __popc(cm & lanemask_lt());
                        o_ent[pos] = ce;
                        o_ev[pos] = cv;
                    }
                    o_n += __popc(cm);
                    cp += 32;
                }
                __syncwarp();
                if (nb > kGateBuf - 32) { act = kBufFull; break; }
                if (o_n < 32 && cp >= cn && !list_done) { act = kNeedChunk; break; }
                if (o_n == 0) { act = kListDone; break; }
                const int nw = min(o_n, 32);
                const bool own = lane < nw;
                const int2 ent = own ? o_ent[lane] : make_int2(0, 0);
                const float4 e = own ? o_ev[lane] : make_float4(0.f, 0.f, 0.f, 0.f);
                {   // the rest of the staged entries to the front
                    const bool mv = lane < o_n - nw;
                    const int2 te = mv ? o_ent[nw + lane] : make_int2(0, 0);
                    const float4 tv = mv ? o_ev[nw + lane] : make_float4(0.f, 0.f, 0.f, 0.f);
                    __syncwarp();
                    if (mv) { o_ent[lane] = te; o_ev[lane] = tv; }
                    __syncwarp();
                    o_n -= nw;
                }
                const unsigned om = __ballot_sync(0xffffffffu, own);
                if (om == 0u) continue;
                const int x0 = ent.y & 0xFFFF, y0 = (ent.y >> 16) & 0x7FFF;
                const int k = ent.x;
                const int pix = (y0 & 7) * 8 + (x0 & 7);
                const unsigned peers = peers_of(own, pix, 6);
                const unsigned prevm = peers & lanemask_lt();
                const int src = prevm ? hi_lane(prevm) : lane;
                const float t_prev_lane = __shfl_sync(0xffffffffu, e.x, src);
                double prev = 0.0;
                int rank = 0;
                if (own) {
                    prev = prevm ? static_cast<double>(t_prev_lane) : lt[pix];
                    rank = pc[pix] + __popc(prevm);
                }
                __syncwarp();
                if (own && lane == hi_lane(peers)) {
                    lt[pix] = static_cast<double>(e.x);
                    pc[pix] += __popc(peers);
                }
                __syncwarp();
                const int k0 = ((y0 >> 1) & 3) * 4 + ((x0 >> 1) & 3);
                const bool pass0 = gate(own, k0, 4, c0);
                const bool in1 = own && pass0;
                const int sub2 = ((y0 >> 2) & 1) * 2 + ((x0 >> 2) & 1);
                bool in2 = false, in3 = false, pass3 = true;
                if (__ballot_sync(0xffffffffu, in1)) {
                    const bool pass1 = gate(in1, sub2, 2, c1);
                    in2 = in1 && pass1;
                    if (a.n_gates > 2 && __ballot_sync(0xffffffffu, in2)) {
                        const bool pass2 = hyb ? gate(in2, sub2, 2, c2) : gate(in2, 0, 0, c2);
                        in3 = in2 && pass2;
                        if (hyb && __ballot_sync(0xffffffffu, in3)) pass3 = gate(in3, 0, 0, c3);
                    }
                }
                if (own) {
                    uint8_t f = F_VALID;
                    if (pass0) f |= F_R1;
                    if (in2) f |= F_R2;
                    if (in3) f |= F_R3;
                    if (in3 && pass3) f |= F_R4;
                    a.rflags[k] = f;
                    const int pos = nb + __popc(om & lanemask_lt());
                    b_k[pos] = k;
                    b_pix[pos] = static_cast<unsigned char>(pix);
                    b_rank[pos] = static_cast<unsigned char>(rank);
                    b_prev[pos] = prev;
                    b_t[pos] = e.x;
                    b_p[pos] = e.w;
                    b_pass0[pos] = pass0 ? 1 : 0;
                }
                nb += __popc(om);
            }
            if (lane == 0) { ch_pos = cp; ph1_act = act; }
          }
          __syncthreads();
          act = ph1_act;
          if (act == kNeedChunk) {
              load_chunk();
              continue;
          }
          break;
        }
        if (warp == 0) {
            if (lane == 0) { b_n = nb; b_done = (act == kListDone) ? 1 : 0; }
            // per-pixel list offsets of this buffer
            int c_lo = pc[2 * lane], c_hi = pc[2 * lane + 1];
            int incl = c_lo + c_hi;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += y;
            }
            po[2 * lane] = incl - c_lo - c_hi;
            po[2 * lane + 1] = incl - c_hi;
        }
        __syncthreads();
        const int n = b_n;
        const int done = b_done;
        // ---- phase 2a: per event dt_norm, v, sigmoid(g); pixel lists
        for (int i = tid; i < n; i += kGateNT) {
            const double prev = b_prev[i];
            float dt;
            if (prev < 0.0) {
                dt = 1.0f;
            } else {
                double v = (static_cast<double>(b_t[i]) - prev) / 1e5;
                if (v < 0.0) v = 0.0;
                if (v > 1.0) v = 1.0;
                dt = static_cast<float>(v);
            }
            const float ep = b_p[i];
            b_dt[i] = dt;
#pragma unroll 2
            for (int c = 0; c < 12; ++c) {
                b_v[i * 12 + c] = fmaf(w0[36 + 12 + c], ep, fmaf(w0[12 + c], dt, 0.0f));
                b_h[i * 12 + c] = ssla_sigmoidf(fmaf(w0[36 + 24 + c], ep, fmaf(w0[24 + c], dt, 0.0f)));
            }
            pl[po[b_pix[i]] + b_rank[i]] = static_cast<unsigned char>(i);
        }
        __syncthreads();
        // ---- phase 2b: the pixel chains, thread = (pixel, channel)
        for (int pr = tid; pr < 64 * 12; pr += kGateNT) {
            const int px = pr / 12, c = pr % 12;
            const int lo = po[px], m = pc[px];
            float h = h0[pr];
            for (int j = 0; j < m; ++j) {
                const int i = pl[lo + j];
                h = fmaf(b_h[i * 12 + c], h, b_v[i * 12 + c]);
                b_h[i * 12 + c] = h;
            }
            h0[pr] = h;
        }
        __syncthreads();
        // ---- phase 2c: per event q * h, goW, residual, LayerNorm
        for (int i = tid; i < n; i += kGateNT) {
            const float dt = b_dt[i], ep = b_p[i];
            float qh[12];
#pragma unroll
            for (int c = 0; c < 12; ++c) qh[c] = fmaf(w0[36 + c], ep, fmaf(w0[c], dt, 0.0f)) * b_h[i * 12 + c];
            float y[12];
            double sum = 0.0;
#pragma unroll 3
            for (int o = 0; o < 12; ++o) {
                float acc = 0.0f;
#pragma unroll
                for (int ii = 0; ii < 12; ++ii) acc = fmaf(w0[96 + ii * 12 + o], qh[ii], acc);
                y[o] = (0.0f + acc) + fmaf(w0[72 + 12 + o], ep, fmaf(w0[72 + o], dt, 0.0f));
                sum += static_cast<double>(y[o]);
            }
            const double mean = sum / 12.0;
            double var = 0.0;
#pragma unroll
            for (int o = 0; o < 12; ++o) {
                const double dd = static_cast<double>(y[o]) - mean;
                var += dd * dd;
            }
            var /= 12.0;
            const double inv = 1.0 / sqrt(var + static_cast<double>(1e-5f));
            const int k = b_k[i];
            float* xo = a.X1 + static_cast<size_t>(k) * 12;
            float* rc = (b_pass0[i] && a.Rcopy) ? a.Rcopy + static_cast<size_t>(k) * 12 : nullptr;
            float xv[12];
#pragma unroll
            for (int o = 0; o < 12; ++o) {
                const double t = (static_cast<double>(y[o]) - mean) * inv;
                xv[o] = static_cast<float>(t * static_cast<double>(w0[240 + o]) +
                                           static_cast<double>(w0[252 + o]));
            }
            // one event's row per thread: three 16-byte stores instead of
            // twelve scalar ones (each warp store touches 32 rows)
            if (v16) {
#pragma unroll
                for (int o = 0; o < 12; o += 4) {
                    const float4 v = make_float4(xv[o], xv[o + 1], xv[o + 2], xv[o + 3]);
                    *reinterpret_cast<float4*>(xo + o) = v;
                    if (rc) *reinterpret_cast<float4*>(rc + o) = v;
                }
            } else {
#pragma unroll
                for (int o = 0; o < 12; ++o) {
                    xo[o] = xv[o];
                    if (rc) rc[o] = xv[o];
                }
            }
        }
        __syncthreads();
        for (int i = tid; i < 64; i += kGateNT) pc[i] = 0;
        __syncthreads();
        if (done) break;
    }
    for (int i = tid; i < 64; i += kGateNT)
        ps.last_t[(by * 8 + i / 8) * W0 + bx * 8 + (i % 8)] = lt[i];
    for (int i = tid; i < 64 * 12; i += kGateNT) {
        const int px = i / 12, c = i % 12;
        ps.hidden[0][(static_cast<size_t>(by * 8 + px / 8) * W0 + bx * 8 + (px % 8)) * 12 + c] = h0[i];
    }
    if (tid < 16) ps.cnt[0][(by * 4 + tid / 4) * W1 + bx * 4 + (tid % 4)] = static_cast<uint8_t>(c0[tid]);
    if (tid < 4) ps.cnt[1][(by * 2 + tid / 2) * W2 + bx * 2 + (tid % 2)] = static_cast<uint8_t>(c1[tid]);
    if (hyb) {
        if (tid < 4) ps.cnt[2][(by * 2 + tid / 2) * W2 + bx * 2 + (tid % 2)] = static_cast<uint8_t>(c2[tid]);
        if (tid == 0) ps.cnt[3][by * W3 + bx] = static_cast<uint8_t>(c3[0]);
    } else if (tid == 0) {
        ps.cnt[2][by * W3 + bx] = static_cast<uint8_t>(c2[0]);
    }
}

// drain_n records entering at stage 2: tdrop_s2 (s2 grid) then, for the
// passing records, tdrop_s3 (s3 grid) -- ssla_s2_s3_head_celled.cuh:1020-1051.
// One warp per (partition, s3 cell); walks the stage-2 tile list holding it.
__global__ void __launch_bounds__(32) k_gates_s2(Gate2Args a) {
    const int p = blockIdx.x, cell = blockIdx.y;
    const int W3 = a.g.W[3], W2 = a.g.W[2];
    const int gx = cell % W3, gy = cell / W3;
    const int lane = threadIdx.x;
    const PartState ps = a.parts[p];
    const int window = a.g.window;
    __shared__ int c2[4], c3[1];
    if (lane < 4) c2[lane] = ps.cnt[2][(gy * 2 + lane / 2) * W2 + gx * 2 + (lane % 2)];
    if (lane == 0) c3[0] = ps.cnt[3][gy * W3 + gx];
    __syncwarp();
    const int ntiles = a.g.tx[2] * a.g.ty[2];
    const int tile = ((gy * 2) / kTile) * a.g.tx[2] + (gx * 2) / kTile;
    const int n_p = a.rec_off[p + 1] - a.rec_off[p];
    const int nseg = min((n_p + a.g.seg - 1) / a.g.seg, a.g.nseg[2]);
    for (int seg = 0; seg < nseg; ++seg) {
        const size_t slot = (static_cast<size_t>(p) * ntiles + tile) * a.g.nseg[2] + seg;
        const int cnt = a.tl2_cnt[slot];
        const int2* lst = a.tl2 + slot * a.g.seg;
        for (int j0 = 0; j0 < cnt; j0 += 32) {
            const int j = j0 + lane;
            int2 ent = make_int2(0, 0);
            if (j < cnt) ent = lst[j];
            const int x2 = ent.y & 0xFFFF, y2 = (ent.y >> 16) & 0x7FFF;
            const bool own = (j < cnt) && (x2 >> 1) == gx && (y2 >> 1) == gy;
            if (__ballot_sync(0xffffffffu, own) == 0u) continue;
            const int sub = (y2 & 1) * 2 + (x2 & 1);
            const bool p2 = warp_gate(own, own ? sub : 100 + lane, c2, window);
            const bool in3 = own && p2;
            const bool p3 = warp_gate(in3, in3 ? 0 : 100 + lane, c3, window);
            if (own) {
                uint8_t f = F_VALID | F_R1 | F_R2;
                if (p2) f |= F_R3;
                if (in3 && p3) f |= F_R4;
                a.rflags[ent.x] = f;
            }
        }
    }
    __syncwarp();
    if (lane < 4) ps.cnt[2][(gy * 2 + lane / 2) * W2 + gx * 2 + (lane % 2)] = static_cast<uint8_t>(c2[lane]);
    if (lane == 0) ps.cnt[3][gy * W3 + gx] = static_cast<uint8_t>(c3[0]);
}

// ---------------------------------------------------------------------------
// Stage-list compaction (stream order) of the events whose reach bit R_s is
// set, for lists s_first+1 .. 4.  Compaction tiles never straddle partitions.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kNT) k_compact_count(CompactArgs a) {
    pdl_enter();
    const int p = blockIdx.x, t = blockIdx.y;
    const int lo = a.ev_off[p] + t * a.ctile;
    const int hi = min(a.ev_off[p + 1], lo + a.ctile);
    int c[4] = {0, 0, 0, 0};
    for (int i = lo + static_cast<int>(threadIdx.x); i < hi; i += kNT) {
        const uint8_t f = a.rflags[i];
#pragma unroll
        for (int s = 0; s < 4; ++s) c[s] += (f >> (s + 1)) & 1;
    }
    __shared__ int red[kNT / 32][4];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int s = 0; s < 4; ++s) {
        int v = c[s];
        for (int o = 16; o > 0; o >>= 1) v += __shfl_down_sync(0xffffffffu, v, o);
        if (lane == 0) red[warp][s] = v;
    }
    __syncthreads();
    if (threadIdx.x < 4) {
        int v = 0;
        for (int w = 0; w < kNT / 32; ++w) v += red[w][threadIdx.x];
        a.tilecnt[(static_cast<size_t>(p) * a.tiles_per_part + t) * 4 + threadIdx.x] = v;
    }
}

__global__ void __launch_bounds__(kNT) k_compact_scan(CompactArgs a) {
    pdl_enter();
    const int n = a.g.P * a.tiles_per_part;
    __shared__ int carry[4];
    __shared__ int wsum[kNT / 32][4];
    if (threadIdx.x < 4) carry[threadIdx.x] = 0;
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int b0 = 0; b0 < n; b0 += kNT) {
        const int i = b0 + threadIdx.x;
        int v[4];
#pragma unroll
        for (int s = 0; s < 4; ++s) v[s] = (i < n) ? a.tilecnt[static_cast<size_t>(i) * 4 + s] : 0;
        int incl[4];
#pragma unroll
        for (int s = 0; s < 4; ++s) {
            int x = v[s];
            for (int o = 1; o < 32; o <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, x, o);
                if (lane >= o) x += y;
            }
            incl[s] = x;
            if (lane == 31) wsum[warp][s] = x;
        }
        __syncthreads();
#pragma unroll
        for (int s = 0; s < 4; ++s) {
            int wo = 0, tot = 0;
            for (int w = 0; w < kNT / 32; ++w) {
                wo += (w < warp) ? wsum[w][s] : 0;
                tot += wsum[w][s];
            }
            if (i < n) a.tilebase[static_cast<size_t>(i) * 4 + s] = carry[s] + wo + incl[s] - v[s];
            __syncthreads();
            if (threadIdx.x == 0) carry[s] += tot;
            __syncthreads();
        }
    }
    if (threadIdx.x < 4) {
        const int s = threadIdx.x + 1;
        if (s > a.s_first) {
            for (int p = 0; p < a.g.P; ++p)
                a.off[s][p] = min(a.tilebase[(static_cast<size_t>(p) * a.tiles_per_part) * 4 + threadIdx.x],
                                  a.g.cap[s]);
            a.off[s][a.g.P] = min(carry[threadIdx.x], a.g.cap[s]);
            a.count[s] = min(carry[threadIdx.x], a.g.cap[s]);
        }
    }
}

__global__ void __launch_bounds__(kNT) k_compact_scatter(CompactArgs a) {
    pdl_enter();
    const int p = blockIdx.x, t = blockIdx.y;
    const int lo = a.ev_off[p] + t * a.ctile;
    const int hi = min(a.ev_off[p + 1], lo + a.ctile);
    if (lo >= hi) return;
    __shared__ int wtot[kNT / 32][4];
    __shared__ int run[4];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (threadIdx.x < 4)
        run[threadIdx.x] = a.tilebase[(static_cast<size_t>(p) * a.tiles_per_part + t) * 4 + threadIdx.x];
    __syncthreads();
    for (int j0 = lo; j0 < hi; j0 += kNT) {
        const int i = j0 + threadIdx.x;
        const uint8_t f = (i < hi) ? a.rflags[i] : 0;
        unsigned m[4];
#pragma unroll
        for (int s = 0; s < 4; ++s) {
            m[s] = __ballot_sync(0xffffffffu, (f >> (s + 1)) & 1);
            if (lane == 0) wtot[warp][s] = __popc(m[s]);
        }
        __syncthreads();
        int pos[4];
#pragma unroll
        for (int s = 0; s < 4; ++s) {
            int wo = 0;
            for (int w = 0; w < warp; ++w) wo += wtot[w][s];
            pos[s] = run[s] + wo + __popc(m[s] & lanemask_lt());
        }
        if (i < hi) {
            const uint32_t xy0 = a.ev_xy[i];
            int prev = i;                           // E_0 index == event index
#pragma unroll
            for (int s = 0; s < 4; ++s) {
                const int list = s + 1;
                if ((f >> list) & 1) {
                    if (list > a.s_first && pos[s] < a.g.cap[list])
                        a.E[list][pos[s]] = StageEntry{i, prev, xy0};
                    prev = (list > a.s_first) ? pos[s] : i;
                }
            }
        }
        __syncthreads();
        if (threadIdx.x < 4) {
            int tot = 0;
            for (int w = 0; w < kNT / 32; ++w) tot += wtot[w][threadIdx.x];
            run[threadIdx.x] += tot;
        }
        __syncthreads();
    }
}

// ---------------------------------------------------------------------------
// k_scan: one warp per (partition, cell) of the layer's grid, 8 cells per CTA.
// Walks, in stream order, the tile-list entries whose 3x3 patch covers the
// cell (only the cell itself for the K=1 layer) and applies lru_step
// (vendor/openeva/prim/rnn.h:80-91): h = sigmoid(g) * h + v (fmaf), and
// q -> q * h for entries whose layer output is consumed.  Lanes own
// channels; hidden state stays in registers for the whole chunk.
// The CTA stages the tile list through shared memory in rounds of 512
// entries, the next round's loads issued before the current round is
// walked, so a warp's walk reads shared memory instead of waiting on an L2
// round trip per 32 entries; hits are applied HP at a time with their rows'
// loads issued ahead of the fmaf chain.
// grid (P, tiles, 8), block 256.
// ---------------------------------------------------------------------------
template <int A, int OUT>
__global__ void __launch_bounds__(kNT, 2) k_scan(ScanArgs a) {
    pdl_enter();
    constexpr int CPL = (OUT + 31) / 32;
    constexpr int HP = 4;                                 // hits per batch (two batches in flight)
    constexpr int kChunk = 2 * kNT;                       // list entries per staged round
    __shared__ int2 sl[kChunk];
    __shared__ int hq_all[kNT / 32][kChunk];              // per warp: its cell's hits of a round
    const int p = blockIdx.x, tile = blockIdx.y;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int s = a.stage;
    const int local = blockIdx.z * (kNT / 32) + warp;     // 0..63 in the tile
    int* const hq = hq_all[warp];
    const int cx = (tile % a.g.tx[s]) * kTile + (local % kTile);
    const int cy = (tile / a.g.tx[s]) * kTile + (local / kTile);
    const int Wl = a.g.W[s], Hl = a.g.H[s];
    const bool active = cx < Wl && cy < Hl && cy >= a.g.row_lo[s] && cy < a.g.row_hi[s];
    if (!__syncthreads_or(active)) return;                // CTA-uniform
    float* hp = a.parts[p].hidden[a.layer] + (static_cast<size_t>(active ? cy : 0) * Wl + (active ? cx : 0)) * OUT;
    float h[CPL];
#pragma unroll
    for (int c = 0; c < CPL; ++c) {
        const int o = lane + 32 * c;
        h[c] = (active && o < OUT) ? hp[o] : 0.0f;
    }
    const int ntiles = a.g.tx[s] * a.g.ty[s];
    const int n_p = a.range[p + 1] - a.range[p];
    const int nseg = min((n_p + a.g.seg - 1) / a.g.seg, a.g.nseg[s]);
    float* __restrict__ S = a.S;
    for (int seg = 0; seg < nseg; ++seg) {
        const size_t slot = (static_cast<size_t>(p) * ntiles + tile) * a.g.nseg[s] + seg;
        const int cnt = a.tl_cnt[slot];
        const int2* lst = a.tl + slot * a.g.seg;
        int2 pre0 = make_int2(0, 0), pre1 = make_int2(0, 0);
        if (static_cast<int>(threadIdx.x) < cnt) pre0 = lst[threadIdx.x];
        if (static_cast<int>(threadIdx.x) + kNT < cnt) pre1 = lst[threadIdx.x + kNT];
        for (int c0 = 0; c0 < cnt; c0 += kChunk) {
            __syncthreads();                              // the previous round is consumed
            sl[threadIdx.x] = pre0;
            sl[threadIdx.x + kNT] = pre1;
            __syncthreads();
            {                                             // next round's loads, in flight during the walk
                const int i0 = c0 + kChunk + static_cast<int>(threadIdx.x);
                pre0 = (i0 < cnt) ? lst[i0] : make_int2(0, 0);
                pre1 = (i0 + kNT < cnt) ? lst[i0 + kNT] : make_int2(0, 0);
            }
            if (!active) continue;
            const int nch = min(kChunk, cnt - c0);
            // 1) the cell's hits of this round, in list order: (row << 1) | output flag
            int nq = 0;
            for (int j0 = 0; j0 < nch; j0 += 32) {
                const int j = j0 + lane;
                int2 ent = make_int2(0, 0);
                if (j < nch) ent = sl[j];
                const int ex = ent.y & 0xFFFF, ey = (ent.y >> 16) & 0x7FFF;
                const int dx = cx - ex, dy = cy - ey;
                bool hit;
                if (A == 1) hit = (j < nch) && dx == 0 && dy == 0;
                else hit = (j < nch) && dx >= -1 && dx <= 1 && dy >= -1 && dy <= 1;
                const int delta = (A == 1) ? 0 : (1 - dy) * 3 + (1 - dx);    // ssla_kernels.cpp:375
                int outf = 1;
                if (a.second) {
                    if (s == 0) outf = (hit && (a.rflags[ent.x] & F_R1)) ? 1 : 0;
                    else outf = (static_cast<uint32_t>(ent.y) >> 31) & 1;
                }
                const unsigned m = __ballot_sync(0xffffffffu, hit);
                if (hit) hq[nq + __popc(m & lanemask_lt())] = ((ent.x * A + delta) << 1) | outf;
                nq += __popc(m);
            }
            __syncwarp();
            // 2) applied HP at a time; the next batch's rows load while this
            //    batch's fmaf chain runs
            float qv[2][HP][CPL], vv[2][HP][CPL], av[2][HP][CPL];
            int row[2][HP], of[2][HP];
            auto fetch = [&](int buf, int b0) {
#pragma unroll
                for (int q = 0; q < HP; ++q) {
                    const bool on = b0 + q < nq;
                    const int v = on ? hq[b0 + q] : 0;
                    row[buf][q] = v >> 1;
                    of[buf][q] = on ? (v & 1) : 0;
                    const float* r = S + static_cast<size_t>(row[buf][q]) * (3 * OUT);
#pragma unroll
                    for (int c = 0; c < CPL; ++c) {
                        const int o = lane + 32 * c;
                        const bool ok = on && (o < OUT);
                        qv[buf][q][c] = (ok && of[buf][q]) ? r[o] : 0.0f;
                        vv[buf][q][c] = ok ? r[OUT + o] : 0.0f;
                        av[buf][q][c] = ok ? r[2 * OUT + o] : 0.0f;
                    }
                }
            };
            auto apply = [&](int buf, int b0) {
#pragma unroll
                for (int q = 0; q < HP; ++q) {
                    if (b0 + q < nq) {
                        float* r = S + static_cast<size_t>(row[buf][q]) * (3 * OUT);
#pragma unroll
                        for (int c = 0; c < CPL; ++c) {
                            const int o = lane + 32 * c;
                            if (o < OUT) {
                                h[c] = fmaf(av[buf][q][c], h[c], vv[buf][q][c]);
                                if (of[buf][q]) r[o] = qv[buf][q][c] * h[c];
                            }
                        }
                    }
                }
            };
            if (nq > 0) fetch(0, 0);
            for (int b0 = 0; b0 < nq; b0 += 2 * HP) {
                if (b0 + HP < nq) fetch(1, b0 + HP);
                apply(0, b0);
                if (b0 + HP < nq) {
                    if (b0 + 2 * HP < nq) fetch(0, b0 + 2 * HP);
                    apply(1, b0 + HP);
                }
            }
            __syncwarp();
        }
    }
    if (active) {
#pragma unroll
        for (int c = 0; c < CPL; ++c) {
            const int o = lane + 32 * c;
            if (o < OUT) hp[o] = h[c];
        }
    }
}

// ---------------------------------------------------------------------------
// k_hot_tiles: one CTA lists, in ascending order, the (partition, tile)
// pairs of a stage whose tile lists hold more than a.threshold entries.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(1024) k_hot_tiles(HotArgs a) {
    pdl_enter();
    const int s = a.stage;
    const int ntiles = a.g.tx[s] * a.g.ty[s];
    const int total = a.g.P * ntiles;
    __shared__ int wsum[32];
    __shared__ int run;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (threadIdx.x == 0) run = 0;
    __syncthreads();
    for (int t0 = 0; t0 < total; t0 += 1024) {
        const int t = t0 + static_cast<int>(threadIdx.x);
        bool hot = false;
        if (t < total) {
            const int p = t / ntiles;
            const int n_p = a.range[p + 1] - a.range[p];
            const int nseg = min((n_p + a.g.seg - 1) / a.g.seg, a.g.nseg[s]);
            int sum = 0;
            for (int sg = 0; sg < nseg; ++sg) sum += a.tl_cnt[static_cast<size_t>(t) * a.g.nseg[s] + sg];
            hot = sum > a.threshold;
            a.hot_flag[t] = hot ? 1 : 0;
        }
        const unsigned m = __ballot_sync(0xffffffffu, hot);
        if (lane == 0) wsum[warp] = __popc(m);
        __syncthreads();
        int before = 0, tot = 0;
        for (int w = 0; w < 32; ++w) {
            before += (w < warp) ? wsum[w] : 0;
            tot += wsum[w];
        }
        if (hot) a.hot[1 + run + before + __popc(m & lanemask_lt())] = t;
        __syncthreads();
        if (threadIdx.x == 0) run += tot;
        __syncthreads();
    }
    if (threadIdx.x == 0) a.hot[0] = run;
}

// ---------------------------------------------------------------------------
// k_scan_group: per-cell LRU scan of a small layer (layers 1-3: IN, OUT <= 24,
// the 9 x IN x 3*OUT qvg weights fit in shared memory) fused with that
// layer's qvg matvec (matvec_ct<IN,3*OUT>, linear.h:80-90).
// Work item = (partition, 8x8 tile, GX x GY cell group: 4x2 for layer 1,
// 2x2 for layers 2-3), taken by one warp from
// an atomic counter; warps never wait on one another.  When the group items
// are fewer than the resident warps (one clustered stream, a strip of a
// large sensor), tiles whose lists exceed kHotTileEntries are listed by
// k_hot_tiles and scanned with one item per cell instead, after the group
// items: four times the parallelism where few tiles hold the drain.  With
// items to spare, splitting would only repeat each tile's list walk.  The warp walks the
// tile's ordered event list and queues, in stream order, one slot per
// (event, cell of the group inside the event's 3x3 patch).  Per 32 slots:
//   B) lane = slot: v and sigmoid(g) as fmaf chains over the input channels
//      (weights from shared memory, delta rows padded to distinct banks);
//   C) lane = (cell, channel): the cell's slots in order apply
//      h = a * h + v (fmaf); after a slot whose output is consumed the
//      state goes to the compact rows QH[(entry * 9 + delta) * OUT], where
//      k_contrib forms q and q * h.
// One owner per cell, no atomics on state; results equal the per-event
// reference (fmaf order over input channels, sigmoid, fmaf update).
// ---------------------------------------------------------------------------
template <int IN, int OUT, int WPC, int GX, int GY>
struct ScanGroupShape {
    static constexpr int NT = 32 * WPC;
    static constexpr int NCELL = GX * GY;               // cells of a group item
    static constexpr int GPT = (kTile / GX) * (kTile / GY);   // group items per tile
    static constexpr int HMAX = (GX < 3 ? GX : 3) * (GY < 3 ? GY : 3);   // hits of one entry at most
    static constexpr int J2 = 3 * OUT;
    static constexpr int DS = IN * J2 + ((IN * J2) % 32 == 16 ? 4 : ((IN * J2) % 32 == 0 ? 4 : 0));
    static constexpr int QR = ((2 * OUT / 4) % 2 == 0) ? 2 * OUT + 4 : 2 * OUT;   // [a | v] row
    static constexpr int QCAP = 32 + 32 * HMAX;         // < 32 pending + 32 entries x HMAX hits
    static constexpr int G4 = OUT / 4;                  // 4-channel slices of a cell (update lanes per cell)
    static constexpr size_t per_warp = sizeof(float) * 32 * QR + (sizeof(int) + 1) * QCAP + 32 + sizeof(int2) * 64;
    static constexpr size_t smem = sizeof(float) * 9 * DS + WPC * per_warp;
    static_assert(IN % 4 == 0 && OUT % 4 == 0 && DS % 4 == 0 && NCELL <= 8 && NCELL * G4 <= 32 &&
                  kTile % GX == 0 && kTile % GY == 0 && (32 * QR + QCAP + QCAP / 4 + 8 + 128) % 4 == 0 &&
                  (QCAP + 32) % 8 == 0, "shape");
};

template <int IN, int OUT, int WPC, int GX, int GY>
__global__ void __launch_bounds__(32 * WPC, WPC == 8 ? 3 : 1) k_scan_group(ScanFusedArgs a) {
    using Sh = ScanGroupShape<IN, OUT, WPC, GX, GY>;
    constexpr int J2 = Sh::J2, DS = Sh::DS, QR = Sh::QR, QCAP = Sh::QCAP, G4 = Sh::G4;
    constexpr int NCELL = Sh::NCELL, GPT = Sh::GPT;
    extern __shared__ __align__(16) float dsm[];
    float* Ws = dsm;                                              // [9][DS]
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    float* Qs = Ws + 9 * DS + warp * (Sh::per_warp / sizeof(float));   // [32][QR]
    int* qk = reinterpret_cast<int*>(Qs + 32 * QR);                    // [QCAP] entry
    unsigned char* qm = reinterpret_cast<unsigned char*>(qk + QCAP);    // [QCAP] delta | cell<<4 | out<<7
    unsigned char* perm = qm + QCAP;                                    // [32] batch lane -> slot
    int2* rbuf = reinterpret_cast<int2*>(perm + 32);                    // [64] relevant list entries
    // the weights are constant: staged before the wait, every load issued
    // before the stores (one round trip)
    {
        constexpr int N4 = 9 * IN * J2 / 4, PT = (N4 + Sh::NT - 1) / Sh::NT;
        float4 v[PT];
#pragma unroll
        for (int q = 0; q < PT; ++q) {
            const int t = threadIdx.x + q * Sh::NT;
            if (t < N4) v[q] = __ldg(reinterpret_cast<const float4*>(a.W) + t);
        }
#pragma unroll
        for (int q = 0; q < PT; ++q) {
            const int t = threadIdx.x + q * Sh::NT;
            if (t < N4) {
                const int d = t / (IN * J2 / 4), r = t % (IN * J2 / 4);
                *reinterpret_cast<float4*>(Ws + d * DS + 4 * r) = v[q];
            }
        }
    }
    pdl_wait();
    __syncthreads();
    const int s = a.stage;
    const int Wl = a.g.W[s], Hl = a.g.H[s];
    const int ntiles = a.g.tx[s] * a.g.ty[s];
    const int n_groups = a.g.P * ntiles * GPT;
    const int n_items = n_groups + (a.hot ? a.hot[0] * 64 : 0);
    float* const QH = a.QH;
    for (;;) {
        int item = 0;
        if (lane == 0) item = atomicAdd(a.work, 1);
        item = __shfl_sync(0xffffffffu, item, 0);
        if (item >= n_items) break;
        int p, tile, gx0, gy0, ncell;
        if (item < n_groups) {
            const int grp = item % GPT;
            tile = (item / GPT) % ntiles;
            p = (item / GPT) / ntiles;
            if (a.hot_flag && a.hot_flag[p * ntiles + tile]) continue;      // scanned cell by cell
            gx0 = (tile % a.g.tx[s]) * kTile + (grp % (kTile / GX)) * GX;
            gy0 = (tile / a.g.tx[s]) * kTile + (grp / (kTile / GX)) * GY;
            ncell = NCELL;
        } else {
            const int h = (item - n_groups) >> 6, cell = (item - n_groups) & 63;
            const int pt = a.hot[1 + h];
            tile = pt % ntiles;
            p = pt / ntiles;
            gx0 = (tile % a.g.tx[s]) * kTile + (cell & 7);
            gy0 = (tile / a.g.tx[s]) * kTile + (cell >> 3);
            ncell = 1;
        }
        if (gx0 >= Wl || gy0 >= Hl || gy0 + (ncell > 1 ? GY - 1 : 0) < a.g.row_lo[s] || gy0 >= a.g.row_hi[s]) continue;
        float* const hid = a.parts[p].hidden[a.layer];
        // update role: lane = (cell cc of the group, 4-channel slice g)
        const int cc = lane / G4, g4 = lane % G4;
        const int ux = gx0 + cc % GX, uy = gy0 + cc / GX;
        const bool uown = lane < NCELL * G4 && cc < ncell && ux < Wl && uy < Hl;
        // the group's cells inside the grid (bit c: cell (c % GX, c / GX))
        unsigned vmask = 0;
#pragma unroll
        for (int c = 0; c < NCELL; ++c)
            if (c < ncell && gx0 + c % GX < Wl && gy0 + c / GX < Hl) vmask |= 1u << c;
        float* const hp = hid + (static_cast<size_t>(uown ? uy : 0) * Wl + (uown ? ux : 0)) * OUT + 4 * g4;
        float4 h4 = uown ? *reinterpret_cast<const float4*>(hp) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        int np = 0;                                   // queued slots (warp-uniform)
        // Runs B, C, D on the first nb (1..32) queued slots.
        auto batch = [&](int nb) {
            // cell and output masks over the slots (bit = slot)
            const bool valid = lane < nb;
            const int m0 = qm[valid ? lane : 0];
            unsigned mk_own = 0;                  // this lane's update cell: its slots
#pragma unroll
            for (int c = 0; c < NCELL; ++c) {
                const unsigned b = __ballot_sync(0xffffffffu, valid && ((m0 >> 4) & 7) == c);
                if (cc == c) mk_own = b;
            }
            const unsigned om = __ballot_sync(0xffffffffu, valid && ((m0 >> 7) & 1));
            // B runs the slots sorted by delta (counting sort, one ballot per
            // delta), so the lanes of a weight read mostly share one row
            {
                const int d0 = valid ? (m0 & 15) : 9;
                const unsigned lt = lanemask_lt();
                int pos = 0, before = 0;
#pragma unroll
                for (int dd = 0; dd <= 9; ++dd) {
                    const unsigned mk = __ballot_sync(0xffffffffu, d0 == dd);
                    if (d0 == dd) pos = before + __popc(mk & lt);
                    before += __popc(mk);
                }
                perm[pos] = static_cast<unsigned char>(lane);
                __syncwarp();
            }
            const int sl = perm[lane];
            const int k = qk[valid ? sl : 0];
            const int d = qm[valid ? sl : 0] & 15;
            float x[IN];
#pragma unroll
            for (int i4 = 0; i4 < IN / 4; ++i4) {
                const float4 t = __ldg(reinterpret_cast<const float4*>(a.X + static_cast<size_t>(k) * IN) + i4);
                x[4 * i4] = t.x; x[4 * i4 + 1] = t.y; x[4 * i4 + 2] = t.z; x[4 * i4 + 3] = t.w;
            }
            const float* wr = Ws + d * DS;
            float* qr = Qs + sl * QR;
            float2 acc[OUT / 2];
            // B: a = sigmoid(g) -> [0, OUT), v -> [OUT, 2*OUT); paired
            // output channels per packed FMA (each component an fmaf)
#pragma unroll
            for (int part = 2; part >= 1; --part) {
#pragma unroll
                for (int j = 0; j < OUT / 2; ++j) acc[j] = make_float2(0.0f, 0.0f);
#pragma unroll
                for (int i = 0; i < IN; ++i) {
                    const float2 xx = make_float2(x[i], x[i]);
#pragma unroll
                    for (int j4 = 0; j4 < OUT / 4; ++j4) {
                        const float4 w4 = *reinterpret_cast<const float4*>(wr + i * J2 + part * OUT + 4 * j4);
                        acc[2 * j4] = __ffma2_rn(make_float2(w4.x, w4.y), xx, acc[2 * j4]);
                        acc[2 * j4 + 1] = __ffma2_rn(make_float2(w4.z, w4.w), xx, acc[2 * j4 + 1]);
                    }
                }
                if (part == 2) {
#pragma unroll
                    for (int j = 0; j < OUT / 2; ++j)
                        acc[j] = ssla_sigmoidf2(acc[j]);
                }
                const int col = (part == 2) ? 0 : OUT;
#pragma unroll
                for (int j4 = 0; j4 < OUT / 4; ++j4)
                    *reinterpret_cast<float4*>(qr + col + 4 * j4) =
                        make_float4(acc[2 * j4].x, acc[2 * j4].y, acc[2 * j4 + 1].x, acc[2 * j4 + 1].y);
            }
            __syncwarp();
            // C: ordered updates, lane = (cell, 4 channels); four hits per
            // round, their rows' loads issued ahead of the fmaf chain
            {
                unsigned mk = uown ? mk_own : 0u;
                float2 hlo = make_float2(h4.x, h4.y), hhi = make_float2(h4.z, h4.w);
                while (mk) {
                    int s4[4];
                    bool on[4];
                    float4 av[4], vv[4];
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        on[q] = mk != 0u;
                        s4[q] = on[q] ? __ffs(mk) - 1 : 0;
                        mk &= mk - 1u;
                        const float* q2 = Qs + s4[q] * QR + 4 * g4;
                        av[q] = *reinterpret_cast<const float4*>(q2);
                        vv[q] = *reinterpret_cast<const float4*>(q2 + OUT);
                    }
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        if (!on[q]) break;
                        // h = a * h + v per channel (each component one fmaf)
                        hlo = __ffma2_rn(make_float2(av[q].x, av[q].y), hlo, make_float2(vv[q].x, vv[q].y));
                        hhi = __ffma2_rn(make_float2(av[q].z, av[q].w), hhi, make_float2(vv[q].z, vv[q].w));
                        if ((om >> s4[q]) & 1u)
                            *reinterpret_cast<float4*>(QH + (static_cast<size_t>(qk[s4[q]]) * 9 + (qm[s4[q]] & 15)) * OUT +
                                                       4 * g4) = make_float4(hlo.x, hlo.y, hhi.x, hhi.y);
                    }
                }
                h4 = make_float4(hlo.x, hlo.y, hhi.x, hhi.y);
            }
            __syncwarp();
        };
        // The tile list arrives as segments; their counts are read 32 at a
        // time (lane i: segment wbase + i) and each 32-entry block's load is
        // issued one block ahead of its walk.
        const int n_p = a.range[p + 1] - a.range[p];
        const int nseg = min((n_p + a.g.seg - 1) / a.g.seg, a.g.nseg[s]);
        const size_t slot0 = (static_cast<size_t>(p) * ntiles + tile) * a.g.nseg[s];
        int wbase = -32, wcnt = 0;
        auto seg_cnt = [&](int sg) -> int {         // warp-uniform, non-decreasing sg
            if (sg >= nseg) return 0;
            if (sg >= wbase + 32) {
                wbase = sg & ~31;
                wcnt = (wbase + lane < nseg) ? a.tl_cnt[slot0 + wbase + lane] : 0;
            }
            return __shfl_sync(0xffffffffu, wcnt, sg - wbase);
        };
        auto load_block = [&](int sg, int j0, int cnt) -> int2 {
            return (sg < nseg && j0 + lane < cnt) ? a.tl[(slot0 + sg) * a.g.seg + j0 + lane] : make_int2(0, 0);
        };
        // Hits of up to 32 relevant entries (rbuf[0, nrel)) into the slot queue,
        // batches of 32 slots run as the queue fills.
        auto queue_hits = [&](int nrel) {
            const bool on = lane < nrel;
            const int2 ent = on ? rbuf[lane] : make_int2(0, 0);
            const int ex = ent.y & 0xFFFF, ey = (ent.y >> 16) & 0x7FFF;
            // cells of the group inside the entry's 3x3 patch: cell (i, j)
            // is hit iff i in [rx - 2, rx] and j in [ry - 2, ry], with (rx, ry)
            // the entry's position relative to the group's corner (-1, -1)
            const int rx = ex - gx0 + 1, ry = ey - gy0 + 1;
            unsigned cmask = 0;
            if (on) {
                const int xl = max(rx - 2, 0), xh = min(rx, GX - 1);
                const int yl = max(ry - 2, 0), yh = min(ry, GY - 1);
                const unsigned xm = (xh >= xl) ? (((2u << xh) - 1u) & ~((1u << xl) - 1u)) : 0u;
#pragma unroll
                for (int jy = 0; jy < GY; ++jy)
                    if (jy >= yl && jy <= yh) cmask |= xm << (jy * GX);
                cmask &= vmask;
            }
            // output flag of a hit: bit 31 of the entry (set for stage-0 lists
            // by k_flag_s0 after the gates, by k_filter for later stages)
            const int outf = a.second ? static_cast<int>(static_cast<uint32_t>(ent.y) >> 31) : 1;
            // queue positions: exclusive prefix of the hit counts (0..6)
            // from one ballot per bit
            const int nc = __popc(cmask);
            const unsigned v0 = __ballot_sync(0xffffffffu, nc & 1);
            const unsigned v1 = __ballot_sync(0xffffffffu, nc & 2);
            const unsigned v2 = __ballot_sync(0xffffffffu, nc & 4);
            const unsigned lt = lanemask_lt();
            const int tot = __popc(v0) + 2 * __popc(v1) + 4 * __popc(v2);
            if (tot == 0) return;
            int pos = np + __popc(v0 & lt) + 2 * __popc(v1 & lt) + 4 * __popc(v2 & lt);
#pragma unroll
            for (int c = 0; c < NCELL; ++c) {
                if ((cmask >> c) & 1u) {
                    const int d = (ry - c / GX) * 3 + (rx - c % GX);      // (1 - dy) * 3 + (1 - dx)
                    qk[pos] = ent.x;
                    qm[pos] = static_cast<unsigned char>(d | (c << 4) | (outf << 7));
                    ++pos;
                }
            }
            np += tot;
            __syncwarp();
            while (np >= 32) {
                batch(32);
                np -= 32;
                // move the remaining queued slots to the front
                for (int b = 0; b < np; b += 32) {
                    int kk = 0, mm = 0;
                    if (b + lane < np) { kk = qk[32 + b + lane]; mm = qm[32 + b + lane]; }
                    __syncwarp();
                    if (b + lane < np) { qk[b + lane] = kk; qm[b + lane] = static_cast<unsigned char>(mm); }
                    __syncwarp();
                }
            }
        };
        // The walk keeps only the entries whose patch touches the group (a
        // few compares per entry), 32 at a time for the hit analysis.
        int nrel = 0;
        int cs = 0, cj = 0, ccnt = seg_cnt(0);
        while (cs < nseg && ccnt == 0) ccnt = seg_cnt(++cs);
        int2 cur = load_block(cs, 0, ccnt);
        while (cs < nseg) {
            int ns = cs, nj = cj + 32, ncnt = ccnt;
            if (nj >= ccnt) {
                ns = cs + 1;
                nj = 0;
                ncnt = seg_cnt(ns);
            }
            const int2 nxt = load_block(ns, nj, ncnt);       // in flight during this block's walk
            {
                const int ex = cur.y & 0xFFFF, ey = (cur.y >> 16) & 0x7FFF;
                const int rx = ex - gx0 + 1, ry = ey - gy0 + 1;
                const bool rel = cj + lane < ccnt && rx >= 0 && rx <= GX + 1 && ry >= 0 && ry <= GY + 1;
                const unsigned m = __ballot_sync(0xffffffffu, rel);
                if (rel) rbuf[nrel + __popc(m & lanemask_lt())] = cur;
                nrel += __popc(m);
                if (nrel >= 32) {
                    __syncwarp();
                    queue_hits(32);
                    nrel -= 32;
                    const int2 t = (lane < nrel) ? rbuf[32 + lane] : make_int2(0, 0);
                    __syncwarp();
                    if (lane < nrel) rbuf[lane] = t;
                }
            }
            cs = ns;
            cj = nj;
            ccnt = ncnt;
            cur = nxt;
            while (cs < nseg && cj >= ccnt) {               // empty segments
                ccnt = seg_cnt(++cs);
                cj = 0;
                cur = load_block(cs, 0, ccnt);
            }
        }
        if (nrel > 0) {
            __syncwarp();
            queue_hits(nrel);
        }
        if (np > 0) batch(np);
        if (uown) *reinterpret_cast<float4*>(hp) = h4;
    }
}

// ---------------------------------------------------------------------------
// Gather, phase 1 -- k_contrib: per patch position delta, the goW
// contribution of every output-producing event (layer_forward_ct,
// src/ssla_kernels.cpp:340-351, matvec_accum_ct linear.h:92-101):
//   C[row][delta][o] = fmaf chain over i of goW[delta][o][i] * qh[row][delta][i]
// A register-tiled FP32 GEMM per (delta, tile of BM rows): the tile's qh
// vectors (one contiguous S row segment each) and goW[delta] are staged in
// shared memory with batched 16-byte loads; a thread owns 8 rows x 3 outputs.
// Rows whose patch position is out of bounds are skipped (never read).
// QIN > 0 (layers 1-3): the staged rows are the cell states after each
// consumed hit; the tile's q = fmaf chain over i of qvgT[delta][i][o] *
// x[row][i] (matvec_ct, linear.h:80-90) is computed first, with the same
// thread tiling, and q * h replaces each staged value.
// ---------------------------------------------------------------------------
template <int A, int OUT, int QIN = 0>
struct ContribShape {
    static constexpr int CG = OUT / 3;           // column groups
    static constexpr int RG = kNT / CG;          // row groups
    static constexpr int BM = RG * 8;            // rows per tile
    static constexpr int BMP = BM + 4;           // padded transposed stride
    static constexpr size_t smem = sizeof(float) * (static_cast<size_t>(OUT) * OUT +
                                                    static_cast<size_t>(OUT) * BMP +
                                                    static_cast<size_t>(QIN) * OUT +
                                                    static_cast<size_t>(QIN) * BMP) +
                                   sizeof(int) * BM;
};

template <int A, int OUT, int QIN = 0>
__global__ void __launch_bounds__(kNT) k_contrib(ContribArgs a) {
    pdl_enter();
    using Sh = ContribShape<A, OUT, QIN>;
    constexpr int BM = Sh::BM, BMP = Sh::BMP, CG = Sh::CG;
    constexpr int Q4 = OUT / 4;                  // float4 per qh row
    constexpr int NA = (BM * Q4 + kNT - 1) / kNT;
    constexpr int NB = (OUT * OUT / 4 + kNT - 1) / kNT;
    extern __shared__ __align__(16) float dsm[];
    float* Bs = dsm;                             // [OUT][OUT]  goWT[delta] (i-major)
    float* As = Bs + OUT * OUT;                  // [OUT][BMP]  qh rows, transposed
    float* Wqs = As + OUT * BMP;                 // [QIN][OUT]  q weights of delta
    float* Xs = Wqs + QIN * OUT;                 // [QIN][BMP]  input rows, transposed
    int* srow_s = reinterpret_cast<int*>(Xs + QIN * BMP);   // S row or -1
    const int tid = threadIdx.x;
    const int cg = tid % CG, rg = tid / CG;
    const int s = a.stage;
    const int n_list = (a.list == 0) ? a.n_static : min(a.count[a.list], a.g.cap[a.list]);
    const int n_tiles = (n_list + BM - 1) / BM;
    const int Wl = a.g.W[s], Hl = a.g.H[s];
    for (int unit = blockIdx.x; unit < n_tiles * A; unit += gridDim.x) {
        const int d = (A - 1) - unit % A, tile = unit / A;
        const int dy = 1 - d / 3, dx = 1 - d % 3;
        __syncthreads();
        // unrolled over a thread's rows so their list and flag loads overlap
#pragma unroll
        for (int q = 0; q < (BM + kNT - 1) / kNT; ++q) {
            const int t = tid + q * kNT;
            if (t >= BM) break;
            const int r = tile * BM + t;
            int srow = -1;
            if (r < n_list) {
                uint32_t xy0;
                int sr;
                bool ok;
                if (a.list == 0) {
                    xy0 = a.ev_xy[r]; sr = r; ok = (a.rflags[r] & (F_VALID | F_FOREIGN)) == F_VALID;
                } else {
                    const StageEntry se = a.E[r];
                    xy0 = se.xy0; sr = a.second ? se.kprev : r; ok = (a.rflags[se.e] & F_FOREIGN) == 0;
                }
                const int cx = static_cast<int>(xy0 & 0xFFFFu) >> s, cy = static_cast<int>(xy0 >> 16) >> s;
                if (A == 9) ok = ok && cx + dx >= 0 && cx + dx < Wl && cy + dy >= 0 && cy + dy < Hl;
                if (ok) srow = sr;
            }
            srow_s[t] = srow;
        }
        __syncthreads();
        {   // batched loads: goW[delta] and the tile's qh rows
            const float4* gsrc = reinterpret_cast<const float4*>(a.goWT + static_cast<size_t>(d) * OUT * OUT);
            float4 bv[NB];
#pragma unroll
            for (int q = 0; q < NB; ++q) {
                const int t = tid + q * kNT;
                if (t < OUT * OUT / 4) bv[q] = __ldg(gsrc + t);
            }
            float4 av[NA];
#pragma unroll
            for (int q = 0; q < NA; ++q) {
                const int t = tid + q * kNT;
                const int r = t % BM, k4 = t / BM;
                av[q] = make_float4(0.f, 0.f, 0.f, 0.f);
                if (t < BM * Q4 && srow_s[r] >= 0)
                    av[q] = *reinterpret_cast<const float4*>(
                        a.S + (static_cast<size_t>(srow_s[r]) * A + d) * a.qstride + 4 * k4);
            }
#pragma unroll
            for (int q = 0; q < NB; ++q) {
                const int t = tid + q * kNT;
                if (t < OUT * OUT / 4) reinterpret_cast<float4*>(Bs)[t] = bv[q];
            }
#pragma unroll
            for (int q = 0; q < NA; ++q) {
                const int t = tid + q * kNT;
                if (t < BM * Q4) {
                    const int r = t % BM, k4 = t / BM;
                    As[(4 * k4 + 0) * BMP + r] = av[q].x;
                    As[(4 * k4 + 1) * BMP + r] = av[q].y;
                    As[(4 * k4 + 2) * BMP + r] = av[q].z;
                    As[(4 * k4 + 3) * BMP + r] = av[q].w;
                }
            }
        }
        if constexpr (QIN > 0) {
            // q weights of delta and the tile's input rows: all of a
            // thread's loads issued before its stores (one round trip)
            constexpr int NWQ = (QIN * OUT + kNT - 1) / kNT;
            constexpr int NXQ = (BM * (QIN / 4) + kNT - 1) / kNT;
            float wq[NWQ];
            float4 xq[NXQ];
#pragma unroll
            for (int q = 0; q < NWQ; ++q) {
                const int t = tid + q * kNT;
                if (t < QIN * OUT)
                    wq[q] = __ldg(a.Wq + (static_cast<size_t>(d) * QIN + t / OUT) * (3 * OUT) + t % OUT);
            }
#pragma unroll
            for (int q = 0; q < NXQ; ++q) {
                const int t = tid + q * kNT;
                const int r = t % BM, k4 = t / BM;
                xq[q] = make_float4(0.f, 0.f, 0.f, 0.f);
                if (t < BM * (QIN / 4) && srow_s[r] >= 0)
                    xq[q] = __ldg(reinterpret_cast<const float4*>(a.Xq + static_cast<size_t>(srow_s[r]) * QIN) + k4);
            }
#pragma unroll
            for (int q = 0; q < NWQ; ++q) {
                const int t = tid + q * kNT;
                if (t < QIN * OUT) Wqs[t] = wq[q];
            }
#pragma unroll
            for (int q = 0; q < NXQ; ++q) {
                const int t = tid + q * kNT;
                if (t < BM * (QIN / 4)) {
                    const int r = t % BM, k4 = t / BM;
                    Xs[(4 * k4 + 0) * BMP + r] = xq[q].x;
                    Xs[(4 * k4 + 1) * BMP + r] = xq[q].y;
                    Xs[(4 * k4 + 2) * BMP + r] = xq[q].z;
                    Xs[(4 * k4 + 3) * BMP + r] = xq[q].w;
                }
            }
            __syncthreads();
            float qa[8][3];
#pragma unroll
            for (int i = 0; i < 8; ++i)
#pragma unroll
                for (int j = 0; j < 3; ++j) qa[i][j] = 0.0f;
#pragma unroll 4
            for (int k = 0; k < QIN; ++k) {
                const float4 x0 = *reinterpret_cast<const float4*>(Xs + k * BMP + rg * 8);
                const float4 x1 = *reinterpret_cast<const float4*>(Xs + k * BMP + rg * 8 + 4);
                const float w0 = Wqs[k * OUT + cg * 3 + 0];
                const float w1 = Wqs[k * OUT + cg * 3 + 1];
                const float w2 = Wqs[k * OUT + cg * 3 + 2];
                const float x[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    qa[i][0] = fmaf(w0, x[i], qa[i][0]);
                    qa[i][1] = fmaf(w1, x[i], qa[i][1]);
                    qa[i][2] = fmaf(w2, x[i], qa[i][2]);
                }
            }
#pragma unroll
            for (int i = 0; i < 8; ++i)
#pragma unroll
                for (int j = 0; j < 3; ++j) {
                    float* e = As + (cg * 3 + j) * BMP + rg * 8 + i;
                    *e = qa[i][j] * *e;
                }
        }
        __syncthreads();
        float acc[8][3];
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int j = 0; j < 3; ++j) acc[i][j] = 0.0f;
#pragma unroll 4
        for (int k = 0; k < OUT; ++k) {
            const float4 a0 = *reinterpret_cast<const float4*>(As + k * BMP + rg * 8);
            const float4 a1 = *reinterpret_cast<const float4*>(As + k * BMP + rg * 8 + 4);
            const float b0 = Bs[k * OUT + cg * 3 + 0];
            const float b1 = Bs[k * OUT + cg * 3 + 1];
            const float b2 = Bs[k * OUT + cg * 3 + 2];
            const float2 xp[4] = {make_float2(a0.x, a0.y), make_float2(a0.z, a0.w),
                                  make_float2(a1.x, a1.y), make_float2(a1.z, a1.w)};
            const float2 bb[3] = {make_float2(b0, b0), make_float2(b1, b1), make_float2(b2, b2)};
            // row pairs per packed FMA (each component an fmaf)
#pragma unroll
            for (int i2 = 0; i2 < 4; ++i2)
#pragma unroll
                for (int j = 0; j < 3; ++j) {
                    const float2 r = __ffma2_rn(bb[j], xp[i2], make_float2(acc[2 * i2][j], acc[2 * i2 + 1][j]));
                    acc[2 * i2][j] = r.x;
                    acc[2 * i2 + 1][j] = r.y;
                }
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int rr = rg * 8 + i;
            if (srow_s[rr] < 0) continue;
            float* c = a.C + (static_cast<size_t>(tile * BM + rr) * A + d) * OUT + cg * 3;
            c[0] = acc[i][0]; c[1] = acc[i][1]; c[2] = acc[i][2];
        }
    }
}

// ---------------------------------------------------------------------------
// Gather, phase 2 -- k_ln: EV output-producing events per CTA.
//   1) (event, channel) pairs: out[o] = ((0 + C[8][o]) + C[7][o]) + ... +
//      C[0][o] (in-bounds patch positions only, the reference's patch
//      order), + residual (add_inplace);
//   2) lane = event: LayerNorm mean / variance as sequential fp64 sums over
//      the channels (layernorm.h:41-62), EV events at once;
//   3) (event, channel) pairs: normalise with gamma / beta and write the
//      layer output row, the copy residual of the stage's second layer,
//      per-event stage outputs and the drain_n slot contents;
//   4) second layers with a next stage: that stage's first-layer residual
//      input_proj * x (matvec_ct<OUT, 2*OUT>), weights staged in smem.
// Every thread owns PPT pairs, fully unrolled so their loads overlap.
// ---------------------------------------------------------------------------
template <int OUT>
struct LnShape {
    static constexpr int EV = OUT <= 24 ? 32 : (OUT == 48 ? 16 : 8);   // events per CTA
    static constexpr int NT = OUT == 12 ? 128 : 256;                   // threads
    static constexpr int PPT = EV * OUT / NT;                          // pairs per thread
    static constexpr int PPT4 = EV * 2 * OUT / NT;                     // residual pairs
    static_assert(EV * OUT % NT == 0 && EV <= 32, "shape");
};

template <int A, int OUT>
__global__ void __launch_bounds__(LnShape<OUT>::NT, 65536 / (LnShape<OUT>::NT * 80)) k_ln(LnArgs a) {
    using Sh = LnShape<OUT>;
    constexpr int EV = Sh::EV, NT = Sh::NT, PPT = Sh::PPT;
    constexpr int ST = OUT + 1;                  // conflict-free lane-per-event rows
    constexpr int IPN = (A == 9 && OUT <= 48) ? OUT * 2 * OUT : 1;
    __shared__ float ybuf[EV * ST];
    __shared__ __align__(16) float ipw[IPN];
    __shared__ double mean_s[EV], inv_s[EV];
    __shared__ int ev_r[EV], ev_sr[EV], ev_e[EV], ev_cx[EV], ev_cy[EV];
    __shared__ unsigned char ev_ok[EV], ev_cp[EV];
    const int tid = threadIdx.x;
    // the next stage's input_proj weights are constant: staged before the
    // wait for the previous kernel, every load issued before the stores
    const bool ipn = (IPN > 1) && a.ipT_next != nullptr;
    if (ipn) {
        if ((reinterpret_cast<uintptr_t>(a.ipT_next) & 15u) == 0) {
            constexpr int N4 = IPN / 4, PT = N4 > 0 ? (N4 + NT - 1) / NT : 1;
            float4 v[PT];
#pragma unroll
            for (int q = 0; q < PT; ++q) {
                const int t = tid + q * NT;
                if (t < N4) v[q] = __ldg(reinterpret_cast<const float4*>(a.ipT_next) + t);
            }
#pragma unroll
            for (int q = 0; q < PT; ++q) {
                const int t = tid + q * NT;
                if (t < N4) reinterpret_cast<float4*>(ipw)[t] = v[q];
            }
        } else {
            for (int t = tid; t < IPN; t += NT) ipw[t] = __ldg(a.ipT_next + t);
        }
    }
    pdl_wait();
    const int s = a.stage;
    const int n_list = (a.list == 0) ? a.n_static : min(a.count[a.list], a.g.cap[a.list]);
    const int Wl = a.g.W[s], Hl = a.g.H[s];
    for (int r0 = blockIdx.x * EV; r0 < n_list; r0 += gridDim.x * EV) {
        __syncthreads();
        if (tid < EV) {
            const int r = r0 + tid;
            int ok = 0, sr = 0, e = 0;
            uint32_t xy0 = 0;
            if (r < n_list) {
                if (a.list == 0) {
                    xy0 = a.ev_xy[r]; sr = r; e = r; ok = (a.rflags[r] & (F_VALID | F_FOREIGN)) == F_VALID;
                } else {
                    const StageEntry se = a.E[r];
                    xy0 = se.xy0; sr = a.second ? se.kprev : r; e = se.e; ok = (a.rflags[e] & F_FOREIGN) == 0;
                }
            }
            ev_r[tid] = r; ev_sr[tid] = sr; ev_e[tid] = e; ev_ok[tid] = static_cast<unsigned char>(ok);
            ev_cx[tid] = static_cast<int>(xy0 & 0xFFFFu) >> s;
            ev_cy[tid] = static_cast<int>(xy0 >> 16) >> s;
            ev_cp[tid] = (ok && a.copyres_bit && (a.rflags[e] & a.copyres_bit)) ? 1 : 0;
        }
        __syncthreads();
        // 1) ordered patch sum + residual
        {
            float c[PPT][A], rv[PPT];
#pragma unroll
            for (int j = 0; j < PPT; ++j) {
                const int t = tid + j * NT;
                const int ei = t / OUT, o = t % OUT;
                const bool ok = ev_ok[ei];
                const int r = ev_r[ei], cx = ev_cx[ei], cy = ev_cy[ei];
#pragma unroll
                for (int d = 0; d < A; ++d) {
                    bool in = ok;
                    if (A == 9) {
                        const int dy = 1 - d / 3, dx = 1 - d % 3;
                        in = in && cx + dx >= 0 && cx + dx < Wl && cy + dy >= 0 && cy + dy < Hl;
                    }
                    c[j][d] = in ? __ldg(a.C + (static_cast<size_t>(r) * A + d) * OUT + o) : 0.0f;
                }
                rv[j] = ok ? __ldg(a.R_in + static_cast<size_t>(ev_sr[ei]) * OUT + o) : 0.0f;
            }
#pragma unroll
            for (int j = 0; j < PPT; ++j) {
                const int t = tid + j * NT;
                const int ei = t / OUT, o = t % OUT;
                const int cx = ev_cx[ei], cy = ev_cy[ei];
                float v = 0.0f;
#pragma unroll
                for (int d = A - 1; d >= 0; --d) {
                    if (A == 9) {
                        const int dy = 1 - d / 3, dx = 1 - d % 3;
                        if (cx + dx < 0 || cx + dx >= Wl || cy + dy < 0 || cy + dy >= Hl) continue;
                    }
                    v = v + c[j][d];
                }
                ybuf[ei * ST + o] = v + rv[j];
            }
        }
        __syncthreads();
        // 2) sequential fp64 statistics, one lane per event
        if (tid < EV && ev_ok[tid]) {
            const float* y = ybuf + tid * ST;
            double sum = 0.0;
#pragma unroll 4
            for (int o = 0; o < OUT; ++o) sum += static_cast<double>(y[o]);
            const double mean = sum / static_cast<double>(OUT);
            double var = 0.0;
#pragma unroll 4
            for (int o = 0; o < OUT; ++o) {
                const double dd = static_cast<double>(y[o]) - mean;
                var += dd * dd;
            }
            var /= static_cast<double>(OUT);
            mean_s[tid] = mean;
            inv_s[tid] = 1.0 / sqrt(var + static_cast<double>(1e-5f));
        }
        __syncthreads();
        // 3) normalise and write
#pragma unroll
        for (int j = 0; j < PPT; ++j) {
            const int t = tid + j * NT;
            const int ei = t / OUT, o = t % OUT;
            if (!ev_ok[ei]) continue;
            const int r = ev_r[ei], e = ev_e[ei];
            const double tt = (static_cast<double>(ybuf[ei * ST + o]) - mean_s[ei]) * inv_s[ei];
            const float xv = static_cast<float>(tt * static_cast<double>(__ldg(a.L.gamma + o)) +
                                                static_cast<double>(__ldg(a.L.beta + o)));
            if (a.X_out) a.X_out[static_cast<size_t>(r) * OUT + o] = xv;
            if (ev_cp[ei]) a.R_next[static_cast<size_t>(r) * OUT + o] = xv;
            if (a.stage_out && a.second) a.stage_out[static_cast<size_t>(e) * OUT + o] = xv;
            if (a.slot_feat) {
                a.slot_feat[static_cast<size_t>(e) * 96 + o] = xv;
                if (OUT == 48) a.slot_feat[static_cast<size_t>(e) * 96 + 48 + o] = 0.0f;
            }
            ybuf[ei * ST + o] = xv;
        }
        if (ipn) {
            __syncthreads();
            // 4) next stage's first-layer residual, row r of the same list
            constexpr int P4 = (IPN > 1) ? Sh::PPT4 : 1;
            float acc[P4];
            int ei4[P4], o24[P4];
#pragma unroll
            for (int j = 0; j < P4; ++j) {
                const int t = tid + j * NT;
                ei4[j] = t / (2 * OUT);
                o24[j] = t % (2 * OUT);
                acc[j] = 0.0f;
            }
#pragma unroll 2
            for (int i = 0; i < OUT; ++i) {
#pragma unroll
                for (int j = 0; j < P4; ++j)
                    acc[j] = fmaf(ipw[i * 2 * OUT + o24[j]], ybuf[ei4[j] * ST + i], acc[j]);
            }
#pragma unroll
            for (int j = 0; j < P4; ++j)
                if (ev_ok[ei4[j]])
                    a.R_ipnext[static_cast<size_t>(ev_r[ei4[j]]) * 2 * OUT + o24[j]] = acc[j];
        }
    }
}

// ---------------------------------------------------------------------------
// k_head: YOLOX head on the stage-3 features of head events
// (decode_yolox_cell_ct, vendor/openeva/heads/async_yolox.h:203-254):
// cls / reg 1x1 convs with BN folded (bias-first fmaf chains) + SiLU, then
// the cls (ncls), reg (4) and obj (1) predictions, then the box decode.
// 32 events per batch; X holds the features in E_4 row order.
// ---------------------------------------------------------------------------
// Dynamic shared memory of k_head for `cols` = 5 + ncls outputs: the two 1x1
// convolutions' weights [96][96] each, the prediction weights [96][cols]
// (reg 0..3, obj 4, cls 5..), the batch's features [96][kMB], activations
// [192][kMB] and results [kMB][cols].
size_t head_smem_bytes(int cols) {
    return sizeof(float) * (2 * 96 * 96 + static_cast<size_t>(96) * cols + 96 * kMB + 192 * kMB +
                            static_cast<size_t>(kMB) * cols);
}

// The weights are constant: staged in shared memory before the wait for the
// previous kernel, so every fmaf chain reads them at shared-memory latency.
// kHeadNT threads: one per (convolution output, group of kEPT events) of a
// batch, so each thread runs one 96-step chain group per batch.
constexpr int kHeadNT = 192 * kGroups;
__global__ void __launch_bounds__(kHeadNT) k_head(HeadArgs a) {
    extern __shared__ __align__(16) float hsm[];
    const int ncls = a.g.ncls, cols = 5 + ncls;
    float* const w_cls = hsm;                    // [96][96] cls_convT
    float* const w_reg = w_cls + 96 * 96;        // [96][96] reg_convT
    float* const x_s = w_reg + 96 * 96;          // [96][kMB]
    float* const act_s = x_s + 96 * kMB;         // [192][kMB]
    float* const w_pred = act_s + 192 * kMB;     // [96][cols]
    float* const res_s = w_pred + 96 * cols;     // [kMB][cols]
    __shared__ int valid_s[kMB], cx_s[kMB], cy_s[kMB];
    const int tid = threadIdx.x;
    {
        const float* const src[2] = {a.head.cls_convT, a.head.reg_convT};
#pragma unroll
        for (int m = 0; m < 2; ++m) {
            float* const dst = hsm + m * 96 * 96;
            if ((reinterpret_cast<uintptr_t>(src[m]) & 15u) == 0) {
                constexpr int N4 = 96 * 96 / 4, PT = (N4 + kHeadNT - 1) / kHeadNT;
                float4 v[PT];
#pragma unroll
                for (int q = 0; q < PT; ++q) {
                    const int t = tid + q * kHeadNT;
                    if (t < N4) v[q] = __ldg(reinterpret_cast<const float4*>(src[m]) + t);
                }
#pragma unroll
                for (int q = 0; q < PT; ++q) {
                    const int t = tid + q * kHeadNT;
                    if (t < N4) reinterpret_cast<float4*>(dst)[t] = v[q];
                }
            } else {
                for (int t = tid; t < 96 * 96; t += kHeadNT) dst[t] = __ldg(src[m] + t);
            }
        }
        for (int t = tid; t < 96 * cols; t += kHeadNT) {
            const int i = t / cols, r = t % cols;
            w_pred[t] = (r < 4) ? __ldg(a.head.reg_predT + i * 4 + r)
                      : (r == 4) ? __ldg(a.head.obj_predT + i)
                                 : __ldg(a.head.cls_predT + i * ncls + (r - 5));
        }
    }
    pdl_wait();
    const int n = min(a.count[4], a.g.cap[4]);
    for (int batch = blockIdx.x; batch * kMB < n; batch += gridDim.x) {
        __syncthreads();
        if (tid < kMB) {
            const int r = batch * kMB + tid;
            valid_s[tid] = r < n;
            const uint32_t xy0 = (r < n) ? a.E4[r].xy0 : 0u;
            cx_s[tid] = static_cast<int>(xy0 & 0xFFFFu) >> 3;
            cy_s[tid] = static_cast<int>(xy0 >> 16) >> 3;
        }
        for (int t = tid; t < 96 * kMB; t += kHeadNT) {
            const int i = t % 96, b = t / 96;
            const int r = batch * kMB + b;
            x_s[i * kMB + b] = (r < n) ? a.X[static_cast<size_t>(r) * 96 + i] : 0.0f;
        }
        __syncthreads();
        for (int item = tid; item < 192 * kGroups; item += kHeadNT) {
            const int j = item % 192, g = item / 192;
            const int jo = j % 96;
            const float* Wt = (j < 96) ? w_cls : w_reg;
            const float bias = __ldg(((j < 96) ? a.head.cls_conv_b : a.head.reg_conv_b) + jo);
            float acc[kEPT];
#pragma unroll
            for (int b = 0; b < kEPT; ++b) acc[b] = bias;
#pragma unroll 4
            for (int i = 0; i < 96; ++i) {
                const float wv = Wt[i * 96 + jo];
                const float4 x0 = *reinterpret_cast<const float4*>(x_s + i * kMB + g * kEPT);
                const float4 x1 = *reinterpret_cast<const float4*>(x_s + i * kMB + g * kEPT + 4);
                acc[0] = fmaf(wv, x0.x, acc[0]); acc[1] = fmaf(wv, x0.y, acc[1]);
                acc[2] = fmaf(wv, x0.z, acc[2]); acc[3] = fmaf(wv, x0.w, acc[3]);
                acc[4] = fmaf(wv, x1.x, acc[4]); acc[5] = fmaf(wv, x1.y, acc[5]);
                acc[6] = fmaf(wv, x1.z, acc[6]); acc[7] = fmaf(wv, x1.w, acc[7]);
            }
#pragma unroll
            for (int b = 0; b < kEPT; ++b)
                act_s[j * kMB + g * kEPT + b] = acc[b] * ssla_sigmoidf(acc[b]);
        }
        __syncthreads();
        for (int item = tid; item < kMB * cols; item += kHeadNT) {
            const int b = item % kMB, r = item / kMB;
            if (!valid_s[b]) continue;
            // reg (0..3) and obj (4) read the reg branch, cls (5..) the cls branch
            const float* act = act_s + (r < 5 ? 96 * kMB : 0) + b;
            float acc = (r < 4) ? __ldg(a.head.reg_pred_b + r)
                      : (r == 4) ? __ldg(a.head.obj_pred_b)
                                 : __ldg(a.head.cls_pred_b + (r - 5));
#pragma unroll 8
            for (int i = 0; i < 96; ++i) acc = fmaf(w_pred[i * cols + r], act[i * kMB], acc);
            res_s[b * cols + r] = acc;
        }
        __syncthreads();
        for (int item = tid; item < kMB * cols; item += kHeadNT) {
            const int b = item % kMB, r = item / kMB;
            if (!valid_s[b]) continue;
            const int row = batch * kMB + b;
            const float v = res_s[b * cols + r];
            float d;
            if (r == 0) d = (v + static_cast<float>(cx_s[b])) * static_cast<float>(a.g.stride_w);
            else if (r == 1) d = (v + static_cast<float>(cy_s[b])) * static_cast<float>(a.g.stride_h);
            else if (r == 2) d = ssla_expf(v) * static_cast<float>(a.g.stride_w);
            else if (r == 3) d = ssla_expf(v) * static_cast<float>(a.g.stride_h);
            else d = v;
            a.head_dec[static_cast<size_t>(row) * cols + r] = d;
            a.head_raw[static_cast<size_t>(row) * cols + r] = v;
        }
    }
}

// ---------------------------------------------------------------------------
// k_gemm: next-layer fused qvg (matvec_ct<IN,3*OUT>, linear.h:80-90) for a set
// of events and a set of weight columns, as a register-tiled FP32 GEMM:
//   Y[row][col] = sum_k X[row][k] * W[k][col]   (fmaf chain, k ascending)
// Columns are ordered part-major (all q, then all v, then all g; inside a
// part by patch position delta, then output channel), so a warp's columns
// share one part and the sigmoid of the g part is warp-uniform:
//   COLS_ALL  q, v, g      (first layers: every output is consumed)
//   COLS_VG   v, g         (second layers: every event)
//   COLS_Q    q            (second layers: events whose output is consumed)
//   COLS_RES  input_proj   (the residual, matvec_ct<IN,OUT>)
// g columns are stored as sigmoid(g).  A CTA computes a BM x BN tile with the
// whole K extent of X and W staged in shared memory (batched 16-byte loads);
// a thread owns 8 rows x 4 columns.  grid-stride over (row tile, col tile).
// ---------------------------------------------------------------------------
template <int K, int OUT2, int BM, int BN>
__global__ void __launch_bounds__(kNT) k_gemm(GemmArgs a) {
    pdl_enter();
    constexpr int J2 = 3 * OUT2;
    constexpr int TN = BN / 4;                  // column groups (threads per row group)
    static_assert((BM / 8) * TN == kNT, "tile shape");
    constexpr int BMP = BM + 4;
    constexpr int NA = (BM * (K / 4) + kNT - 1) / kNT;
    constexpr int NB = (K * (BN / 4) + kNT - 1) / kNT;
    extern __shared__ __align__(16) float dsm[];
    float* As = dsm;                            // [K][BMP]
    float* Bs = dsm + K * BMP;                  // [K][BN]
    __shared__ int xrow_s[BM];
    const int tid = threadIdx.x;
    const int tx = tid % TN, ty = tid / TN;
    const int n_rows = (a.list == 0) ? a.n_static : min(a.count[a.list], a.g_cap);
    const int n_rt = (n_rows + BM - 1) / BM;
    const int n_ct = (a.n_cols + BN - 1) / BN;
    constexpr int A2 = 9;                       // layers 4-7: 3x3 patches
    constexpr int per_part = A2 * OUT2;
    const int part0 = (a.colmode == COLS_VG) ? 1 : 0;
    constexpr size_t srow_stride = static_cast<size_t>(A2) * J2;
    for (int unit = blockIdx.x; unit < n_rt * n_ct; unit += gridDim.x) {
        const int rt = unit / n_ct, ct = unit % n_ct;
        const int r0 = rt * BM, c0 = ct * BN;
        __syncthreads();
        if (tid < BM) {
            const int r = r0 + tid;
            xrow_s[tid] = (r < n_rows) ? (a.E ? a.E[r].kprev : r) : -1;
        }
        __syncthreads();
        float4 av[NA], bv[NB];
#pragma unroll
        for (int q = 0; q < NA; ++q) {
            const int t = tid + q * kNT;
            const int r = t % BM, k4 = t / BM;
            av[q] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (t < BM * (K / 4) && xrow_s[r] >= 0)
                av[q] = *reinterpret_cast<const float4*>(a.X + static_cast<size_t>(xrow_s[r]) * K + 4 * k4);
        }
#pragma unroll
        for (int q = 0; q < NB; ++q) {
            const int t = tid + q * kNT;
            const int c4 = t % (BN / 4), k = t / (BN / 4);
            const int col = c0 + 4 * c4;
            bv[q] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (t < K * (BN / 4) && col < a.n_cols) {
                const float* src;
                if (a.colmode == COLS_RES) {
                    src = a.W + static_cast<size_t>(k) * OUT2 + col;
                } else {
                    const int part = part0 + col / per_part, rem = col % per_part;
                    const int d = rem / OUT2, o = rem % OUT2;
                    src = a.W + (static_cast<size_t>(d) * K + k) * J2 + part * OUT2 + o;
                }
                bv[q] = __ldg(reinterpret_cast<const float4*>(src));
            }
        }
#pragma unroll
        for (int q = 0; q < NA; ++q) {
            const int t = tid + q * kNT;
            if (t < BM * (K / 4)) {
                const int r = t % BM, k4 = t / BM;
                As[(4 * k4 + 0) * BMP + r] = av[q].x;
                As[(4 * k4 + 1) * BMP + r] = av[q].y;
                As[(4 * k4 + 2) * BMP + r] = av[q].z;
                As[(4 * k4 + 3) * BMP + r] = av[q].w;
            }
        }
#pragma unroll
        for (int q = 0; q < NB; ++q) {
            const int t = tid + q * kNT;
            if (t < K * (BN / 4)) {
                const int c4 = t % (BN / 4), k = t / (BN / 4);
                *reinterpret_cast<float4*>(Bs + k * BN + 4 * c4) = bv[q];
            }
        }
        __syncthreads();
        // column pairs per packed FMA (each component an fmaf)
        float2 acc2[8][2];
#pragma unroll
        for (int i = 0; i < 8; ++i) acc2[i][0] = acc2[i][1] = make_float2(0.0f, 0.0f);
#pragma unroll 4
        for (int k = 0; k < K; ++k) {
            const float4 a0 = *reinterpret_cast<const float4*>(As + k * BMP + ty * 8);
            const float4 a1 = *reinterpret_cast<const float4*>(As + k * BMP + ty * 8 + 4);
            const float4 b = *reinterpret_cast<const float4*>(Bs + k * BN + tx * 4);
            const float x[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
            const float2 w01 = make_float2(b.x, b.y), w23 = make_float2(b.z, b.w);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const float2 xx = make_float2(x[i], x[i]);
                acc2[i][0] = __ffma2_rn(xx, w01, acc2[i][0]);
                acc2[i][1] = __ffma2_rn(xx, w23, acc2[i][1]);
            }
        }
        float acc[8][4];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            acc[i][0] = acc2[i][0].x; acc[i][1] = acc2[i][0].y;
            acc[i][2] = acc2[i][1].x; acc[i][3] = acc2[i][1].y;
        }
        // epilogue: 4 consecutive columns share part and delta
        const int col = c0 + tx * 4;
        if (col < a.n_cols) {
            int jcol = col, part = 0;
            if (a.colmode != COLS_RES) {
                part = part0 + col / per_part;
                const int rem = col % per_part;
                jcol = (rem / OUT2) * J2 + part * OUT2 + rem % OUT2;
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int xr = xrow_s[ty * 8 + i];
                if (xr < 0) continue;
                float4 v = make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
                if (a.colmode == COLS_RES) {
                    *reinterpret_cast<float4*>(a.R + static_cast<size_t>(xr) * OUT2 + col) = v;
                } else {
                    if (part == 2) {
                        const float2 s01 = ssla_sigmoidf2(make_float2(v.x, v.y));
                        const float2 s23 = ssla_sigmoidf2(make_float2(v.z, v.w));
                        v = make_float4(s01.x, s01.y, s23.x, s23.y);
                    }
                    *reinterpret_cast<float4*>(a.S + static_cast<size_t>(xr) * srow_stride + jcol) = v;
                }
            }
        }
    }
}

// ---------------------------------------------------------------------------
// k_commit: one warp per (partition, s3 cell): the last head event of the
// chunk at the cell (stream order) sets the cell's prediction rows, and the
// version counter advances by the number of head writes
// (ssla_kernels.cpp:927-967 last-writer semantics; ssla_s2_s3_head_celled.cuh:
// 887-901 ownership + version).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kNT) k_commit(CommitArgs a) {
    pdl_enter();
    const int p = blockIdx.x;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int W3 = a.g.W[3], H3 = a.g.H[3];
    const int cell = blockIdx.y * (kNT / 32) + warp;
    if (cell >= W3 * H3) return;
    const PartState ps = a.parts[p];
    const int lo = a.off4[p], hi = min(a.off4[p + 1], a.g.cap[4]);
    int count = 0, last = -1;
    for (int j0 = lo; j0 < hi; j0 += 32) {
        const int j = j0 + lane;
        bool hit = false;
        if (j < hi) {
            const uint32_t xy0 = a.E4[j].xy0;
            const int x0 = static_cast<int>(xy0 & 0xFFFFu), y0 = static_cast<int>(xy0 >> 16);
            const int x2 = x0 >> 2, y2 = y0 >> 2;
            hit = ((y0 >> 3) * W3 + (x0 >> 3)) == cell && x2 >= ps.own_x0 && x2 < ps.own_x1 &&
                  y2 >= ps.own_y0 && y2 < ps.own_y1;
        }
        const unsigned m = __ballot_sync(0xffffffffu, hit);
        count += __popc(m);
        if (m) last = j0 + hi_lane(m);
    }
    if (count == 0) return;
    const int cols = 5 + a.g.ncls;
    if (lane < cols) {
        ps.preds_dec[static_cast<size_t>(cell) * cols + lane] = a.head_dec[static_cast<size_t>(last) * cols + lane];
        ps.preds_raw[static_cast<size_t>(cell) * cols + lane] = a.head_raw[static_cast<size_t>(last) * cols + lane];
    }
    if (lane == 0) ps.version[cell] += static_cast<uint32_t>(count);
}

// Reset: prediction rows = head(0 feature) for every cell
// (prepopulate_head_zero, ssla_kernels.cpp:969-989); raw rows and versions 0.
__global__ void k_reset_preds(Geo g, const PartState* parts, DevHead hd) {
    const int p = blockIdx.x;
    const int n3 = g.W[3] * g.H[3];
    const int cols = 5 + g.ncls;
    const PartState ps = parts[p];
    for (int cell = threadIdx.x; cell < n3; cell += blockDim.x) {
        float cls_f[96], reg_f[96];
        for (int j = 0; j < 96; ++j) {
            float acc = hd.cls_conv_b[j];
            float acc2 = hd.reg_conv_b[j];
            for (int i = 0; i < 96; ++i) {
                acc = fmaf(hd.cls_convT[i * 96 + j], 0.0f, acc);
                acc2 = fmaf(hd.reg_convT[i * 96 + j], 0.0f, acc2);
            }
            cls_f[j] = acc * ssla_sigmoidf(acc);
            reg_f[j] = acc2 * ssla_sigmoidf(acc2);
        }
        float res[21];
        for (int r = 0; r < cols; ++r) {
            float acc;
            if (r < 4) {
                acc = hd.reg_pred_b[r];
                for (int i = 0; i < 96; ++i) acc = fmaf(hd.reg_predT[i * 4 + r], reg_f[i], acc);
            } else if (r == 4) {
                acc = hd.obj_pred_b[0];
                for (int i = 0; i < 96; ++i) acc = fmaf(hd.obj_predT[i], reg_f[i], acc);
            } else {
                acc = hd.cls_pred_b[r - 5];
                for (int i = 0; i < 96; ++i) acc = fmaf(hd.cls_predT[i * g.ncls + (r - 5)], cls_f[i], acc);
            }
            res[r] = acc;
        }
        const int gx = cell % g.W[3], gy = cell / g.W[3];
        for (int r = 0; r < cols; ++r) {
            float d;
            if (r == 0) d = (res[0] + static_cast<float>(gx)) * static_cast<float>(g.stride_w);
            else if (r == 1) d = (res[1] + static_cast<float>(gy)) * static_cast<float>(g.stride_h);
            else if (r == 2) d = ssla_expf(res[2]) * static_cast<float>(g.stride_w);
            else if (r == 3) d = ssla_expf(res[3]) * static_cast<float>(g.stride_h);
            else d = res[r];
            ps.preds_dec[static_cast<size_t>(cell) * cols + r] = d;
            ps.preds_raw[static_cast<size_t>(cell) * cols + r] = 0.0f;
        }
        ps.version[cell] = 0u;
    }
}

// drain_n output slots (ssla_s2_s3_head_celled.cuh:1066-1087): pass codes
// 1 owner-passed / 0 owner-dropped / -1 halo, and the s3_feat slot as the
// reference kernel leaves it.  outs: device array of per-block slot arrays.
__global__ void k_write_slots(int n, int P, const int* __restrict__ rec_off,
                              const uint8_t* __restrict__ rflags,
                              const uint32_t* __restrict__ ev_xy,
                              const PartState* __restrict__ parts,
                              const float* __restrict__ slot_feat,
                              HybridS2S3OutputSlot* const* outs) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        int p = 0;
        while (p + 1 < P && i >= rec_off[p + 1]) ++p;
        const PartState& ps = parts[p];
        const uint32_t xy0 = ev_xy[i];
        const int x2 = static_cast<int>(xy0 & 0xFFFFu) >> 2, y2 = static_cast<int>(xy0 >> 16) >> 2;
        const bool owner = x2 >= ps.own_x0 && x2 < ps.own_x1 && y2 >= ps.own_y0 && y2 < ps.own_y1;
        const uint8_t f = rflags[i];
        const int p2 = (f & F_R3) ? 1 : 0;
        const int p3 = (f & F_R4) ? 1 : 0;
        if (outs[p] == nullptr) continue;
        HybridS2S3OutputSlot* o = outs[p] + (i - rec_off[p]);
        o->pass2 = owner ? p2 : -1;
        o->pass3 = owner ? (p2 ? p3 : 0) : -1;
        for (int c = 0; c < 96; ++c) o->s3_feat[c] = slot_feat[static_cast<size_t>(i) * 96 + c];
    }
}

// drain_n timing words: every (t_pop, t_done) pair of a block's batch_clk
// array gets the drain's start / end %globaltimer stamps.
__global__ void k_fill_clk(int P, const int* __restrict__ rec_off,
                           const unsigned long long* __restrict__ stamps,
                           unsigned long long* const* clks) {
    const int p = blockIdx.x;
    if (clks[p] == nullptr) return;
    const int nb = (rec_off[p + 1] - rec_off[p] + 7) / 8;
    for (int b = threadIdx.x; b < nb; b += blockDim.x) {
        clks[p][2 * b] = stamps[0];
        clks[p][2 * b + 1] = stamps[1];
    }
}

// Per-block timing words of the drain_n contract: global nanosecond timer.
__global__ void k_stamp(unsigned long long* dst) {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    *dst = t;
}

// ---------------------------------------------------------------------------
// Explicit instantiations used by the engine.
// ---------------------------------------------------------------------------
template __global__ void k_scan<1, 12>(ScanArgs);
template __global__ void k_scan<9, 12>(ScanArgs);
template __global__ void k_scan<9, 24>(ScanArgs);
template __global__ void k_scan<9, 48>(ScanArgs);
template __global__ void k_scan<9, 96>(ScanArgs);


}  // namespace ssla

// ---------------------------------------------------------------------------
// Host launchers
// ---------------------------------------------------------------------------
namespace ssla {

namespace {
__global__ void k_fill_f64(double* p, size_t n, double v) {
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<size_t>(gridDim.x) * blockDim.x)
        p[i] = v;
}
int grid_for(size_t n, int per_block, int cap = 148 * 16) {
    const size_t g = (n + per_block - 1) / per_block;
    return static_cast<int>(g < 1 ? 1 : (g > static_cast<size_t>(cap) ? cap : g));
}
}  // namespace


void launch_prep(cudaStream_t st, const float4* ev, int n, int W0, int H0,
                 uint32_t* ev_xy, uint8_t* rflags) {
    if (n <= 0) return;
    pdl_launch(k_prep, grid_for(n, kNT), kNT, 0, st, ev, n, W0, H0, ev_xy, rflags);
}

void launch_prep_records(cudaStream_t st, const void* rec, int n, StageEntry* E2,
                         uint32_t* ev_xy, uint8_t* rflags, float* feat) {
    if (n <= 0) return;
    k_prep_records<<<grid_for(n, kNT), kNT, 0, st>>>(static_cast<const HybridInputRec*>(rec), n,
                                                      E2, ev_xy, rflags, feat);
}

// ---------------------------------------------------------------------------
// k_records: the ring record of every event that passed gate 1 (stage-2
// list entry r): t, stage-2 coordinates, the stage-1 output feat1 -- the
// record the shard workers push after stage 1 (lib_stage01_to_gpu.cpp:
// 262-300).  seq_done / t_push_ns / t_emit_ns are left zero for the host.
// ---------------------------------------------------------------------------
__global__ void k_records(int n_cap, const int* __restrict__ count2, const StageEntry* __restrict__ E2,
                          const float4* __restrict__ ev, const float* __restrict__ feat1,
                          HybridInputRec* __restrict__ rec) {
    const int n = min(count2[0], n_cap);
    for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < n; r += gridDim.x * blockDim.x) {
        const StageEntry se = E2[r];
        HybridInputRec o;
        o.seq_done = 0;
        o.t = ev[se.e].x;
        o.x = static_cast<uint16_t>((se.xy0 & 0xFFFFu) >> 2);
        o.y = static_cast<uint16_t>((se.xy0 >> 16) >> 2);
#pragma unroll
        for (int c = 0; c < 24; ++c) o.feat1[c] = feat1[static_cast<size_t>(r) * 24 + c];
        o.t_push_ns = 0;
        o.t_emit_ns = 0;
        rec[r] = o;
    }
}

void launch_records(cudaStream_t st, int n_cap, const int* count2, const StageEntry* E2,
                    const float4* ev, const float* feat1, void* rec) {
    k_records<<<grid_for(n_cap, kNT), kNT, 0, st>>>(n_cap, count2, E2, ev, feat1,
                                                     static_cast<HybridInputRec*>(rec));
}

void launch_filter(cudaStream_t st, const FilterArgs& a0) {
    FilterArgs a = a0;
    const int s = a.stage;
    // tile rows whose lists can hold entries: a tile row t lists stage-s rows
    // [8t - 1, 8t + 8]; without a row window, all of them.  Tiles outside
    // keep count 0 (the counts are zeroed when allocated and when the window
    // is set).
    int t_lo = 0, t_hi = a.g.ty[s];
    if (a.ev_row_hi > a.ev_row_lo) {
        const int lo_s = a.ev_row_lo >> s, hi_s = ((a.ev_row_hi - 1) >> s) + 1;
        t_lo = std::max(0, (lo_s - kTile) / kTile);
        t_hi = std::min(a.g.ty[s], hi_s / kTile + 1);
    }
    if (t_hi <= t_lo) return;
    a.trow0 = t_lo;
    if (s == 0)
        pdl_launch(k_filter, dim3(a.g.P, t_hi - t_lo, a.g.nseg[0]), kNT, 0, st, a);
    else
        pdl_launch(k_filter_tiles, dim3(a.g.P, a.g.tx[s] * (t_hi - t_lo), a.g.nseg[s]), kNT, 0, st, a);
}

void launch_gates(cudaStream_t st, const GateArgs& a) {
    pdl_launch(k_gates, dim3(a.g.P, a.g.W[3] * a.g.H[3]), kGateNT, 0, st, a);
}

void launch_gates_s2(cudaStream_t st, const Gate2Args& a) {
    k_gates_s2<<<dim3(a.g.P, a.g.W[3] * a.g.H[3]), 32, 0, st>>>(a);
}

void launch_compact(cudaStream_t st, const CompactArgs& a) {
    const dim3 grid(a.g.P, a.tiles_per_part);
    pdl_launch(k_compact_count, grid, kNT, 0, st, a);
    pdl_launch(k_compact_scan, 1, kNT, 0, st, a);
    pdl_launch(k_compact_scatter, grid, kNT, 0, st, a);
}

void launch_scan(cudaStream_t st, int layer, const ScanArgs& a) {
    const int s = layer / 2;
    const dim3 grid(a.g.P, a.g.tx[s] * a.g.ty[s], (kTile * kTile) / (kNT / 32));
    switch (layer) {
        case 0: pdl_launch(k_scan<1, 12>, grid, kNT, 0, st, a); break;
        case 1: pdl_launch(k_scan<9, 12>, grid, kNT, 0, st, a); break;
        case 2: case 3: pdl_launch(k_scan<9, 24>, grid, kNT, 0, st, a); break;
        case 4: case 5: pdl_launch(k_scan<9, 48>, grid, kNT, 0, st, a); break;
        default: pdl_launch(k_scan<9, 96>, grid, kNT, 0, st, a); break;
    }
}

void launch_contrib(cudaStream_t st, int layer, const ContribArgs& a, long long max_rows) {
    auto go = [&](auto kern, auto shape) {
        using Sh = decltype(shape);
        const long long units = ((max_rows + Sh::BM - 1) / Sh::BM) * (layer == 0 ? 1 : 9);
        const int grid = static_cast<int>(std::max(1LL, std::min(units, 148LL * 16)));
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(Sh::smem));
        pdl_launch(kern, grid, kNT, Sh::smem, st, a);
    };
    switch (layer) {
        case 0: go(k_contrib<1, 12>, ContribShape<1, 12>{}); break;
        case 1: go(k_contrib<9, 12, 12>, ContribShape<9, 12, 12>{}); break;
        case 2: go(k_contrib<9, 24, 12>, ContribShape<9, 24, 12>{}); break;
        case 3: go(k_contrib<9, 24, 24>, ContribShape<9, 24, 24>{}); break;
        case 4: case 5: go(k_contrib<9, 48>, ContribShape<9, 48>{}); break;
        default: go(k_contrib<9, 96>, ContribShape<9, 96>{}); break;
    }
}

// Resident CTAs of a stage-0/1 scan kernel (computed once per kernel).
template <typename K, typename Sh>
int scan_fused_grid(K kern, Sh) {
    static int grid = 0;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(Sh::smem));
    cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    if (grid == 0) {
        int dev = 0, sms = 0, per_sm = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, Sh::NT, Sh::smem);
        grid = std::max(1, sms * std::max(1, per_sm));
    }
    return grid;
}

int scan_fused_resident_warps(int layer) {
    switch (layer) {
        case 1: return scan_fused_grid(k_scan_group<12, 12, 8, 2, 2>, ScanGroupShape<12, 12, 8, 2, 2>{}) * 8;
        case 2: return scan_fused_grid(k_scan_group<12, 24, 20, 2, 2>, ScanGroupShape<12, 24, 20, 2, 2>{}) * 20;
        default: return scan_fused_grid(k_scan_group<24, 24, 20, 2, 2>, ScanGroupShape<24, 24, 20, 2, 2>{}) * 20;
    }
}

int scan_fused_groups_per_tile(int layer, long long tile_count) {
    const long long warps = scan_fused_resident_warps(layer);
    if (layer == 1) {
        // 4x2 groups (half the list walks of 2x2) when that still leaves
        // two items per resident warp
        if (tile_count * ScanGroupShape<12, 12, 8, 4, 2>::GPT >= 2 * warps) return ScanGroupShape<12, 12, 8, 4, 2>::GPT;
        return ScanGroupShape<12, 12, 8, 2, 2>::GPT;
    }
    // layers 2-3: 2x1 groups where 2x2 groups would leave between one and
    // two items per resident warp (a second item for few warps: the tail)
    const long long g22 = tile_count * ScanGroupShape<12, 24, 20, 2, 2>::GPT;
    if (g22 >= warps && g22 < 2 * warps) return ScanGroupShape<12, 24, 20, 2, 1>::GPT;
    return ScanGroupShape<12, 24, 20, 2, 2>::GPT;
}

void launch_scan_fused(cudaStream_t st, int layer, const ScanFusedArgs& a) {
    auto go = [&](auto kern, auto shape) {
        using Sh = decltype(shape);
        const int grid = scan_fused_grid(kern, shape);
        const int s = layer / 2;
        const int items = a.g.P * a.g.tx[s] * a.g.ty[s] * 64;      // bound with every tile hot
        const int need = (items + (Sh::NT / 32) - 1) / (Sh::NT / 32);
        pdl_launch(kern, std::min(grid, need), Sh::NT, Sh::smem, st, a);
    };
    switch (layer) {
        case 1:
            if (a.gpt == ScanGroupShape<12, 12, 8, 4, 2>::GPT) go(k_scan_group<12, 12, 8, 4, 2>, ScanGroupShape<12, 12, 8, 4, 2>{});
            else go(k_scan_group<12, 12, 8, 2, 2>, ScanGroupShape<12, 12, 8, 2, 2>{});
            break;
        case 2:
            if (a.gpt == ScanGroupShape<12, 24, 20, 2, 1>::GPT) go(k_scan_group<12, 24, 20, 2, 1>, ScanGroupShape<12, 24, 20, 2, 1>{});
            else go(k_scan_group<12, 24, 20, 2, 2>, ScanGroupShape<12, 24, 20, 2, 2>{});
            break;
        default:
            if (a.gpt == ScanGroupShape<24, 24, 20, 2, 1>::GPT) go(k_scan_group<24, 24, 20, 2, 1>, ScanGroupShape<24, 24, 20, 2, 1>{});
            else go(k_scan_group<24, 24, 20, 2, 2>, ScanGroupShape<24, 24, 20, 2, 2>{});
            break;
    }
}

void launch_flag_s0(cudaStream_t st, const FilterArgs& a) {
    const long long slots = static_cast<long long>(a.g.P) * a.g.tx[0] * a.g.ty[0] * a.g.nseg[0];
    const long long blocks = std::max(1LL, std::min((slots + (kNT / 32) - 1) / (kNT / 32), 148LL * 16));
    pdl_launch(k_flag_s0, dim3(static_cast<unsigned>(blocks)), dim3(kNT), 0, st, a);
}

void launch_hot_tiles(cudaStream_t st, const HotArgs& a) {
    pdl_launch(k_hot_tiles, 1, 1024, 0, st, a);
}

void launch_ln(cudaStream_t st, int layer, const LnArgs& a, long long max_rows) {
    auto go = [&](auto kern, auto shape) {
        using Sh = decltype(shape);
        const int grid = static_cast<int>(std::max(1LL, std::min((max_rows + Sh::EV - 1) / Sh::EV, 148LL * 32)));
        pdl_launch(kern, grid, Sh::NT, 0, st, a);
    };
    switch (layer) {
        case 0: go(k_ln<1, 12>, LnShape<12>{}); break;
        case 1: go(k_ln<9, 12>, LnShape<12>{}); break;
        case 2: case 3: go(k_ln<9, 24>, LnShape<24>{}); break;
        case 4: case 5: go(k_ln<9, 48>, LnShape<48>{}); break;
        default: go(k_ln<9, 96>, LnShape<96>{}); break;
    }
}

void launch_head(cudaStream_t st, const HeadArgs& a, long long max_rows) {
    const int grid = static_cast<int>(std::max(1LL, std::min((max_rows + kMB - 1) / kMB, 148LL * 8)));
    const size_t smem = head_smem_bytes(5 + a.g.ncls);
    cudaFuncSetAttribute(k_head, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    pdl_launch(k_head, grid, kHeadNT, smem, st, a);
}

int gemm_cols(int layer, int colmode) {
    static const int kOut[8] = {12, 12, 24, 24, 48, 48, 96, 96};
    const int out2 = kOut[layer], a2 = (layer == 0) ? 1 : 9;
    switch (colmode) {
        case COLS_ALL: return a2 * 3 * out2;
        case COLS_VG: return a2 * 2 * out2;
        case COLS_Q: return a2 * out2;
        default: return out2;
    }
}

void launch_gemm(cudaStream_t st, int layer, const GemmArgs& a, long long max_rows) {
    auto go = [&](auto kern, int K, int BM, int BN) {
        const long long units = ((max_rows + BM - 1) / BM) * ((a.n_cols + BN - 1) / BN);
        const int grid = static_cast<int>(std::max(1LL, std::min(units, 148LL * 12)));
        const size_t smem = sizeof(float) * static_cast<size_t>(K) * (BM + 4 + BN);
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        pdl_launch(kern, grid, kNT, smem, st, a);
    };
    switch (layer) {                       // next layer: K = its IN, OUT2 = its OUT
        case 1: go(k_gemm<12, 12, 128, 64>, 12, 128, 64); break;
        case 2: go(k_gemm<12, 24, 128, 64>, 12, 128, 64); break;
        case 3: go(k_gemm<24, 24, 128, 64>, 24, 128, 64); break;
        case 4: go(k_gemm<24, 48, 64, 128>, 24, 64, 128); break;
        case 5: go(k_gemm<48, 48, 64, 128>, 48, 64, 128); break;
        case 6: go(k_gemm<48, 96, 64, 128>, 48, 64, 128); break;
        default: go(k_gemm<96, 96, 64, 128>, 96, 64, 128); break;
    }
}

void launch_commit(cudaStream_t st, const CommitArgs& a) {
    const int n3 = a.g.W[3] * a.g.H[3];
    pdl_launch(k_commit, dim3(a.g.P, (n3 + 7) / 8), kNT, 0, st, a);
}

void launch_reset_preds(cudaStream_t st, const Geo& g, const PartState* parts, const DevHead& hd) {
    k_reset_preds<<<g.P, 128, 0, st>>>(g, parts, hd);
}

void launch_fill_f64(cudaStream_t st, double* p, size_t n, double v) {
    if (n == 0) return;
    k_fill_f64<<<grid_for(n, kNT), kNT, 0, st>>>(p, n, v);
}

void launch_write_slots(cudaStream_t st, int n, int P, const int* rec_off, const uint8_t* rflags,
                        const uint32_t* ev_xy, const PartState* parts, const float* slot_feat,
                        void* const* outs) {
    if (n <= 0) return;
    k_write_slots<<<grid_for(n, kNT), kNT, 0, st>>>(n, P, rec_off, rflags, ev_xy, parts, slot_feat,
                                                     reinterpret_cast<HybridS2S3OutputSlot* const*>(outs));
}

void launch_fill_clk(cudaStream_t st, int P, const int* rec_off, const unsigned long long* stamps,
                     unsigned long long* const* clks) {
    k_fill_clk<<<P, kNT, 0, st>>>(P, rec_off, stamps, clks);
}

void launch_stamp(cudaStream_t st, unsigned long long* dst) { k_stamp<<<1, 1, 0, st>>>(dst); }

namespace {
// Drain results into mapped pinned host memory (zero-copy writes over the
// host link), 16 bytes per store where both sides are 16-byte aligned.
__global__ void __launch_bounds__(kNT) k_results_to_host(const uint8_t* __restrict__ flags, int n_flags,
                                                         uint8_t* flags_host, const float* __restrict__ preds,
                                                         int n_preds, float* preds_host) {
    pdl_enter();
    const int stride = gridDim.x * blockDim.x;
    const int t0 = blockIdx.x * blockDim.x + threadIdx.x;
    if (flags_host) {
        const bool vec = ((reinterpret_cast<uintptr_t>(flags_host) | reinterpret_cast<uintptr_t>(flags)) & 15) == 0;
        const int n16 = vec ? n_flags / 16 : 0;
        for (int i = t0; i < n16; i += stride)
            reinterpret_cast<uint4*>(flags_host)[i] = reinterpret_cast<const uint4*>(flags)[i];
        for (int i = n16 * 16 + t0; i < n_flags; i += stride) flags_host[i] = flags[i];
    }
    if (preds_host) {
        const bool vec = ((reinterpret_cast<uintptr_t>(preds_host) | reinterpret_cast<uintptr_t>(preds)) & 15) == 0;
        const int n4 = vec ? n_preds / 4 : 0;
        for (int i = t0; i < n4; i += stride)
            reinterpret_cast<float4*>(preds_host)[i] = reinterpret_cast<const float4*>(preds)[i];
        for (int i = n4 * 4 + t0; i < n_preds; i += stride) preds_host[i] = preds[i];
    }
}
}  // namespace

void launch_results_to_host(cudaStream_t st, const uint8_t* flags, int n_flags, uint8_t* flags_host,
                            const float* preds, int n_preds, float* preds_host) {
    const int bytes = (flags_host ? n_flags : 0) + (preds_host ? n_preds * 4 : 0);
    const int blocks = std::max(1, std::min(148, (bytes / 16 + kNT - 1) / kNT));
    pdl_launch(k_results_to_host, dim3(blocks), dim3(kNT), 0, st, flags, n_flags, flags_host, preds, n_preds,
               preds_host);
}

namespace {
// 8 independent FFMA chains per thread; a and b come from memory so nothing
// folds, the result is stored only under a never-true runtime condition.
__global__ void __launch_bounds__(512) k_ffma_peak(const float* __restrict__ ab, int iters, float* sink) {
    const float a = ab[0], b = ab[1];
    float r[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) r[k] = static_cast<float>(threadIdx.x + k);
    for (int i = 0; i < iters; ++i) {
#pragma unroll
        for (int k = 0; k < 8; ++k) r[k] = fmaf(r[k], a, b);
    }
    float s = 0.0f;
#pragma unroll
    for (int k = 0; k < 8; ++k) s += r[k];
    if (s == 123456.789f) sink[threadIdx.x] = s;
}
// ssla_rcp_rn against the IEEE round-to-nearest reciprocal for the float bit
// patterns [lo, hi): mismatches counted, the first (lowest seen) recorded.
__global__ void __launch_bounds__(256) k_rcp_check(uint32_t lo, uint32_t hi, unsigned long long* bad,
                                                   unsigned* first) {
    unsigned long long n = 0;
    for (uint64_t u = lo + static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; u < hi;
         u += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        const float y = __uint_as_float(static_cast<uint32_t>(u));
        if (__float_as_uint(ssla_rcp_rn(y)) != __float_as_uint(__frcp_rn(y))) {
            ++n;
            atomicMin(first, static_cast<unsigned>(u));
        }
    }
    if (n) atomicAdd(bad, n);
}
// ssla_sigmoidf2 against two ssla_sigmoidf calls: every float bit pattern u
// in [lo, hi) as the first component, u ^ 0x80000000 (the same magnitude,
// other sign) as the second; results compared bit for bit.
__global__ void __launch_bounds__(256) k_sigmoid2_check(uint32_t lo, uint32_t hi, unsigned long long* bad,
                                                        unsigned* first) {
    unsigned long long n = 0;
    for (uint64_t u = lo + static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; u < hi;
         u += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        const uint32_t b0 = static_cast<uint32_t>(u), b1 = b0 ^ 0x80000000u;
        const float2 x = make_float2(__uint_as_float(b0), __uint_as_float(b1));
        const float2 s = ssla_sigmoidf2(x);
        if (__float_as_uint(s.x) != __float_as_uint(ssla_sigmoidf(x.x)) ||
            __float_as_uint(s.y) != __float_as_uint(ssla_sigmoidf(x.y))) {
            ++n;
            atomicMin(first, b0);
        }
    }
    if (n) atomicAdd(bad, n);
}
}  // namespace

unsigned long long check_sigmoid_pair(unsigned* first_bad) {
    unsigned long long* d = nullptr;
    if (cudaMalloc(&d, 16) != cudaSuccess) throw std::runtime_error("cudaMalloc failed");
    unsigned long long init[2] = {0, 0xFFFFFFFFull};
    cudaMemcpy(d, init, sizeof init, cudaMemcpyHostToDevice);
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    // the 2^31 positive patterns, each paired with its negative twin
    k_sigmoid2_check<<<sms * 8, 256>>>(0x00000000u, 0x80000000u, d, reinterpret_cast<unsigned*>(d + 1));
    const cudaError_t err = cudaDeviceSynchronize();
    unsigned long long out[2] = {0, 0};
    cudaMemcpy(out, d, sizeof out, cudaMemcpyDeviceToHost);
    cudaFree(d);
    if (err != cudaSuccess) throw std::runtime_error(cudaGetErrorString(err));
    if (first_bad) *first_bad = static_cast<unsigned>(out[1]);
    return out[0];
}

unsigned long long check_reciprocal(unsigned* first_bad) {
    unsigned long long* d = nullptr;
    if (cudaMalloc(&d, 16) != cudaSuccess) throw std::runtime_error("cudaMalloc failed");
    unsigned long long init[2] = {0, 0xFFFFFFFFull};
    cudaMemcpy(d, init, sizeof init, cudaMemcpyHostToDevice);
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    // every float in [1, 2^126): the reciprocals the sigmoid takes
    k_rcp_check<<<sms * 8, 256>>>(0x3F800000u, 0x7E800000u, d, reinterpret_cast<unsigned*>(d + 1));
    const cudaError_t err = cudaDeviceSynchronize();
    unsigned long long out[2] = {0, 0};
    cudaMemcpy(out, d, sizeof out, cudaMemcpyDeviceToHost);
    cudaFree(d);
    if (err != cudaSuccess) throw std::runtime_error(cudaGetErrorString(err));
    if (first_bad) *first_bad = static_cast<unsigned>(out[1]);
    return out[0];
}

double measure_ffma_peak() {
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        return 0.0;
    float* buf = nullptr;
    if (cudaMalloc(&buf, 4096) != cudaSuccess) return 0.0;
    const float ab[2] = {0.999999f, 1e-7f};
    cudaMemcpy(buf, ab, sizeof ab, cudaMemcpyHostToDevice);
    cudaEvent_t e0, e1;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    const int iters = 1 << 16, threads = 512, blocks = sms * 4;
    double best = 0.0;
    for (int rep = 0; rep < 3; ++rep) {
        cudaEventRecord(e0);
        k_ffma_peak<<<blocks, threads>>>(buf, iters, buf + 16);
        cudaEventRecord(e1);
        cudaEventSynchronize(e1);
        float ms = 0.0f;
        cudaEventElapsedTime(&ms, e0, e1);
        const double flops = 2.0 * 8.0 * iters * static_cast<double>(threads) * blocks;
        if (ms > 0.0f && rep > 0) best = std::max(best, flops / (ms * 1e-3) / 1e12);
    }
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    cudaFree(buf);
    return best;
}

}  // namespace ssla
