// Live event loop: a resident thread-block cluster that takes raw events
// {t, x, y, p} (openeva::Event, vendor/openeva/event.h:8-13) from a ring in
// pinned host memory with the SPSC head / tail protocol (include/spsc.h:9-11,
// orin/orin/ring.py:34-152) and runs each through preprocess, the four
// tdrop gates, stages 0-3 and the head, one event at a time, writing the
// event's flags and prediction row back into pinned memory and publishing
// `events_done` -- the full-pipeline counterpart of the reference's polling
// kernel k_ssla_s2s3_celled_persistent_multi
// (orin/kernels/ssla_s2_s3_head_celled.cuh:1547-1784; tails, events_done and
// stop_flag as orin/hybrid_runner_multi.py:445-462 allocates them).
//
// The cluster (11 CTAs) keeps the weights resident across events:
//   CTA 0   coordinator: polls the ring, preprocess and gates, all of
//           stages 0-1 (layers 0-3 resident in shared memory), the residual,
//           the 9-owner gather and LayerNorm of layers 4-7;
//   CTA 1+d worker of patch position d (delta = (1-dy)*3 + (1-dx)) for
//           layers 4-7: layers 4-5 resident, 6-7 streamed by bulk copies
//           as soon as an event is known to reach stage 3;
//   CTA 10  head: the YOLOX head weights resident; writes flags, the
//           prediction row and events_done.
// CTAs exchange layer inputs, goW contributions and event messages by
// st.async into the receiver's shared memory, each completing on the
// receiver's mbarrier; completion arrivals (release at cluster scope)
// order every state write of an event before the next event's reads.
// Every wait is bounded; the loop ends on the stop flag, or by itself after
// `idle_ns` without an event, and reports why in the status word.
// Arithmetic is the step kernel's, so results are bit-identical to the
// oracle.
#include <atomic>
#include <mutex>

#include "ssla_b200.h"
#include "ssla_cluster.cuh"
#include "ssla_kernels.cuh"

namespace ssla {

namespace {

using namespace cl;

constexpr int kLiveNT = 512;
constexpr int kWorkers = 9;
constexpr int kHeadCta = 10;
constexpr int kLiveCTAs = 11;
constexpr int kIssuer = kLiveNT - 32;
constexpr unsigned kStopMsg = 0x100u;     // flag word of the message that ends the loop
constexpr unsigned long long kIdleMargin = 200ull * 1000ull * 1000ull;

// barriers (one shared-memory array, the same indices in every CTA)
enum {
    B_EV = 0,      // workers, head: event message {t, x, y, p, flags}
    B_X = 1,       // workers: layer l input, B_X + l - 4
    B_C = 5,       // coordinator: layer l contributions, B_C + l - 4
    B_DONE = 9,    // coordinator: the workers finished an event (9 arrivals)
    B_INIT = 10,   // every CTA: resident copies
    B_S6 = 11,     // workers: layer-6 copies
    B_S7Q = 12,    // workers: layer-7 qvg block
    B_S7G = 13,    // workers: layer-7 goW block
    B_FIN = 14,    // head: event finished {flags (, layer-7 output)}
    B_HDONE = 15,  // coordinator: the head CTA has taken an event's inputs
    kNBar = 16
};

// ---- shared-memory plans (floats) ------------------------------------------------
// coordinator: layers 0-3 [qvg A*IN*3*OUT][goW A*OUT*OUT][gamma][beta][input_proj]
template <int IN, int OUT, int A, bool IP>
struct SL {
    static constexpr int J2 = 3 * OUT, WQ = A * IN * J2, WG = A * OUT * OUT;
    static constexpr int GAM = WQ + WG, BET = GAM + OUT, WI = BET + OUT;
    static constexpr int size = WI + (IP ? IN * OUT : 0);
};
using SL0 = SL<2, 12, 1, true>;
using SL1 = SL<12, 12, 9, false>;
using SL2 = SL<12, 24, 9, true>;
using SL3 = SL<24, 24, 9, false>;
constexpr int kC1 = SL0::size, kC2 = kC1 + SL1::size, kC3 = kC2 + SL2::size;
constexpr int kCgb = kC3 + SL3::size;          // gamma | beta of layers 4-7 (48, 48, 96, 96)
constexpr int kCip4 = kCgb + 2 * (48 + 48 + 96 + 96);
constexpr int kCip6 = kCip4 + 24 * 48;
constexpr int kCscr = kCip6 + 48 * 96;         // layers 0-3 scratch: qvg values | q*h | contributions
constexpr int kCcon = kCscr + 9 * 72 + 9 * 24 + 9 * 24;   // layers 4-7 contributions [9][96]
constexpr int kCres = kCcon + 9 * 96;          // residual [96]
constexpr int kCend = kCres + 96;
// workers: layers 4-5 resident (qvg | goW of the position), one stream area
// for layer 6 then 7: qvg block at its start, goW block at kWSg.
constexpr int kW5 = 24 * 144 + 48 * 48;
constexpr int kWS = kW5 + 48 * 144 + 48 * 48;
constexpr int kWSg = kWS + 96 * 288;
constexpr int kWend = kWSg + 96 * 96;
// head: cls conv | reg conv [96][96], reg pred [96][4], obj pred [96],
// cls pred [96][ncls], cls | reg conv biases; activations after it.
constexpr int kHeadRp = 2 * 96 * 96, kHeadOb = kHeadRp + 96 * 4, kHeadCp = kHeadOb + 96;
__host__ __device__ constexpr int head_cb(int ncls) { return kHeadCp + 96 * ncls; }
__host__ __device__ constexpr int head_act(int ncls) { return head_cb(ncls) + 192; }
constexpr int kDyn = kCend > kWend ? kCend : kWend;
static_assert(kC1 % 4 == 0 && kC2 % 4 == 0 && kC3 % 4 == 0 && kCgb % 4 == 0 && kCip4 % 4 == 0 &&
                  kCip6 % 4 == 0 && kCcon % 4 == 0 && kCres % 4 == 0 && kW5 % 4 == 0 && kWS % 4 == 0 && kWSg % 4 == 0,
              "16-byte aligned buffers");

__host__ __device__ constexpr int gb_off(int l) { return l == 4 ? 0 : l == 5 ? 96 : l == 6 ? 192 : 384; }

struct LiveShared {
    uint64_t bar[kNBar];
    float ev[5];        // event message: t, x, y, p, flag word
    float fin;          // head: flag word of the finished event
    __align__(16) float x[96];      // layer input (coordinator: own; worker: received)
    __align__(16) float xh[2][96];  // head: layer-7 output, by event parity
    __align__(16) float qvg[288];   // worker: q | v | g of its cell
    __align__(16) float qh[96];     // worker: q * h
    float4 e;           // coordinator: the event taken from the ring
    int cmd;            // coordinator: 0 event, 1 stop flag, 2 idle
    int flags;          // coordinator: the event's flags
    // bulk copy in flight on barrier i: 0 none, else 1 + the parity of the
    // phase it completes (set by the issuing thread, cleared by thread 0
    // once that phase has been waited for)
    uint8_t inflight[kNBar];
};
static_assert(sizeof(LiveShared) + sizeof(float) * kDyn <= kMaxBlockSmem, "shared memory");

__device__ __forceinline__ bool wait_bar(LiveShared& sh, int i, uint32_t& ph, unsigned* err, unsigned code,
                                         unsigned long long limit = kWaitNs) {
    const bool ok = mbar_wait(&sh.bar[i], (ph >> i) & 1u, err, code, limit);
    if (ok && threadIdx.x == 0 && sh.inflight[i]) sh.inflight[i] = 0;
    ph ^= 1u << i;
    return ok;
}

// The issuing thread records a bulk copy completing on barrier i (before
// issuing it): the copy lands in the phase this thread waits for next.
__device__ __forceinline__ void mark_copy(LiveShared& sh, int i, uint32_t ph) {
    sh.inflight[i] = static_cast<uint8_t>(1u + ((ph >> i) & 1u));
}

// Every CTA leaves through here, on every path (stop, idle, or a wait that
// ran out): no bulk copy of its own may still be writing its shared memory
// (bounded wait for each one recorded in flight), and no CTA returns
// before every other CTA of the cluster has stopped sending messages and
// remote arrivals into it (cluster barrier; every earlier wait is bounded,
// so every CTA gets here).
__device__ void live_exit(LiveShared& sh) {
    __syncthreads();
    if (threadIdx.x == 0)
        for (int i = 0; i < kNBar; ++i)
            if (sh.inflight[i]) mbar_wait(&sh.bar[i], sh.inflight[i] - 1u, nullptr, 0u);
    __syncthreads();
    cluster_arrive();
    cluster_wait();
}

// ---- system-scope accesses to the ring (pinned host memory) -----------------------
__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys(unsigned long long* p, unsigned long long v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ int ld_volatile(const int* p) {
    int v;
    asm volatile("ld.volatile.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ float4 ld_volatile4(const float4* p) {
    float4 v;
    asm volatile("ld.volatile.global.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(p)
                 : "memory");
    return v;
}

// ---- resident copies ----------------------------------------------------------------------
template <int IN, int OUT, int A, bool IP>
__device__ void issue_small_res(const DevLayer& L, float* b, uint64_t* bar) {
    using S = SL<IN, OUT, A, IP>;
    bulk(b, L.qvgT, S::WQ, bar);
    bulk(b + S::WQ, L.goWT, S::WG, bar);
    bulk(b + S::GAM, L.gamma, OUT, bar);
    bulk(b + S::BET, L.beta, OUT, bar);
    if (IP) bulk(b + S::WI, L.ipT, IN * OUT, bar);
}

__device__ void issue_resident(int rank, const LiveArgs& a, float* wsm, uint64_t* bar) {
    if (rank == 0) {
        issue_small_res<2, 12, 1, true>(a.L[0], wsm, bar);
        issue_small_res<12, 12, 9, false>(a.L[1], wsm + kC1, bar);
        issue_small_res<12, 24, 9, true>(a.L[2], wsm + kC2, bar);
        issue_small_res<24, 24, 9, false>(a.L[3], wsm + kC3, bar);
        for (int l = 4; l < 8; ++l) {
            const int OUT = chans(l / 2);
            bulk(wsm + kCgb + gb_off(l), a.L[l].gamma, OUT, bar);
            bulk(wsm + kCgb + gb_off(l) + OUT, a.L[l].beta, OUT, bar);
        }
        bulk(wsm + kCip4, a.L[4].ipT, 24 * 48, bar);
        bulk(wsm + kCip6, a.L[6].ipT, 48 * 96, bar);
    } else if (rank == kHeadCta) {
        const DevHead& hd = a.head;
        const int ncls = a.g.ncls;
        bulk(wsm, hd.cls_convT, 96 * 96, bar);
        bulk(wsm + 96 * 96, hd.reg_convT, 96 * 96, bar);
        bulk(wsm + kHeadRp, hd.reg_predT, 96 * 4, bar);
        bulk(wsm + kHeadOb, hd.obj_predT, 96, bar);
        bulk(wsm + kHeadCp, hd.cls_predT, 96 * ncls, bar);
        bulk(wsm + head_cb(ncls), hd.cls_conv_b, 96, bar);
        bulk(wsm + head_cb(ncls) + 96, hd.reg_conv_b, 96, bar);
    } else {
        const int d = rank - 1;
        bulk(wsm, a.L[4].qvgT + static_cast<size_t>(d) * 24 * 144, 24 * 144, bar);
        bulk(wsm + 24 * 144, a.L[4].goWT + static_cast<size_t>(d) * 48 * 48, 48 * 48, bar);
        bulk(wsm + kW5, a.L[5].qvgT + static_cast<size_t>(d) * 48 * 144, 48 * 144, bar);
        bulk(wsm + kW5 + 48 * 144, a.L[5].goWT + static_cast<size_t>(d) * 48 * 48, 48 * 48, bar);
    }
    mbar_arrive(bar);
}

// ---- gather + LayerNorm (warp 0 of the coordinator) -------------------------------
// y[t] = (sum over in-bounds positions d = A-1..0 of con[d][t]) + res[t],
// lane g holding channels 4g..4g+3; x = LN(y) into sh.x and, when `bmask`
// has bits, to those CTAs' sh.x (completing on their barrier `bar_next`).
template <int OUT, int A>
__device__ __forceinline__ void gather_ln(LiveShared& sh, const float* con, int cstride, unsigned inb,
                                          const float* res, const float* gam, const float* bet, int bar_next,
                                          unsigned bmask) {
    const int g = threadIdx.x & 31;
    float4 y = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    if (g < OUT / 4) {
#pragma unroll
        for (int d = A - 1; d >= 0; --d)
            if ((inb >> d) & 1u) {
                const float4 c = *reinterpret_cast<const float4*>(con + d * cstride + 4 * g);
                y.x = y.x + c.x;
                y.y = y.y + c.y;
                y.z = y.z + c.z;
                y.w = y.w + c.w;
            }
        const float4 r = *reinterpret_cast<const float4*>(res + 4 * g);
        y.x = y.x + r.x;
        y.y = y.y + r.y;
        y.z = y.z + r.z;
        y.w = y.w + r.w;
    }
    const float4 x = ln4<OUT>(y, gam, bet);
    if (g < OUT / 4) {
        *reinterpret_cast<float4*>(sh.x + 4 * g) = x;
        for (int r = 1; r < kLiveCTAs; ++r)
            if ((bmask >> r) & 1u) send4(sh.x + 4 * g, &sh.bar[bar_next], r, x);
    }
}

// ---- coordinator: layers 0-3 ---------------------------------------------------------------
// Every patch position: (position, 4-column group) items form q, v,
// sigmoid(g), (position, channel) items update the cells (their rows were
// loaded at the event's start into `hr`), (position, 4-channel group) items
// form the goW contributions; warp 0 sums, adds the residual and
// normalises.  Returns false when the layer is the event's last.
template <int IN, int OUT, int A, bool IP>
__device__ bool c_small(int l, const Plan& P, const LiveArgs& a, LiveShared& sh, float* wsm, int base, float hr,
                        unsigned bmask) {
    using S = SL<IN, OUT, A, IP>;
    constexpr int J2 = S::J2, G2 = J2 / 4, GO = OUT / 4;
    const int tid = threadIdx.x;
    const int s = l / 2;
    const bool used = P.used(l);
    const unsigned inb = A > 1 ? P.inb(l) : 1u;
    const float* wq = wsm + base;
    const float* wg = wq + S::WQ;
    const float* wi = wq + S::WI;
    float* qvg = wsm + kCscr;
    float* qh = qvg + 9 * 72;
    float* con = qh + 9 * 24;
    float* res = wsm + kCres;
    const float4 z4 = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    if (used && tid < GO)
        *reinterpret_cast<float4*>(res + 4 * tid) =
            IP ? dot4<IN>(wi + 4 * tid, OUT, sh.x, z4) : *reinterpret_cast<const float4*>(sh.x + 4 * tid);
    const int g0 = used ? 0 : GO;
    for (int it = tid; it < A * (G2 - g0); it += kLiveNT) {
        const int d = it / (G2 - g0), c = 4 * (g0 + it % (G2 - g0));
        if (!((inb >> d) & 1u)) continue;
        *reinterpret_cast<float4*>(qvg + d * J2 + c) = dot4<IN>(wq + d * IN * J2 + c, J2, sh.x, z4);
    }
    __syncthreads();
    const int hd = tid / OUT, ht = tid % OUT;
    const bool hact = tid < A * OUT && ((inb >> hd) & 1u);
    float h = 0.0f;
    if (hact) {
        const float* q = qvg + hd * J2;
        h = fmaf(ssla_sigmoidf(q[2 * OUT + ht]), hr, q[OUT + ht]);
        if (used) qh[hd * OUT + ht] = q[ht] * h;
    }
    if (used) {
        __syncthreads();
        if (tid < A * GO) {
            const int d = tid / GO, t = 4 * (tid % GO);
            if ((inb >> d) & 1u)
                *reinterpret_cast<float4*>(con + d * OUT + t) = dot4<OUT>(wg + d * OUT * OUT + t, OUT, qh + d * OUT, z4);
        }
    }
    if (hact) {
        int cx, cy;
        patch_cell(A, hd, P.px >> s, P.py >> s, a.g.W[s], a.g.H[s], cx, cy);
        a.ps.hidden[l][(static_cast<size_t>(cy) * a.g.W[s] + cx) * OUT + ht] = h;
    }
    __syncthreads();
    if (!used) return false;                     // state-only second layer: the event ends
    if (tid < 32) gather_ln<OUT, A>(sh, con, OUT, inb, res, wq + S::GAM, wq + S::BET, B_X, bmask);
    __syncthreads();
    return true;
}

// Coordinator part of layer l (4-7), output used: residual, contributions of
// the in-bounds positions, gather + LayerNorm; the output goes on to the
// workers of layer l+1.
template <int IN, int OUT>
__device__ bool c_big(int l, const Plan& P, const LiveArgs& a, LiveShared& sh, float* wsm, uint32_t& ph) {
    const int tid = threadIdx.x;
    float* res = wsm + kCres;
    if (tid < OUT / 4) {
        const float4 z4 = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        *reinterpret_cast<float4*>(res + 4 * tid) =
            (l & 1) == 0 ? dot4<IN>(wsm + (l == 4 ? kCip4 : kCip6) + 4 * tid, OUT, sh.x, z4)
                         : *reinterpret_cast<const float4*>(sh.x + 4 * tid);
    }
    const bool ok = wait_bar(sh, B_C + l - 4, ph, a.err, SSLA_LIVE_ERR_CONTRIB);
    __syncthreads();
    if (tid < 32) {
        const unsigned bmask = (l < 7 && P.runs(l + 1)) ? (P.inb(l + 1) << 1) : 0u;
        const float* gb = wsm + kCgb + gb_off(l);
        gather_ln<OUT, 9>(sh, wsm + kCcon, 96, P.inb(l), res, gb, gb + OUT, B_X + (l + 1) - 4, bmask);
    }
    __syncthreads();
    return ok;
}

// Thread 0 of the coordinator: waits for the next event of the ring.
// Returns 0 with the event, 1 when the stop flag is set, 2 after idle_ns.
__device__ int poll_event(const LiveArgs& a, unsigned long long seq, float4& e) {
    const unsigned long long t0 = gtime();
    for (;;) {
        if (ld_acquire_sys(a.head_idx) > seq) {
            e = ld_volatile4(a.events + (seq & a.mask));
            st_release_sys(a.tail, seq + 1);
            return 0;
        }
        if (ld_volatile(a.stop) != 0) return 1;
        if (gtime() - t0 > a.idle_ns) return 2;
    }
}

__device__ void coordinator(const LiveArgs& a, LiveShared& sh, float* wsm, uint32_t& ph) {
    const int tid = threadIdx.x;
    const Geo& g = a.g;
    const PartState& ps = a.ps;
    const bool hyb = g.layout == LAYOUT_HYBRID;
    bool pending = false;              // the head CTA's acknowledgement of the last event is outstanding
    bool done_pending = false;         // the workers' completion of the last event is outstanding
    for (unsigned long long seq = a.start;; ++seq) {
        if (tid == 0) {
            float4 e;
            sh.cmd = poll_event(a, seq, e);
            sh.e = e;
        }
        __syncthreads();
        const int cmd = sh.cmd;
        if (cmd != 0) {
            if (done_pending) wait_bar(sh, B_DONE, ph, a.err, SSLA_LIVE_ERR_DONE);
            if (pending) wait_bar(sh, B_HDONE, ph, a.err, SSLA_LIVE_ERR_DONE);
            if (tid >= 32 && tid < 32 + kLiveCTAs - 1) {
                const int r = tid - 31;
                send(&sh.ev[4], &sh.bar[B_EV], r, __uint_as_float(kStopMsg));
                for (int i = 0; i < 4; ++i) send(&sh.ev[i], &sh.bar[B_EV], r, 0.0f);
            }
            if (tid == 0 && a.err) atomicOr_system(a.err, cmd == 1 ? SSLA_LIVE_EXIT_STOP : SSLA_LIVE_EXIT_IDLE);
            return;
        }
        const float4 e = sh.e;
        const bool valid = e.y > -1.0f && e.y < static_cast<float>(g.W[0]) && e.z > -1.0f &&
                           e.z < static_cast<float>(g.H[0]);
        const int px = valid ? static_cast<int>(e.y) : 0, py = valid ? static_cast<int>(e.z) : 0;
        // the state rows of layers 0-3 this thread updates, loaded up front
        float hr[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        if (valid) {
#pragma unroll
            for (int l = 0; l < 4; ++l) {
                const int s = l / 2, OUT = chans(s), A = l == 0 ? 1 : 9;
                if (tid < A * OUT) {
                    int cx, cy;
                    if (patch_cell(A, tid / OUT, px >> s, py >> s, g.W[s], g.H[s], cx, cy))
                        hr[l] = ps.hidden[l][(static_cast<size_t>(cy) * g.W[s] + cx) * OUT + tid % OUT];
                }
            }
        }
        if (tid == 0) {
            int k[4];
            gate_cells(g, px, py, k);
            int c[4] = {0, 0, 0, 0};
            double lt = 0.0;
            if (valid) {
                c[0] = ps.cnt[0][k[0]];
                c[1] = ps.cnt[1][k[1]];
                c[2] = ps.cnt[2][k[2]];
                if (hyb) c[3] = ps.cnt[3][k[3]];
                lt = ps.last_t[py * g.W[0] + px];
            }
            const int flags = gate_flags(valid, c, g.window, hyb);
            if (valid) {
                ps.last_t[py * g.W[0] + px] = static_cast<double>(e.x);
                ps.cnt[0][k[0]] = static_cast<uint8_t>(c[0] + 1);
                if (flags & F_R1) ps.cnt[1][k[1]] = static_cast<uint8_t>(c[1] + 1);
                if (flags & F_R2) ps.cnt[2][k[2]] = static_cast<uint8_t>(c[2] + 1);
                if (hyb && (flags & F_R3)) ps.cnt[3][k[3]] = static_cast<uint8_t>(c[3] + 1);
            }
            sh.flags = flags;
            sh.x[0] = dt_norm(lt, e.x);
            sh.x[1] = e.w;
        }
        __syncthreads();
        const int flags = sh.flags;
        Plan P;
        make_plan(P, flags, px, py, g);
        if (tid == 0)
            for (int l = 4; l < 8; ++l)
                if (P.used(l)) mbar_arrive_tx(&sh.bar[B_C + l - 4], 4u * chans(l / 2) * __popc(P.inb(l)));
        // the event message, once the workers are done with the previous event
        // and the head CTA has taken its inputs
        bool acked = true;
        if (done_pending) acked = wait_bar(sh, B_DONE, ph, a.err, SSLA_LIVE_ERR_DONE) && acked;
        if (pending) acked = wait_bar(sh, B_HDONE, ph, a.err, SSLA_LIVE_ERR_DONE) && acked;
        if (!__syncthreads_and(acked)) return;       // the loop cannot go on: the status word says why
        pending = true;
        if (tid >= 32 && tid < 32 + kLiveCTAs - 1) {
            const int r = tid - 31;
            send(&sh.ev[0], &sh.bar[B_EV], r, e.x);
            send(&sh.ev[1], &sh.bar[B_EV], r, e.y);
            send(&sh.ev[2], &sh.bar[B_EV], r, e.z);
            send(&sh.ev[3], &sh.bar[B_EV], r, e.w);
            send(&sh.ev[4], &sh.bar[B_EV], r, __int_as_float(flags));
        }
        // ---- layers 0-3 ----
        bool ok = true;
        if (P.runs(0) && c_small<2, 12, 1, true>(0, P, a, sh, wsm, 0, hr[0], 0u) &&
            c_small<12, 12, 9, false>(1, P, a, sh, wsm, kC1, hr[1], 0u) &&
            c_small<12, 24, 9, true>(2, P, a, sh, wsm, kC2, hr[2], 0u)) {
            const unsigned b4 = P.runs(4) ? (P.inb(4) << 1) : 0u;
            if (c_small<24, 24, 9, false>(3, P, a, sh, wsm, kC3, hr[3], b4)) {
                // ---- layers 4-7 ----
                for (int l = 4; l < 8 && P.used(l) && ok; ++l) {
                    switch (l) {
                        case 4: ok = c_big<24, 48>(4, P, a, sh, wsm, ph); break;
                        case 5: ok = c_big<48, 48>(5, P, a, sh, wsm, ph); break;
                        case 6: ok = c_big<48, 96>(6, P, a, sh, wsm, ph); break;
                        default: ok = c_big<96, 96>(7, P, a, sh, wsm, ph); break;
                    }
                }
            }
        }
        // ---- once the workers' state writes are done the head CTA finishes the
        // event; when no worker took part, their acknowledgement can wait ----
        if (P.runs(4)) ok = wait_bar(sh, B_DONE, ph, a.err, SSLA_LIVE_ERR_DONE) && ok;
        done_pending = !P.runs(4);
        if (tid < 32 && seq != a.withhold_fin) {
            if (flags & F_R4)
                for (int t = tid; t < 96; t += 32) send(&sh.xh[seq & 1][t], &sh.bar[B_FIN], kHeadCta, sh.x[t]);
            if (tid == 0) send(&sh.fin, &sh.bar[B_FIN], kHeadCta, __int_as_float(flags));
        }
        if (!__syncthreads_and(ok)) return;   // a wait ran out: the status word says which
    }
}

// ---- workers: layers 4-7 of patch position d ------------------------------------------------
__device__ __forceinline__ const float* w_qvg(float* wsm, int l) {
    return wsm + (l == 4 ? 0 : l == 5 ? kW5 : kWS);
}
__device__ __forceinline__ const float* w_goW(float* wsm, int l) {
    return l == 4 ? wsm + 24 * 144 : l == 5 ? wsm + kW5 + 48 * 144 : wsm + kWSg;
}

template <int IN, int OUT>
__device__ bool w_layer(int l, int d, const Plan& P, const LiveArgs& a, LiveShared& sh, float* wsm, float hr,
                        uint32_t& ph, bool issue7q, bool issue7g) {
    constexpr int J2 = 3 * OUT;
    const int tid = threadIdx.x;
    const bool used = P.used(l);
    bool ok = wait_bar(sh, B_X + l - 4, ph, a.err, SSLA_LIVE_ERR_INPUT);
    if (l == 6) ok = wait_bar(sh, B_S6, ph, a.err, SSLA_LIVE_ERR_WEIGHTS) && ok;
    if (l == 7) ok = wait_bar(sh, B_S7Q, ph, a.err, SSLA_LIVE_ERR_WEIGHTS) && ok;
    const float* wq = w_qvg(wsm, l);
    {
        const int col = (used ? 0 : OUT) + tid;   // state-only: v and g columns
        if (col < J2) sh.qvg[col] = dot1<IN>(wq + col, J2, sh.x, 0.0f);
    }
    __syncthreads();
    if (l == 6 && issue7q && tid == kIssuer) {         // layer 6's qvg block is consumed
        mark_copy(sh, B_S7Q, ph);
        bulk(wsm + kWS, a.L[7].qvgT + static_cast<size_t>(d) * 96 * 288, 96 * 288, &sh.bar[B_S7Q]);
        mbar_arrive(&sh.bar[B_S7Q]);
    }
    float h = 0.0f;
    if (tid < OUT) {
        h = fmaf(ssla_sigmoidf(sh.qvg[2 * OUT + tid]), hr, sh.qvg[OUT + tid]);
        if (used) sh.qh[tid] = sh.qvg[tid] * h;
    }
    if (used) {
        __syncthreads();
        if (l == 7) ok = wait_bar(sh, B_S7G, ph, a.err, SSLA_LIVE_ERR_WEIGHTS) && ok;
        if (tid < OUT) send(wsm + kCcon + d * 96 + tid, &sh.bar[B_C + l - 4], 0, dot1<OUT>(w_goW(wsm, l) + tid, OUT, sh.qh, 0.0f));
    }
    if (tid < OUT) {
        const int s = l / 2;
        int cx, cy;
        patch_cell(9, d, P.px >> s, P.py >> s, a.g.W[s], a.g.H[s], cx, cy);
        a.ps.hidden[l][(static_cast<size_t>(cy) * a.g.W[s] + cx) * OUT + tid] = h;
    }
    __syncthreads();                   // this layer's buffers are consumed
    if (l == 6 && issue7g && tid == kIssuer) {
        mark_copy(sh, B_S7G, ph);
        bulk(wsm + kWSg, a.L[7].goWT + static_cast<size_t>(d) * 96 * 96, 96 * 96, &sh.bar[B_S7G]);
        mbar_arrive(&sh.bar[B_S7G]);
    }
    return ok;
}

__device__ void worker(int d, const LiveArgs& a, LiveShared& sh, float* wsm, uint32_t& ph) {
    const int tid = threadIdx.x;
    const Geo& g = a.g;
    for (;;) {
        if (tid == 0) mbar_arrive_tx(&sh.bar[B_EV], 20u);
        if (!__syncthreads_and(wait_bar(sh, B_EV, ph, a.err, SSLA_LIVE_ERR_EVENT, a.idle_ns + kIdleMargin)))
            return;
        const unsigned fw = __float_as_uint(sh.ev[4]);
        if (fw & kStopMsg) return;
        const float4 e = make_float4(sh.ev[0], sh.ev[1], sh.ev[2], sh.ev[3]);
        const int flags = static_cast<int>(fw);
        const int px = (flags & F_VALID) ? static_cast<int>(e.y) : 0;
        const int py = (flags & F_VALID) ? static_cast<int>(e.z) : 0;
        Plan P;
        make_plan(P, flags, px, py, g);
        bool act[8];
        float hr[8];
#pragma unroll
        for (int l = 4; l < 8; ++l) {
            act[l] = P.runs(l) && ((P.inb(l) >> d) & 1u);
            hr[l] = 0.0f;
            const int s = l / 2, OUT = chans(s);
            if (act[l] && tid < OUT) {
                int cx, cy;
                patch_cell(9, d, px >> s, py >> s, g.W[s], g.H[s], cx, cy);
                hr[l] = a.ps.hidden[l][(static_cast<size_t>(cy) * g.W[s] + cx) * OUT + tid];
            }
        }
        if (tid == 0)
            for (int l = 4; l < 8; ++l)
                if (act[l]) mbar_arrive_tx(&sh.bar[B_X + l - 4], 4u * (l == 4 ? 24 : l == 7 ? 96 : 48));
        if (tid == kIssuer) {
            if (act[6]) {
                mark_copy(sh, B_S6, ph);
                bulk(wsm + kWS, a.L[6].qvgT + static_cast<size_t>(d) * 48 * 288, 48 * 288, &sh.bar[B_S6]);
                bulk(wsm + kWSg, a.L[6].goWT + static_cast<size_t>(d) * 96 * 96, 96 * 96, &sh.bar[B_S6]);
                mbar_arrive(&sh.bar[B_S6]);
            } else if (act[7]) {       // the stream area is free now
                mark_copy(sh, B_S7Q, ph);
                bulk(wsm + kWS, a.L[7].qvgT + static_cast<size_t>(d) * 96 * 288, 96 * 288, &sh.bar[B_S7Q]);
                mbar_arrive(&sh.bar[B_S7Q]);
                if (P.used(7)) {
                    mark_copy(sh, B_S7G, ph);
                    bulk(wsm + kWSg, a.L[7].goWT + static_cast<size_t>(d) * 96 * 96, 96 * 96, &sh.bar[B_S7G]);
                    mbar_arrive(&sh.bar[B_S7G]);
                }
            }
        }
        bool ok = true;
        for (int l = 4; l < 8 && P.runs(l); ++l) {
            if (act[l]) {
                switch (l) {
                    case 4: ok = w_layer<24, 48>(4, d, P, a, sh, wsm, hr[4], ph, false, false) && ok; break;
                    case 5: ok = w_layer<48, 48>(5, d, P, a, sh, wsm, hr[5], ph, false, false) && ok; break;
                    case 6:
                        ok = w_layer<48, 96>(6, d, P, a, sh, wsm, hr[6], ph, act[7], act[7] && P.used(7)) && ok;
                        break;
                    default: ok = w_layer<96, 96>(7, d, P, a, sh, wsm, hr[7], ph, false, false) && ok; break;
                }
            }
            if (!P.used(l)) break;
        }
        const bool all_ok = __syncthreads_and(ok);   // every state row of the event is written
        if (tid == 0) mbar_arrive_remote(&sh.bar[B_DONE], 0);
        if (!all_ok) return;
    }
}

// ---- head CTA ---------------------------------------------------------------------------------
// async_yolox.h:203-254: cls / reg convs with SiLU, then the 2 + 4 + 1
// predictions; the decoded row goes to the owned cell (raw row beside it)
// and to the ring's output slot.
__device__ void head_cta(const LiveArgs& a, LiveShared& sh, float* wsm, uint32_t& ph) {
    const int tid = threadIdx.x;
    const Geo& g = a.g;
    const PartState& ps = a.ps;
    const int ncls = g.ncls, cols = 5 + ncls;
    float pbias = 0.0f;
    if (tid < cols)
        pbias = tid < 4 ? __ldg(a.head.reg_pred_b + tid)
                        : tid == 4 ? __ldg(a.head.obj_pred_b) : __ldg(a.head.cls_pred_b + (tid - 5));
    const float* h = wsm;
    float* act = wsm + head_act(ncls);
    for (unsigned long long seq = a.start;; ++seq) {
        if (tid == 0) mbar_arrive_tx(&sh.bar[B_EV], 20u);
        if (!__syncthreads_and(wait_bar(sh, B_EV, ph, a.err, SSLA_LIVE_ERR_EVENT, a.idle_ns + kIdleMargin)))
            return;
        const unsigned fw = __float_as_uint(sh.ev[4]);
        if (fw & kStopMsg) return;
        const int flags = static_cast<int>(fw);
        const int px = (flags & F_VALID) ? static_cast<int>(sh.ev[1]) : 0;
        const int py = (flags & F_VALID) ? static_cast<int>(sh.ev[2]) : 0;
        const bool head = (flags & F_R4) != 0;
        if (tid == 0) mbar_arrive_tx(&sh.bar[B_FIN], head ? 4u + 96u * 4u : 4u);
        // every thread has taken the event message
        if (!__syncthreads_and(wait_bar(sh, B_FIN, ph, a.err, SSLA_LIVE_ERR_DONE, a.idle_ns + kIdleMargin)))
            return;
        if (tid == 0) mbar_arrive_remote_relaxed(&sh.bar[B_HDONE], 0);
        const float* x = sh.xh[seq & 1];
        const unsigned long long slot = seq & a.mask;
        if (head) {
            if (tid < 48) {                // cls | reg conv, 4 outputs per thread, SiLU
                const int j = 4 * tid;
                const float* Wt = h + (j < 96 ? 0 : 96 * 96) + (j % 96);
                float4 acc = dot4<96>(Wt, 96, x, *reinterpret_cast<const float4*>(h + head_cb(ncls) + j));
                acc.x = acc.x * ssla_sigmoidf(acc.x);
                acc.y = acc.y * ssla_sigmoidf(acc.y);
                acc.z = acc.z * ssla_sigmoidf(acc.z);
                acc.w = acc.w * ssla_sigmoidf(acc.w);
                *reinterpret_cast<float4*>(act + j) = acc;
            }
            __syncthreads();
            float v = 0.0f;
            if (tid < cols) {
                if (tid < 4) v = dot1<96>(h + kHeadRp + tid, 4, act + 96, pbias);
                else if (tid == 4) v = dot1<96>(h + kHeadOb, 1, act + 96, pbias);
                else v = dot1<96>(h + kHeadCp + (tid - 5), ncls, act, pbias);
                const int c3x = px >> 3, c3y = py >> 3;
                const int x2 = px >> 2, y2 = py >> 2;
                const bool own = x2 >= ps.own_x0 && x2 < ps.own_x1 && y2 >= ps.own_y0 && y2 < ps.own_y1;
                const int cell = c3y * g.W[3] + c3x;
                const int r = tid;
                float dv;
                if (r == 0) dv = (v + static_cast<float>(c3x)) * static_cast<float>(g.stride_w);
                else if (r == 1) dv = (v + static_cast<float>(c3y)) * static_cast<float>(g.stride_h);
                else if (r == 2) dv = ssla_expf(v) * static_cast<float>(g.stride_w);
                else if (r == 3) dv = ssla_expf(v) * static_cast<float>(g.stride_h);
                else dv = v;
                if (a.preds_out) a.preds_out[slot * cols + r] = dv;
                if (own) {
                    ps.preds_dec[static_cast<size_t>(cell) * cols + r] = dv;
                    ps.preds_raw[static_cast<size_t>(cell) * cols + r] = v;
                    if (r == 0) ps.version[cell] += 1u;
                }
            }
        }
        if (tid == 0 && a.flags_out) a.flags_out[slot] = static_cast<uint8_t>(flags);
        __syncthreads();
        if (tid == 0) st_release_sys(a.done, seq + 1);   // outputs and state of the event are visible
    }
}

__global__ void __launch_bounds__(kLiveNT, 1) k_live(LiveArgs a) {
    __shared__ __align__(16) LiveShared sh;
    extern __shared__ __align__(128) float wsm[];
    const int rank = static_cast<int>(cta_rank());
    const int tid = threadIdx.x;
    if (tid == 0) {
        for (int i = 0; i < kNBar; ++i) {
            mbar_init(&sh.bar[i], i == B_DONE ? kWorkers : 1);
            sh.inflight[i] = 0;
        }
        fence_mbar_init();
    }
    __syncthreads();
    if (tid == kIssuer) {
        mark_copy(sh, B_INIT, 0u);
        issue_resident(rank, a, wsm, &sh.bar[B_INIT]);
    }
    cluster_arrive();                  // every CTA's barriers exist before any message
    cluster_wait();
    uint32_t ph = 0;
    if (__syncthreads_and(wait_bar(sh, B_INIT, ph, a.err, SSLA_LIVE_ERR_WEIGHTS))) {
        if (rank == 0) coordinator(a, sh, wsm, ph);
        else if (rank == kHeadCta) head_cta(a, sh, wsm, ph);
        else worker(rank - 1, a, sh, wsm, ph);
    }
    live_exit(sh);
}

}  // namespace

int live_max_ncls() { return (kDyn - head_act(0) - 192) / 96; }

cudaError_t launch_live(cudaStream_t st, const LiveArgs& a) {
    constexpr size_t smem = sizeof(float) * kDyn;
    if (head_act(a.g.ncls) + 192 > kDyn) return cudaErrorInvalidValue;
    static std::mutex mu;
    static unsigned long long attr_done = 0;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(kLiveCTAs);
    cfg.blockDim = dim3(kLiveNT);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = kLiveCTAs;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    {
        std::lock_guard<std::mutex> lk(mu);
        const unsigned long long bit = 1ull << (dev & 63);
        if (!(attr_done & bit)) {
            e = cudaFuncSetAttribute(k_live, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
            if (e == cudaSuccess)
                e = cudaFuncSetAttribute(k_live, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
            int nclusters = 0;
            if (e == cudaSuccess) e = cudaOccupancyMaxActiveClusters(&nclusters, k_live, &cfg);
            if (e == cudaSuccess && nclusters < 1) e = cudaErrorInvalidConfiguration;
            if (e != cudaSuccess) return e;
            attr_done |= bit;
        }
    }
    return cudaLaunchKernelEx(&cfg, k_live, a);
}

}  // namespace ssla
