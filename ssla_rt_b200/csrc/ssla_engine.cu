// ssla_engine.cu -- host side of the B200 engine and the C ABI of
// include/ssla_b200.h.
//
// An SslaEngine owns the device copy of one model (weights reshaped at load
// time), per-partition recurrent state and a workspace sized for one drain
// call.  A drain enqueues the fixed kernel sequence of ssla_kernels.cu on the
// caller's stream; every size the kernels need beyond the host-known event
// counts lives on the device, so the sequence never synchronises.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <string>
#include <chrono>
#include <thread>
#include <time.h>
#include <vector>

#include "ssla_b200.h"
#include "ssla_kernels.cuh"
#include "ssla_weights.h"

namespace ssla {
namespace {

thread_local std::string g_last_error;

struct CudaError : std::runtime_error {
    explicit CudaError(const std::string& m) : std::runtime_error(m) {}
};

#define SSLA_CK(call)                                                                   \
    do {                                                                                \
        const cudaError_t e_ = (call);                                                  \
        if (e_ != cudaSuccess)                                                          \
            throw ::ssla::CudaError(std::string(#call) + ": " + cudaGetErrorString(e_)); \
    } while (0)

void check_launch(const char* what) {
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) throw CudaError(std::string(what) + ": " + cudaGetErrorString(e));
}

// Optional per-phase timing: one CUDA event after each phase of a drain.
struct Prof {
    bool on = false;
    std::vector<cudaEvent_t> ev;
    std::vector<std::string> names;
    std::vector<int> nl;
    int used = 0;
    int launches = 0;
    ~Prof() {
        for (auto e : ev) cudaEventDestroy(e);
    }
    void begin(cudaStream_t st) {
        used = 0;
        launches = 0;
        names.clear();
        nl.clear();
        if (on) record(st);
    }
    void record(cudaStream_t st) {
        if (used == static_cast<int>(ev.size())) {
            cudaEvent_t e;
            if (cudaEventCreate(&e) != cudaSuccess) throw std::runtime_error("cudaEventCreate failed");
            ev.push_back(e);
        }
        if (cudaEventRecord(ev[used], st) != cudaSuccess) throw std::runtime_error("cudaEventRecord failed");
        ++used;
    }
    void mark(const char* name, int n_launch, cudaStream_t st) {
        launches += n_launch;
        if (!on) return;
        names.emplace_back(name);
        nl.push_back(n_launch);
        record(st);
    }
};

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        SSLA_CK(cudaSetDevice(dev));
    }
    ~DeviceGuard() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

// Owning device allocation.
struct DevBuf {
    void* p = nullptr;
    size_t n = 0;
    DevBuf() = default;
    DevBuf(const DevBuf&) = delete;
    DevBuf& operator=(const DevBuf&) = delete;
    ~DevBuf() { release(); }
    void release() {
        if (p) cudaFree(p);
        p = nullptr;
        n = 0;
    }
    void alloc(size_t bytes) {
        release();
        if (bytes == 0) bytes = 16;
        SSLA_CK(cudaMalloc(&p, bytes));
        n = bytes;
    }
    template <typename T> T* as() const { return static_cast<T*>(p); }
};

template <typename T>
void upload(DevBuf& b, const std::vector<T>& v) {
    b.alloc(v.size() * sizeof(T));
    if (!v.empty()) SSLA_CK(cudaMemcpy(b.p, v.data(), v.size() * sizeof(T), cudaMemcpyHostToDevice));
}

int cells(const Geo& g, int s) { return g.W[s] * g.H[s]; }

int host_gate_grid(int layout, int gate) {
    return gate == 0 ? 1 : gate == 1 ? 2 : gate == 2 ? (layout == LAYOUT_HYBRID ? 2 : 3) : 3;
}

// Upper bound of the events passing a gate with `cells_g` counters when `n`
// events reach it: at one counter, passes among c consecutive arrivals are
// at most ceil(c / w) when w divides 256 (the counter period), and at most
// ceil(c / 256) * ceil(256 / w) otherwise.
long long gate_bound(long long n, int cells_g, int window) {
    if (window <= 1) return n;
    long long b;
    if (256 % window == 0) {
        b = n / window + cells_g;
    } else {
        const long long per = (256 + window - 1) / window;
        b = (n / 256 + cells_g) * per;
    }
    return std::min(n, b);
}

void make_geo(Geo& g, int H, int W, int P, int layout, int window, int ncls) {
    std::memset(&g, 0, sizeof g);
    for (int s = 0; s < 4; ++s) {
        g.H[s] = H >> s;
        g.W[s] = W >> s;
        g.tx[s] = (g.W[s] + kTile - 1) / kTile;
        g.ty[s] = (g.H[s] + kTile - 1) / kTile;
        g.row_lo[s] = 0;
        g.row_hi[s] = g.H[s];
    }
    if (g.tx[0] > kMaxTileCols) throw std::invalid_argument("sensor wider than 512 pixels");
    g.P = P;
    g.layout = layout;
    g.window = window;
    g.ncls = ncls;
    g.stride_h = H / g.H[3];
    g.stride_w = W / g.W[3];
}

// Per-drain workspace: stage lists, tile lists, per-(entry, delta) layer
// records and residuals, sized from proven upper bounds of the events that
// can reach each stage.
struct Workspace {
    int P = 0, mpe = 0, n_max = 0, s_first = 0, tiles_per_part = 1, ctile = kCompactTile, n_active = 0;
    long long cap_part[5] = {0}, cap[5] = {0};
    DevBuf ev, ev_off, ev_xy, rflags, E[5], off[5], count, tilecnt, tilebase;
    DevBuf tl[4], tl_cnt[4], S_A, S_B, QH, R_A, R_B, X, C, head_dec, head_raw, slot_feat, stamps, work;
    DevBuf hot[2], hot_flag[2];    // hot tiles of stages 0-1 (k_hot_tiles)
    bool hot_on[2] = {false, false};   // this drain splits hot tiles of stage s
    int gpt[2] = {16, 16};             // group items per tile of the stage-s scans
    DevBuf stage_out[4];

    void plan(Geo& g, int P_, int mpe_, int n_max_, int s_first_, bool record) {
        P = P_; mpe = mpe_; n_max = n_max_; s_first = s_first_;
        g.seg = std::min(4096, std::max(256, ((mpe + 255) / 256) * 256));
        cap_part[s_first] = mpe;
        cap[s_first] = n_max;
        for (int s = s_first; s < 4; ++s) {
            // DECOMP has no gate after stage 3: every stage-3 event reaches the head.
            if (s == 3 && g.layout != LAYOUT_HYBRID) {
                cap_part[4] = cap_part[3];
                cap[4] = cap[3];
                break;
            }
            const int cg = cells(g, host_gate_grid(g.layout, s));
            cap_part[s + 1] = gate_bound(cap_part[s], cg, g.window);
            cap[s + 1] = std::min(cap[s], gate_bound(cap[s], cg * P, g.window));
        }
        for (int s = 0; s < 4; ++s)
            g.nseg[s] = s < s_first ? 0 : static_cast<int>((cap_part[s] + g.seg - 1) / g.seg);
        for (int s = 0; s < 5; ++s) g.cap[s] = static_cast<int>(s < s_first ? 0 : cap[s]);
        // compaction tiles: about four per SM over the chunk (one CTA walks a
        // tile in order, so few large tiles leave SMs idle), 512..4096 events
        ctile = static_cast<int>(std::min<long long>(
            kCompactTile, std::max<long long>(512, ((static_cast<long long>(P) * mpe / 592 + 255) / 256) * 256)));
        tiles_per_part = static_cast<int>((mpe + ctile - 1) / ctile);
        if (tiles_per_part < 1) tiles_per_part = 1;

        ev.alloc(static_cast<size_t>(n_max) * sizeof(float4));
        ev_off.alloc(sizeof(int) * (P + 1));
        ev_xy.alloc(sizeof(uint32_t) * n_max);
        rflags.alloc(n_max);
        for (int s = 1; s <= 4; ++s) {
            E[s].alloc(sizeof(StageEntry) * std::max<long long>(cap[s], 1));
            off[s].alloc(sizeof(int) * (P + 1));
        }
        count.alloc(sizeof(int) * 5);
        tilecnt.alloc(sizeof(int) * 4 * P * tiles_per_part);
        tilebase.alloc(sizeof(int) * 4 * P * tiles_per_part);
        for (int s = s_first; s < 4; ++s) {
            const size_t slots = static_cast<size_t>(P) * g.tx[s] * g.ty[s] * g.nseg[s];
            tl[s].alloc(slots * g.seg * sizeof(int2));
            tl_cnt[s].alloc(slots * sizeof(int));
            SSLA_CK(cudaMemset(tl_cnt[s].p, 0, slots * sizeof(int)));   // tiles no filter launch covers
            if (s < 2) {
                const size_t nt = static_cast<size_t>(P) * g.tx[s] * g.ty[s];
                hot[s].alloc(sizeof(int) * (nt + 1));
                hot_flag[s].alloc(nt);
            }
        }
        // Stage 0-1 layers keep compact q*h rows (QH); stage 2-3 layers use
        // GEMM-built (q, v, sigmoid(g)) rows (S_A first layers, S_B second).
        size_t sa = 1, qh = 1, rx = 1, cmax = 1;
        for (int s = s_first; s < 4; ++s) {
            const size_t c = chans(s), k = static_cast<size_t>(std::max<long long>(cap[s], 1));
            if (s >= 2) sa = std::max(sa, k * 9 * 3 * c);
            else qh = std::max(qh, k * 9 * c);
            rx = std::max(rx, k * 2 * c);       // X rows, residual rows (next-stage width)
            cmax = std::max(cmax, k * 9 * c);
        }
        S_A.alloc(sa * 4); S_B.alloc(sa * 4); QH.alloc(qh * 4);
        R_A.alloc(rx * 4); R_B.alloc(rx * 4); X.alloc(rx * 4); C.alloc(cmax * 4);
        const int cols = 5 + g.ncls;
        head_dec.alloc(sizeof(float) * cols * std::max<long long>(cap[4], 1));
        head_raw.alloc(sizeof(float) * cols * std::max<long long>(cap[4], 1));
        stamps.alloc(sizeof(unsigned long long) * 2);
        work.alloc(sizeof(int) * 8);
        if (s_first == 2) slot_feat.alloc(sizeof(float) * 96 * n_max);
        for (int s = 0; s < 4; ++s) {
            if (record) stage_out[s].alloc(sizeof(float) * chans(s) * static_cast<size_t>(n_max));
            else stage_out[s].release();
        }
    }
};

// Enqueues layers 1..7 (s_first = 0; layer 0 is done by k_gates) or 4..7
// (s_first = 2, drain_n).  On entry X holds the input rows of the first
// layer to run and R_B (s_first = 0) / R_A (s_first = 2) its residuals.
// Per layer l (stage s, half = l % 2):
//   stages 0-1: k_scan_fused (qvg computed per hit from X rows, q*h -> QH)
//   stages 2-3: k_gemm builds the (q, v, sigmoid(g)) rows of the layer from X
//               (all columns for first layers; v,g for every event and q
//               for output-producing events for second layers), k_scan
//   then k_contrib (goW contributions) and k_ln (ordered sum, residual,
//   LayerNorm) write the layer output back into X, plus the residual of the
//   next layer (copy for a stage's second layer, input_proj for the next
//   stage's first); after layer 7 k_head.
// Layers [l_begin, l_end) of a drain, then the head when do_head; l_stop is
// the layer after which the whole drain ends (the last layers' fused
// next-stage residual is skipped there).
void run_layers(cudaStream_t st, const Geo& g, Workspace& w, const PartState* d_parts,
                const DevLayer* L, const DevHead* head, bool do_head, bool record, Prof& prof,
                int l_end = 8, int l_begin = 0, int l_stop = -1) {
    if (l_stop < 0) l_stop = l_end;
    static const char* kScan[8] = {"scan_L0", "scan_L1", "scan_L2", "scan_L3",
                                   "scan_L4", "scan_L5", "scan_L6", "scan_L7"};
    static const char* kContrib[8] = {"contrib_L0", "contrib_L1", "contrib_L2", "contrib_L3",
                                      "contrib_L4", "contrib_L5", "contrib_L6", "contrib_L7"};
    static const char* kLn[8] = {"ln_L0", "ln_L1", "ln_L2", "ln_L3", "ln_L4", "ln_L5", "ln_L6", "ln_L7"};
    static const char* kGemmA[8] = {"", "", "", "", "gemm_L4_all", "gemm_L5_vg", "gemm_L6_all", "gemm_L7_vg"};
    const int* d_count = w.count.as<int>();
    float* X = w.X.as<float>();
    float* R_first = w.R_A.as<float>();        // residual rows of first layers
    float* R_second = w.R_B.as<float>();       // residual rows of second layers
    const int l0 = (w.s_first == 0) ? 1 : 4;
    // the layer-1..3 work counters were zeroed by k_flag_s0 in the drain's front
    for (int l = std::max(l0, l_begin); l < l_end; ++l) {
        const int s = l / 2, half = l % 2;
        const int* range = (s == 0) ? w.ev_off.as<int>() : w.off[s].as<int>();
        // rows of this layer's scan entries (the stage list) and of its output
        const long long n_s = (s == 0) ? w.n_active : w.cap[s];
        const long long n_out = half ? w.cap[s + 1] : n_s;
        const float* S_rows;
        int qstride;
        if (s < 2) {
            if (l == 1 || l == 2) {
                // split hot tiles only when the cell-group items of the rows
                // this engine scans are fewer than the kernel's resident warps
                const int ty_lo = g.row_lo[s] / kTile, ty_hi = (g.row_hi[s] + kTile - 1) / kTile;
                const long long tiles = static_cast<long long>(g.P) * g.tx[s] * std::max(0, ty_hi - ty_lo);
                w.gpt[s] = scan_fused_groups_per_tile(l, tiles);
                const long long groups = tiles * w.gpt[s];
                w.hot_on[s] = groups < scan_fused_resident_warps(l);
                if (w.hot_on[s]) {
                    HotArgs ha{};
                    ha.threshold = kHotTileEntries;
                    ha.g = g; ha.stage = s; ha.tl_cnt = w.tl_cnt[s].as<int>(); ha.range = range;
                    ha.hot = w.hot[s].as<int>(); ha.hot_flag = w.hot_flag[s].as<uint8_t>();
                    launch_hot_tiles(st, ha);
                    check_launch("k_hot_tiles");
                    prof.mark(s == 0 ? "hot_s0" : "hot_s1", 1, st);
                }
            }
            ScanFusedArgs fa{};
            fa.g = g; fa.stage = s; fa.layer = l; fa.tl = w.tl[s].as<int2>(); fa.tl_cnt = w.tl_cnt[s].as<int>();
            fa.range = range; fa.parts = d_parts; fa.rflags = w.rflags.as<uint8_t>(); fa.second = half;
            fa.X = X; fa.W = L[l].qvgT; fa.QH = w.QH.as<float>(); fa.work = w.work.as<int>() + l;
            fa.hot = w.hot_on[s] ? w.hot[s].as<int>() : nullptr;
            fa.hot_flag = w.hot_on[s] ? w.hot_flag[s].as<uint8_t>() : nullptr;
            fa.gpt = w.gpt[s];
            launch_scan_fused(st, l, fa);
            check_launch("k_scan_fused");
            prof.mark(kScan[l], 1, st);
            S_rows = w.QH.as<float>();
            qstride = chans(s);
        } else {
            float* S_l = half ? w.S_B.as<float>() : w.S_A.as<float>();
            GemmArgs gm{};
            gm.count = d_count; gm.X = X; gm.A2 = 9; gm.W = L[l].qvgT; gm.S = S_l;
            gm.list = s; gm.g_cap = static_cast<int>(w.cap[s]);
            gm.colmode = half ? COLS_VG : COLS_ALL;
            gm.n_cols = gemm_cols(l, gm.colmode);
            launch_gemm(st, l, gm, n_s);
            check_launch("k_gemm");
            prof.mark(kGemmA[l], 1, st);
            if (half) {
                GemmArgs gq = gm;
                gq.list = s + 1; gq.g_cap = static_cast<int>(w.cap[s + 1]);
                gq.E = w.E[s + 1].as<StageEntry>();
                gq.colmode = COLS_Q; gq.n_cols = gemm_cols(l, COLS_Q);
                launch_gemm(st, l, gq, w.cap[s + 1]);
                check_launch("k_gemm q");
                prof.mark(l == 5 ? "gemm_L5_q" : "gemm_L7_q", 1, st);
            }
            ScanArgs sa{};
            sa.g = g; sa.stage = s; sa.layer = l; sa.tl = w.tl[s].as<int2>(); sa.tl_cnt = w.tl_cnt[s].as<int>();
            sa.range = range; sa.S = S_l; sa.parts = d_parts; sa.rflags = w.rflags.as<uint8_t>(); sa.second = half;
            launch_scan(st, l, sa);
            check_launch("k_scan");
            prof.mark(kScan[l], 1, st);
            S_rows = S_l;
            qstride = 3 * chans(s);
        }
        ContribArgs ca{};
        LnArgs la{};
        ca.g = la.g = g; ca.stage = la.stage = s; ca.second = la.second = half;
        ca.count = la.count = d_count;
        ca.ev_xy = la.ev_xy = w.ev_xy.as<uint32_t>();
        ca.rflags = la.rflags = w.rflags.as<uint8_t>();
        ca.S = S_rows; ca.qstride = qstride; ca.goWT = L[l].goWT; ca.C = w.C.as<float>();
        if (s < 2) { ca.Xq = X; ca.Wq = L[l].qvgT; }
        la.C = w.C.as<float>(); la.R_in = half ? R_second : R_first; la.L = L[l]; la.X_out = X;
        la.stage_out = record ? w.stage_out[s].as<float>() : nullptr;
        la.slot_feat = (w.s_first == 2) ? w.slot_feat.as<float>() : nullptr;
        if (half == 0) {
            if (s == 0) { ca.list = la.list = 0; ca.n_static = la.n_static = w.n_active; }
            else { ca.list = la.list = s; ca.E = la.E = w.E[s].as<StageEntry>(); }
            la.copyres_bit = static_cast<uint8_t>(F_R1 << s);      // R_{s+1}
            la.R_next = R_second;
        } else {
            ca.list = la.list = s + 1;
            ca.E = la.E = w.E[s + 1].as<StageEntry>();
            if (s < 3 && l + 1 < l_stop) { la.ipT_next = L[l + 1].ipT; la.R_ipnext = R_first; }
        }
        launch_contrib(st, l, ca, n_out);
        check_launch("k_contrib");
        prof.mark(kContrib[l], 1, st);
        launch_ln(st, l, la, n_out);
        check_launch("k_ln");
        prof.mark(kLn[l], 1, st);
    }
    if (do_head) {
        HeadArgs ha{};
        ha.g = g; ha.count = d_count; ha.E4 = w.E[4].as<StageEntry>(); ha.X = X;
        ha.head = *head; ha.head_dec = w.head_dec.as<float>(); ha.head_raw = w.head_raw.as<float>();
        ha.tc_w1 = head->tc_w1; ha.err = head->tc_err;
        if (head->tc_w1) {
            launch_head_tc(st, ha, w.cap[4]);
            check_launch("k_head_tc");
        } else {
            launch_head(st, ha, w.cap[4]);
            check_launch("k_head");
        }
        prof.mark("head", 1, st);
    }
}

}  // namespace

// Error text of the calling thread, for entry points defined in other files.
void set_last_error(const std::string& msg) { g_last_error = msg; }

// ---------------------------------------------------------------------------
// Engine
// ---------------------------------------------------------------------------
struct Engine {
    int device = 0;
    Geo g{};
    int layout = LAYOUT_HYBRID;
    int max_events = 0, mpe = 0;
    bool record = false;
    HostModel model;
    DevBuf wbuf[8][5];          // qvgT, goWT, ipT, gamma, beta per layer
    DevBuf hbuf[10];
    DevLayer L[8]{};
    DevHead head{};
    DevBuf head_tc;                         // tensor-core head operand (see DevHead::tc_w1)
    unsigned* head_tc_err = nullptr;        // host-mapped status bits of k_head_tc
    // state
    DevBuf hidden[8], cnt[4], last_t, preds_dec, preds_raw, version, parts;
    std::vector<PartState> h_parts;
    Workspace ws;
    Prof prof;
    // Pinned staging of the partition offsets: a ring of slots, each reused
    // only after the copy that read it has executed.
    static constexpr int kOffSlots = 8;
    int* pinned_off = nullptr;
    int* pinned_rec_off = nullptr;
    // Status word of the step kernel (host-mapped): bits of bounded waits
    // that ran out, read and cleared by the next step call.
    unsigned* step_err = nullptr;
    // Live loop: status word (host-mapped) and the stream it runs on.
    unsigned* live_err = nullptr;
    cudaStream_t live_stream = nullptr;
    bool live_running = false;
    unsigned long long live_withhold = ~0ull;   // test hook for the next live loop (~0: off)
    cudaEvent_t off_done[kOffSlots] = {};
    int off_slot = 0;
    long long last_counts[5] = {0};
    int last_n = 0;

    ~Engine() {
        for (auto& e : off_done)
            if (e) cudaEventDestroy(e);
        if (pinned_off) cudaFreeHost(pinned_off);
        if (pinned_rec_off) cudaFreeHost(pinned_rec_off);
        if (live_running) cudaStreamSynchronize(live_stream);   // ends on its stop flag or idle bound
        for (void* p : strip.opened)
            if (p) cudaIpcCloseMemHandle(p);
        if (strip.err) cudaFreeHost(strip.err);
        if (head_tc_err) cudaFreeHost(head_tc_err);
        if (step_err) cudaFreeHost(step_err);
        if (live_err) cudaFreeHost(live_err);
        if (hpipe.st) cudaStreamSynchronize(hpipe.st);
        for (int k = 0; k < 2; ++k) {
            if (hpipe.copied[k]) cudaEventDestroy(hpipe.copied[k]);
            if (hpipe.consumed[k]) cudaEventDestroy(hpipe.consumed[k]);
        }
        if (hpipe.st) cudaStreamDestroy(hpipe.st);
    }

    size_t state_elems(int kind, int index) const {
        switch (kind) {
            case SSLA_STATE_HIDDEN: return static_cast<size_t>(cells(g, index / 2)) * chans(index / 2);
            case SSLA_STATE_COUNTER: return static_cast<size_t>(cells(g, host_gate_grid(layout, index)));
            case SSLA_STATE_LAST_T: return static_cast<size_t>(cells(g, 0));
            case SSLA_STATE_PREDS_DEC:
            case SSLA_STATE_PREDS_RAW: return static_cast<size_t>(cells(g, 3)) * (5 + g.ncls);
            case SSLA_STATE_VERSION: return static_cast<size_t>(cells(g, 3));
            case SSLA_STATE_STAGE_OUT: return static_cast<size_t>(max_events) * chans(index);
            case SSLA_STATE_FLAGS: return static_cast<size_t>(max_events);
            default: return 0;
        }
    }
    static size_t elem_size(int kind) {
        switch (kind) {
            case SSLA_STATE_COUNTER: case SSLA_STATE_FLAGS: return 1;
            case SSLA_STATE_LAST_T: return 8;
            case SSLA_STATE_VERSION: return 4;
            default: return 4;
        }
    }
    char* state_ptr(int kind, int p, int index) {
        const size_t per = state_elems(kind, index) * elem_size(kind);
        switch (kind) {
            case SSLA_STATE_HIDDEN: return hidden[index].as<char>() + per * p;
            case SSLA_STATE_COUNTER: return cnt[index].as<char>() + per * p;
            case SSLA_STATE_LAST_T: return last_t.as<char>() + per * p;
            case SSLA_STATE_PREDS_DEC: return preds_dec.as<char>() + per * p;
            case SSLA_STATE_PREDS_RAW: return preds_raw.as<char>() + per * p;
            case SSLA_STATE_VERSION: return version.as<char>() + per * p;
            case SSLA_STATE_STAGE_OUT: return record ? ws.stage_out[index].as<char>() : nullptr;
            case SSLA_STATE_FLAGS: return ws.rflags.as<char>();
            default: return nullptr;
        }
    }

    void create(const char* dir, const SslaEngineConfig& c) {
        device = c.device;
        int ndev = 0;
        if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) throw CudaError("no CUDA device");
        if (device < 0 || device >= ndev) throw std::invalid_argument("device ordinal out of range");
        DeviceGuard dg(device);
        model = load_model(dir);
        layout = c.layout;
        record = c.record_stage_outputs != 0;
        max_events = c.max_events;
        const int P = c.n_partitions;
        mpe = c.max_events_per_partition > 0 ? c.max_events_per_partition : (max_events + P - 1) / P;
        make_geo(g, model.meta.height, model.meta.width, P, layout, model.meta.tdrop_window,
                 model.meta.num_classes);
        for (int l = 0; l < 8; ++l) {
            const HostLayer& hl = model.layers[l];
            upload(wbuf[l][0], hl.qvgT);
            upload(wbuf[l][1], hl.goWT);
            if (!hl.ipT.empty()) upload(wbuf[l][2], hl.ipT);
            upload(wbuf[l][3], hl.gamma);
            upload(wbuf[l][4], hl.beta);
            L[l].qvgT = wbuf[l][0].as<float>();
            L[l].goWT = wbuf[l][1].as<float>();
            L[l].ipT = hl.ipT.empty() ? nullptr : wbuf[l][2].as<float>();
            L[l].gamma = wbuf[l][3].as<float>();
            L[l].beta = wbuf[l][4].as<float>();
        }
        const HostHead& hh = model.head;
        const std::vector<float>* hv[10] = {&hh.cls_convT, &hh.cls_conv_b, &hh.reg_convT, &hh.reg_conv_b,
                                            &hh.cls_predT, &hh.cls_pred_b, &hh.reg_predT, &hh.reg_pred_b,
                                            &hh.obj_predT, &hh.obj_pred_b};
        for (int i = 0; i < 10; ++i) upload(hbuf[i], *hv[i]);
        head = DevHead{hbuf[0].as<float>(), hbuf[1].as<float>(), hbuf[2].as<float>(), hbuf[3].as<float>(),
                       hbuf[4].as<float>(), hbuf[5].as<float>(), hbuf[6].as<float>(), hbuf[7].as<float>(),
                       hbuf[8].as<float>(), hbuf[9].as<float>(), nullptr, nullptr};
        // the tensor-core head's operand: [cls_conv | reg_conv] as [192 out][96 in]
        // rows, split into TF32 hi terms and TF32 lo terms (the remainder)
        {
            auto tf32 = [](float x) {
                uint32_t u;
                std::memcpy(&u, &x, 4);
                if ((u & 0x7F800000u) != 0x7F800000u) u = (u + 0x1000u) & 0xFFFFE000u;
                float r;
                std::memcpy(&r, &u, 4);
                return r;
            };
            std::vector<float> w1(2 * 192 * 96);
            for (int o = 0; o < 192; ++o)
                for (int i = 0; i < 96; ++i) {
                    const float w = o < 96 ? hh.cls_convT[i * 96 + o] : hh.reg_convT[i * 96 + (o - 96)];
                    const float hi = tf32(w);
                    w1[o * 96 + i] = hi;
                    w1[192 * 96 + o * 96 + i] = tf32(w - hi);
                }
            upload(head_tc, w1);
            SSLA_CK(cudaHostAlloc(&head_tc_err, sizeof(unsigned), cudaHostAllocMapped));
            *head_tc_err = 0;
        }
        // state
        for (int l = 0; l < 8; ++l) hidden[l].alloc(state_elems(SSLA_STATE_HIDDEN, l) * 4 * P);
        for (int gi = 0; gi < 4; ++gi) cnt[gi].alloc(state_elems(SSLA_STATE_COUNTER, gi) * P);
        last_t.alloc(state_elems(SSLA_STATE_LAST_T, 0) * 8 * P);
        preds_dec.alloc(state_elems(SSLA_STATE_PREDS_DEC, 0) * 4 * P);
        preds_raw.alloc(state_elems(SSLA_STATE_PREDS_RAW, 0) * 4 * P);
        version.alloc(state_elems(SSLA_STATE_VERSION, 0) * 4 * P);
        h_parts.assign(P, PartState{});
        for (int p = 0; p < P; ++p) {
            PartState& ps = h_parts[p];
            for (int l = 0; l < 8; ++l) ps.hidden[l] = reinterpret_cast<float*>(state_ptr(SSLA_STATE_HIDDEN, p, l));
            for (int gi = 0; gi < 4; ++gi) ps.cnt[gi] = reinterpret_cast<uint8_t*>(state_ptr(SSLA_STATE_COUNTER, p, gi));
            ps.last_t = reinterpret_cast<double*>(state_ptr(SSLA_STATE_LAST_T, p, 0));
            ps.preds_dec = reinterpret_cast<float*>(state_ptr(SSLA_STATE_PREDS_DEC, p, 0));
            ps.preds_raw = reinterpret_cast<float*>(state_ptr(SSLA_STATE_PREDS_RAW, p, 0));
            ps.version = reinterpret_cast<uint32_t*>(state_ptr(SSLA_STATE_VERSION, p, 0));
            ps.own_x0 = 0; ps.own_x1 = g.W[2]; ps.own_y0 = 0; ps.own_y1 = g.H[2];
        }
        upload(parts, h_parts);
        ws.plan(g, P, mpe, max_events, 0, record);
        SSLA_CK(cudaMallocHost(&pinned_off, sizeof(int) * (P + 1) * kOffSlots));
        for (auto& e : off_done) SSLA_CK(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
        SSLA_CK(cudaMallocHost(&pinned_rec_off, sizeof(int) * (P + 1)));
        SSLA_CK(cudaHostAlloc(&step_err, sizeof(unsigned), cudaHostAllocMapped));
        *step_err = 0;
        SSLA_CK(cudaHostAlloc(&live_err, sizeof(unsigned), cudaHostAllocMapped));
        *live_err = 0;
        reset(nullptr);
        SSLA_CK(cudaStreamSynchronize(nullptr));
    }

    void reset(cudaStream_t st) {
        DeviceGuard dg(device);
        for (int l = 0; l < 8; ++l) SSLA_CK(cudaMemsetAsync(hidden[l].p, 0, hidden[l].n, st));
        for (int gi = 0; gi < 4; ++gi) SSLA_CK(cudaMemsetAsync(cnt[gi].p, 0, cnt[gi].n, st));
        launch_fill_f64(st, last_t.as<double>(), last_t.n / 8, -1.0);
        check_launch("fill last_t");
        launch_reset_preds(st, g, parts.as<PartState>(), head);
        check_launch("k_reset_preds");
    }

    // One event of partition p through the whole path (k_step); flag_out /
    // pred_out may be device or pinned host memory.  Asynchronous on st.
    void step(int p, const float* e4, uint8_t* flag_out, float* pred_out, cudaStream_t st) {
        if (p < 0 || p >= g.P) throw std::invalid_argument("partition out of range");
        StepArgs a{};
        a.g = g;
        a.ps = h_parts[p];
        for (int l = 0; l < 8; ++l) a.L[l] = L[l];
        a.head = head;
        a.ev = make_float4(e4[0], e4[1], e4[2], e4[3]);
        a.flag_out = flag_out;
        a.pred_out = pred_out;
        a.err = step_err;
        check_step_status();
        SSLA_CK(launch_step(st, a));
        check_launch("k_step");
    }

    // Raises (and clears) the status of earlier steps: a wait inside k_step
    // that ran out means that step's outputs are not valid.
    void check_step_status() {
        const unsigned v = __atomic_load_n(step_err, __ATOMIC_ACQUIRE);
        if (v) {
            __atomic_store_n(step_err, 0u, __ATOMIC_RELEASE);
            throw std::runtime_error("k_step: a bounded wait ran out (status " + std::to_string(v) +
                                     "; 1 = weight copies, 2 = layer input, 4 = contributions)");
        }
    }

    // ---- exact strip sharding (ssla_strip.cu) ----
    struct Strip {
        bool on = false;
        int lo = 0, hi = 0, band = 0, cap = 0;
        int has[2] = {0, 0};
        DevBuf idx, cnt, recv[2], ctr;
        char* peer[2] = {nullptr, nullptr};     // the neighbour's receive buffer for my rows of side s
        int peer_cap[2] = {0, 0};               // rows per parity of that buffer (the neighbour's cap)
        void* opened[2] = {nullptr, nullptr};   // IPC mappings to close
        unsigned long long seq = 0;
        unsigned* err = nullptr;                // host-mapped SSLA_STRIP_ERR_* bits
    } strip;
    // receive-buffer header: u64 sequence, u64 row count per parity, u64 the
    // buffer's rows per parity (its owner's cap; senders size the parity
    // regions and clamp their row counts with it)
    static constexpr size_t kStripHdr = 32;

    size_t strip_recv_bytes() const { return kStripHdr + 2 * static_cast<size_t>(strip.cap) * 96 * sizeof(float); }

    void strip_init(int lo, int hi, int band, int has_up, int has_down, int cap) {
        if (g.P != 1) throw std::invalid_argument("strip sharding needs an engine with one partition");
        if (lo < 0 || hi > g.H[0] || lo >= hi || lo % 8 || hi % 8 || band <= 0 || band % 8 || cap <= 0)
            throw std::invalid_argument("strip rows must be multiples of 8 inside the sensor, band > 0");
        if ((has_up && lo == 0) || (has_down && hi == g.H[0]))
            throw std::invalid_argument("a neighbour beyond the sensor edge");
        strip.lo = lo; strip.hi = hi; strip.band = band; strip.cap = cap;
        strip.has[0] = has_up ? 1 : 0; strip.has[1] = has_down ? 1 : 0;
        strip.idx.alloc(sizeof(int) * 12 * static_cast<size_t>(cap));
        strip.cnt.alloc(sizeof(int) * 12);
        strip.ctr.alloc(sizeof(unsigned) * 2);
        SSLA_CK(cudaMemset(strip.ctr.p, 0, sizeof(unsigned) * 2));
        for (int sd = 0; sd < 2; ++sd)
            if (strip.has[sd]) {
                strip.recv[sd].alloc(strip_recv_bytes());
                SSLA_CK(cudaMemset(strip.recv[sd].p, 0, strip_recv_bytes()));
                const unsigned long long rows = static_cast<unsigned long long>(cap);
                SSLA_CK(cudaMemcpy(strip.recv[sd].as<char>() + 24, &rows, sizeof rows, cudaMemcpyHostToDevice));
            }
        if (!strip.err) SSLA_CK(cudaHostAlloc(&strip.err, sizeof(unsigned), cudaHostAllocMapped));
        *strip.err = 0;
        strip.seq = 0;
        set_owned(0, 0, g.W[2], lo >> 2, hi >> 2, nullptr);
        // the filters now cover only the strip's tile rows: no list outside them may keep old counts
        for (int s = 0; s < 4; ++s)
            if (ws.tl_cnt[s].p) SSLA_CK(cudaMemset(ws.tl_cnt[s].p, 0, ws.tl_cnt[s].n));
        // scans update the rows owned events read: own rows and one beyond each side
        for (int s = 0; s < 4; ++s) {
            g.row_lo[s] = std::max(0, (lo >> s) - 1);
            g.row_hi[s] = std::min(g.H[s], (hi >> s) + 1);
        }
        strip.on = true;
    }

    void strip_recv_buffer(int side, void** ptr, void* handle) {
        if (!strip.on || side < 0 || side > 1 || !strip.has[side]) throw std::invalid_argument("no such strip side");
        if (ptr) *ptr = strip.recv[side].p;
        if (handle)
            SSLA_CK(cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(handle), strip.recv[side].p));
    }

    void strip_connect(int side, void* ptr, const void* handle) {
        if (!strip.on || side < 0 || side > 1 || !strip.has[side]) throw std::invalid_argument("no such strip side");
        if (handle) {
            cudaIpcMemHandle_t h;
            std::memcpy(&h, handle, sizeof h);
            void* p = nullptr;
            SSLA_CK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
            strip.opened[side] = p;
            strip.peer[side] = static_cast<char*>(p);
        } else {
            if (!ptr) throw std::invalid_argument("strip_connect needs a device address or an IPC handle");
            strip.peer[side] = static_cast<char*>(ptr);
        }
        // the neighbour's rows per parity, from its buffer's header
        unsigned long long rows = 0;
        SSLA_CK(cudaMemcpy(&rows, strip.peer[side] + 24, sizeof rows, cudaMemcpyDeviceToHost));
        if (rows == 0 || rows > (1ull << 30)) throw std::invalid_argument("strip_connect: the peer buffer has no row capacity");
        strip.peer_cap[side] = static_cast<int>(rows);
    }

    // Step j of a strip drain: 0 = front, band lists, layer 1; 1..5 = layer
    // j+1; 6 = layer 7, head and commit.
    void strip_step(int j, const float* ev, int n, uint8_t* flags, cudaStream_t st) {
        if (!strip.on) throw std::invalid_argument("strip_init first");
        if (j == 0) {
            const int off[2] = {0, n};
            drain_front(ev, off, st, 3);
            StripSelectArgs sa{};
            for (int k = 0; k <= 4; ++k) { sa.E[k] = ws.E[k].as<StageEntry>(); sa.g_cap[k] = g.cap[k]; }
            sa.count = ws.count.as<int>();
            sa.lo = strip.lo; sa.hi = strip.hi; sa.band = strip.band;
            sa.has[0] = strip.has[0]; sa.has[1] = strip.has[1];
            sa.cap = strip.cap; sa.idx = strip.idx.as<int>(); sa.cnt = strip.cnt.as<int>(); sa.err = strip.err;
            launch_band_select(st, sa);
            check_launch("k_band_select");
            launch_mark_foreign(st, n, ws.ev_xy.as<uint32_t>(), ws.rflags.as<uint8_t>(), strip.lo, strip.hi);
            check_launch("k_mark_foreign");
            run_layers(st, g, ws, parts.as<PartState>(), L, &head, false, record, prof, 2, 0, 8);
        } else if (j < 6) {
            run_layers(st, g, ws, parts.as<PartState>(), L, &head, false, record, prof, j + 2, j + 1, 8);
        } else {
            run_layers(st, g, ws, parts.as<PartState>(), L, &head, true, record, prof, 8, 7, 8);
            drain_back(n, flags, st);
        }
    }

    // Exchange after layer j + 1 (j = 0..5): the next layer's input rows,
    // stage list k = (j + 2) / 2, channels chans((j + 1) / 2).
    void strip_xfer(int j, bool do_export, unsigned long long seq, bool wait, cudaStream_t st) {
        const int l = j + 1, k = (l + 1) / 2, C = chans(l / 2);
        const int parity = static_cast<int>(seq & 1u);
        for (int sd = 0; sd < 2; ++sd) {
            if (!strip.has[sd]) continue;
            // parity regions of the buffer written: the receiver's rows per
            // parity (its cap), whether it is the neighbour's or this engine's
            const int rows = do_export ? strip.peer_cap[sd] : strip.cap;
            const size_t data_off = kStripHdr + static_cast<size_t>(parity) * rows * 96 * sizeof(float);
            StripXferArgs xa{};
            xa.X = ws.X.as<float>(); xa.C = C; xa.cap = std::min(strip.cap, rows); xa.parity = parity; xa.seq = seq;
            xa.err = strip.err;
            const int q = (k - 1) * 4 + sd * 2 + (do_export ? 0 : 1);
            xa.idx = strip.idx.as<int>() + static_cast<size_t>(q) * strip.cap;
            xa.cnt = strip.cnt.as<int>() + q;
            if (do_export) {
                if (!strip.peer[sd]) throw std::invalid_argument("strip side not connected");
                xa.data = reinterpret_cast<float*>(strip.peer[sd] + data_off);
                xa.header = reinterpret_cast<unsigned long long*>(strip.peer[sd]);
                xa.done_ctr = strip.ctr.as<unsigned>() + sd;
                launch_strip_export(st, xa);
                check_launch("k_strip_export");
            } else {
                xa.data = reinterpret_cast<float*>(strip.recv[sd].as<char>() + data_off);
                xa.header = strip.recv[sd].as<unsigned long long>();
                xa.wait = wait ? 1 : 0;
                xa.wait_ns = 5ull * 1000ull * 1000ull * 1000ull;
                launch_strip_import(st, xa);
                check_launch("k_strip_import");
            }
        }
    }

    // One strip drain on this GPU, the neighbours' rows awaited on the device.
    void strip_drain(const float* ev, int n, uint8_t* flags, cudaStream_t st) {
        for (int j = 0; j < 7; ++j) {
            strip_step(j, ev, n, flags, st);
            if (j < 6) {
                const unsigned long long seq = ++strip.seq;
                strip_xfer(j, true, seq, false, st);
                strip_xfer(j, false, seq, true, st);
            }
        }
    }

    unsigned strip_status() {
        if (!strip.err) return 0;
        SSLA_CK(cudaDeviceSynchronize());
        const unsigned v = __atomic_exchange_n(strip.err, 0u, __ATOMIC_ACQ_REL);
        return v;
    }

    // Owned range of a partition in stage-2 cells [x0, x1) x [y0, y1): only
    // events there commit predictions (the reference's HybridStrip owned
    // bounds, ssla_s2_s3_head_celled.cuh:1663-1670); the rest are halo.
    void set_owned(int p, int x0, int x1, int y0, int y1, cudaStream_t st) {
        if (p < 0 || p >= g.P) throw std::invalid_argument("partition out of range");
        if (x0 < 0 || y0 < 0 || x1 > g.W[2] || y1 > g.H[2] || x0 > x1 || y0 > y1)
            throw std::invalid_argument("owned range outside the stage-2 grid");
        PartState& ps = h_parts[p];
        ps.own_x0 = x0; ps.own_x1 = x1; ps.own_y0 = y0; ps.own_y1 = y1;
        SSLA_CK(cudaMemcpyAsync(parts.as<PartState>() + p, &ps, sizeof(PartState), cudaMemcpyHostToDevice, st));
        SSLA_CK(cudaStreamSynchronize(st));
    }

    // The live loop touches the ring from the device: every buffer must be
    // pinned host memory that the device reaches at the same address.
    static void need_mapped(const void* p, size_t bytes, const char* what) {
        if (!p) throw std::invalid_argument(std::string("live ring: ") + what + " is NULL");
        for (const char* q : {static_cast<const char*>(p), static_cast<const char*>(p) + bytes - 1}) {
            cudaPointerAttributes at{};
            if (cudaPointerGetAttributes(&at, q) != cudaSuccess || at.type != cudaMemoryTypeHost ||
                at.devicePointer != at.hostPointer) {
                cudaGetLastError();
                throw std::invalid_argument(std::string("live ring: ") + what +
                                            " is not pinned, device-mapped host memory");
            }
        }
    }

    void live_start(int p, const SslaLiveRing& r, unsigned idle_ms, cudaStream_t st) {
        if (p < 0 || p >= g.P) throw std::invalid_argument("partition out of range");
        if (live_running) throw std::invalid_argument("a live loop is already running on this engine");
        if (r.capacity < 2 || (r.capacity & (r.capacity - 1))) throw std::invalid_argument("ring capacity must be a power of two >= 2");
        if (g.ncls > live_max_ncls()) throw std::invalid_argument("too many classes for the live loop");
        if (reinterpret_cast<uintptr_t>(r.events) % 16) throw std::invalid_argument("live ring: events must be 16-byte aligned");
        const size_t cols = 5 + static_cast<size_t>(g.ncls);
        need_mapped(r.events, 16 * r.capacity, "events");
        need_mapped(r.head, 8, "head");
        need_mapped(r.tail, 8, "tail");
        need_mapped(r.events_done, 8, "events_done");
        need_mapped(r.stop_flag, 4, "stop_flag");
        if (r.flags) need_mapped(r.flags, r.capacity, "flags");
        if (r.preds) need_mapped(r.preds, sizeof(float) * cols * r.capacity, "preds");
        LiveArgs a{};
        a.g = g;
        a.ps = h_parts[p];
        for (int l = 0; l < 8; ++l) a.L[l] = L[l];
        a.head = head;
        a.events = reinterpret_cast<const float4*>(r.events);
        a.mask = r.capacity - 1;
        a.head_idx = r.head;
        a.tail = r.tail;
        a.done = r.events_done;
        a.flags_out = r.flags;
        a.preds_out = r.preds;
        a.stop = r.stop_flag;
        a.start = __atomic_load_n(r.tail, __ATOMIC_ACQUIRE);
        a.idle_ns = static_cast<unsigned long long>(idle_ms) * 1000000ull;
        a.err = live_err;
        a.withhold_fin = live_withhold;
        live_withhold = ~0ull;
        __atomic_store_n(live_err, 0u, __ATOMIC_RELEASE);
        SSLA_CK(launch_live(st, a));
        check_launch("k_live");
        live_stream = st;
        live_running = true;
    }

    // Waits for the loop to end and returns its status word; with `check`,
    // a wait that ran out inside the loop is raised as an error.
    unsigned live_join(bool check = true) {
        if (!live_running) throw std::invalid_argument("no live loop is running on this engine");
        live_running = false;
        SSLA_CK(cudaStreamSynchronize(live_stream));
        const unsigned v = __atomic_load_n(live_err, __ATOMIC_ACQUIRE);
        if (check && (v & 0xFFu)) throw CudaError(live_status_text(v));
        return v;
    }
    static std::string live_status_text(unsigned v) {
        return "k_live: a bounded wait ran out (status " + std::to_string(v) +
               "; 1 weights, 2 layer input, 4 contributions, 8 event message, 16 completion)";
    }

    // Device alias of a pinned, device-mapped host pointer (page-locked
    // memory with unified addressing), or null for any other pointer.
    template <typename T>
    static T* mapped_alias(T* host) {
        cudaPointerAttributes at{};
        if (cudaPointerGetAttributes(&at, host) != cudaSuccess) {
            cudaGetLastError();                    // pageable memory: clear the sticky query error
            return nullptr;
        }
        if (at.type != cudaMemoryTypeHost || !at.devicePointer) return nullptr;
        return static_cast<T*>(at.devicePointer);
    }

    // ---- pipelined host drains: copy-in on a copy stream, double-buffered ----
    struct HostPipe {
        cudaStream_t st = nullptr;
        DevBuf ev[2];
        cudaEvent_t copied[2] = {}, consumed[2] = {};
        int slot = 0;
    } hpipe;

    // Events from pinned host memory: the copy of this drain's events runs on
    // the engine's copy stream, into the device buffer the drain before last
    // used (after that drain's results were copied out), while the previous
    // drain runs on `st`; the drain waits for its copy, then its flags and
    // all partitions' decoded predictions are copied back to flags_host /
    // preds_host (either may be null) on `st`.
    // Returns without waiting; the host buffers belong to the call until
    // `st` has passed it.
    void drain_host_async(const float* ev_host, const int* off, uint8_t* flags_host, float* preds_host,
                          cudaStream_t st) {
        const int n = off[g.P];
        if (n < 0 || n > max_events) throw std::length_error("more events than max_events");
        if (n > 0 && !ev_host) throw std::invalid_argument("null events");
        if (!hpipe.st) {
            SSLA_CK(cudaStreamCreateWithFlags(&hpipe.st, cudaStreamNonBlocking));
            for (int k = 0; k < 2; ++k) {
                hpipe.ev[k].alloc(static_cast<size_t>(max_events) * sizeof(float4));
                SSLA_CK(cudaEventCreateWithFlags(&hpipe.copied[k], cudaEventDisableTiming));
                SSLA_CK(cudaEventCreateWithFlags(&hpipe.consumed[k], cudaEventDisableTiming));
                SSLA_CK(cudaEventRecord(hpipe.consumed[k], hpipe.st));
            }
        }
        const int k = hpipe.slot;
        hpipe.slot ^= 1;
        SSLA_CK(cudaStreamWaitEvent(hpipe.st, hpipe.consumed[k], 0));
        if (n > 0)
            SSLA_CK(cudaMemcpyAsync(hpipe.ev[k].p, ev_host, sizeof(float) * 4 * n, cudaMemcpyHostToDevice, hpipe.st));
        SSLA_CK(cudaEventRecord(hpipe.copied[k], hpipe.st));
        SSLA_CK(cudaStreamWaitEvent(st, hpipe.copied[k], 0));
        drain(hpipe.ev[k].as<float>(), off, nullptr, st);
        // Results: pinned outputs are written by a kernel chained to the
        // drain (no copy-engine round trip on the drain stream); pageable
        // ones are copied.
        uint8_t* fdev = (flags_host && n > 0) ? mapped_alias(flags_host) : nullptr;
        float* pdev = preds_host ? mapped_alias(preds_host) : nullptr;
        if (fdev || pdev) {
            launch_results_to_host(st, ws.rflags.as<uint8_t>(), n, fdev, preds_dec.as<float>(),
                                   static_cast<int>(preds_dec.n / sizeof(float)), pdev);
            check_launch("k_results_to_host");
        }
        if (flags_host && n > 0 && !fdev)
            SSLA_CK(cudaMemcpyAsync(flags_host, ws.rflags.p, n, cudaMemcpyDeviceToHost, st));
        if (preds_host && !pdev)
            SSLA_CK(cudaMemcpyAsync(preds_host, preds_dec.p, preds_dec.n, cudaMemcpyDeviceToHost, st));
        // The copy-in of the drain after next (same buffer) starts once this
        // drain's results are out: issued earlier it would take the copy
        // engine while the results wait behind it, and it still has the
        // whole next drain to finish.
        SSLA_CK(cudaEventRecord(hpipe.consumed[k], st));
    }

    // ---- ring drains (ssla_rings.cu): one pinned ring per partition ----
    struct Rings {
        static constexpr int kSlots = 4;
        std::vector<SslaLiveRing> r;
        std::vector<unsigned long long> next;    // ring index after every enqueued take
        std::vector<unsigned long long> first;   // ring index at attach
        std::vector<int> off;
        RingTake* pinned = nullptr;              // [kSlots][P] staging of the take descriptors
        DevBuf dev[kSlots];
        cudaEvent_t copied[kSlots] = {};
        int slot = 0;
        DevBuf ctr;
        ~Rings() {
            for (auto& e : copied)
                if (e) cudaEventDestroy(e);
            if (pinned) cudaFreeHost(pinned);
        }
    } rings;

    void rings_attach(const SslaLiveRing* rr, int n) {
        if (n != g.P) throw std::invalid_argument("rings_attach needs one ring per partition");
        if (live_running) throw std::invalid_argument("a live loop is running on this engine");
        const size_t cols = 5 + static_cast<size_t>(g.ncls);
        for (int p = 0; p < n; ++p) {
            const SslaLiveRing& r = rr[p];
            if (r.capacity < 2 || (r.capacity & (r.capacity - 1)))
                throw std::invalid_argument("ring capacity must be a power of two >= 2");
            if (reinterpret_cast<uintptr_t>(r.events) % 16) throw std::invalid_argument("ring events must be 16-byte aligned");
            need_mapped(r.events, 16 * r.capacity, "events");
            need_mapped(r.head, 8, "head");
            need_mapped(r.tail, 8, "tail");
            need_mapped(r.events_done, 8, "events_done");
            if (r.flags) need_mapped(r.flags, r.capacity, "flags");
            if (r.preds) need_mapped(r.preds, sizeof(float) * cols * r.capacity, "preds");
        }
        SSLA_CK(cudaDeviceSynchronize());        // no drain in flight reads the old descriptors
        rings.r.assign(rr, rr + n);
        rings.next.resize(n);
        rings.first.resize(n);
        for (int p = 0; p < n; ++p) rings.next[p] = rings.first[p] = __atomic_load_n(rr[p].tail, __ATOMIC_ACQUIRE);
        rings.off.assign(n + 1, 0);
        if (!rings.pinned) {
            SSLA_CK(cudaMallocHost(&rings.pinned, sizeof(RingTake) * Rings::kSlots * n));
            for (int k = 0; k < Rings::kSlots; ++k) {
                rings.dev[k].alloc(sizeof(RingTake) * n);
                SSLA_CK(cudaEventCreateWithFlags(&rings.copied[k], cudaEventDisableTiming));
            }
            rings.ctr.alloc(sizeof(unsigned));
            SSLA_CK(cudaMemset(rings.ctr.p, 0, sizeof(unsigned)));
        }
    }

    // Takes up to max_per_ring published events from every ring (at most
    // max_total in all) and drains them; returns the number taken, taken[p]
    // (may be null) the share of ring p.  Asynchronous on st.
    int drain_rings(int max_per_ring, long long max_total, cudaStream_t st, int* taken) {
        if (rings.r.empty()) throw std::invalid_argument("ssla_engine_rings_attach first");
        if (max_per_ring < 1) throw std::invalid_argument("max_per_ring must be >= 1");
        const int P = g.P;
        std::vector<int>& off = rings.off;
        long long budget = std::min<long long>(max_total, max_events);
        off[0] = 0;
        for (int p = 0; p < P; ++p) {
            const SslaLiveRing& r = rings.r[p];
            const unsigned long long h = __atomic_load_n(r.head, __ATOMIC_ACQUIRE);
            const unsigned long long t = rings.next[p];
            if (h < t || h - t > r.capacity)
                throw std::runtime_error("ring " + std::to_string(p) + ": head outside [tail, tail + capacity]");
            const long long n = std::max(0LL, std::min({static_cast<long long>(h - t), static_cast<long long>(max_per_ring),
                                                        static_cast<long long>(mpe), budget}));
            budget -= n;
            off[p + 1] = off[p] + static_cast<int>(n);
        }
        const int total = off[P];
        if (taken)
            for (int p = 0; p < P; ++p) taken[p] = off[p + 1] - off[p];
        if (total == 0) return 0;
        const int slot = rings.slot;
        rings.slot = (slot + 1) % Rings::kSlots;
        SSLA_CK(cudaEventSynchronize(rings.copied[slot]));
        RingTake* tk = rings.pinned + static_cast<size_t>(slot) * P;
        for (int p = 0; p < P; ++p) {
            const SslaLiveRing& r = rings.r[p];
            tk[p] = RingTake{reinterpret_cast<const float4*>(r.events), r.capacity - 1, rings.next[p], r.tail,
                             r.events_done, r.flags, r.preds, off[p], off[p + 1] - off[p]};
        }
        SSLA_CK(cudaMemcpyAsync(rings.dev[slot].p, tk, sizeof(RingTake) * P, cudaMemcpyHostToDevice, st));
        SSLA_CK(cudaEventRecord(rings.copied[slot], st));
        RingArgs a{};
        a.P = P; a.n_total = total; a.cols = 5 + g.ncls;
        a.take = rings.dev[slot].as<RingTake>();
        a.ev = ws.ev.as<float4>();
        a.rflags = ws.rflags.as<uint8_t>();
        a.E4 = ws.E[4].as<StageEntry>(); a.count4 = ws.count.as<int>() + 4; a.cap4 = g.cap[4];
        a.head_dec = ws.head_dec.as<float>();
        a.ctr = rings.ctr.as<unsigned>();
        launch_ring_gather(st, a);
        check_launch("k_ring_gather");
        for (int p = 0; p < P; ++p) rings.next[p] += static_cast<unsigned long long>(off[p + 1] - off[p]);
        drain(ws.ev.as<float>(), off.data(), nullptr, st);
        launch_ring_scatter(st, a);
        check_launch("k_ring_scatter");
        prof.launches += 2;
        return total;
    }

    static unsigned long long mono_ns() {
        timespec ts;
        clock_gettime(CLOCK_MONOTONIC, &ts);
        return static_cast<unsigned long long>(ts.tv_sec) * 1000000000ull + static_cast<unsigned long long>(ts.tv_nsec);
    }

    // Serves the rings until `total` events have been drained or idle_ms
    // passes with nothing published and nothing in flight.  Each drain is
    // formed while the previous one runs; when a drain completes its time
    // and per-ring shares are logged and its events' flags copied out.
    unsigned long long serve_rings(int max_per_ring, unsigned long long total, unsigned idle_ms, SslaServeLog* log,
                                   cudaStream_t st) {
        if (rings.r.empty()) throw std::invalid_argument("ssla_engine_rings_attach first");
        const int P = g.P;
        struct Drain {
            std::vector<unsigned long long> base;
            std::vector<int> n;
            int total = 0;
            cudaEvent_t ev = nullptr;
        } dr[2];
        for (auto& d : dr) {
            d.base.resize(P);
            d.n.resize(P);
            SSLA_CK(cudaEventCreateWithFlags(&d.ev, cudaEventDisableTiming));
        }
        struct EvGuard {
            Drain* d;
            ~EvGuard() {
                for (int k = 0; k < 2; ++k) cudaEventDestroy(d[k].ev);
            }
        } guard{dr};
        if (log) { log->n = 0; log->drains = 0; }
        unsigned long long taken = 0, done = 0;
        int cur = 0;
        bool prev = false;
        unsigned long long last_new = mono_ns();
        const unsigned long long idle = static_cast<unsigned long long>(idle_ms) * 1000000ull;
        while (done < total) {
            Drain& d = dr[cur];
            int n = 0;
            if (taken < total) {
                d.base = rings.next;
                n = drain_rings(max_per_ring, static_cast<long long>(total - taken), st, d.n.data());
            }
            if (n > 0) {
                SSLA_CK(cudaEventRecord(d.ev, st));
                d.total = n;
                taken += static_cast<unsigned long long>(n);
                last_new = mono_ns();
            }
            if (prev) {
                Drain& q = dr[cur ^ 1];
                SSLA_CK(cudaEventSynchronize(q.ev));
                const unsigned long long t = mono_ns();
                done += static_cast<unsigned long long>(q.total);
                if (log) log_drain(*log, q.base, q.n, t);
                prev = false;
            }
            if (n > 0) {
                cur ^= 1;
                prev = true;
            } else if (!prev) {
                if (mono_ns() - last_new > idle) break;
                std::this_thread::yield();
            }
        }
        return done;
    }

    void log_drain(SslaServeLog& log, const std::vector<unsigned long long>& base, const std::vector<int>& n,
                   unsigned long long t) {
        const int P = g.P;
        const int k = log.drains++;
        if (k < log.cap) {
            if (log.done_ns) log.done_ns[k] = t;
            if (log.taken)
                for (int p = 0; p < P; ++p) log.taken[static_cast<size_t>(k) * P + p] = n[p];
            log.n = k + 1;
        }
        if (!log.flags_hist) return;
        for (int p = 0; p < P; ++p) {
            const SslaLiveRing& r = rings.r[p];
            uint8_t* h = log.flags_hist[p];
            if (!h || !r.flags) continue;
            for (int j = 0; j < n[p]; ++j) {
                const unsigned long long idx = base[p] + static_cast<unsigned long long>(j);
                const unsigned long long rel = idx - rings.first[p];
                if (rel < log.hist_len) h[rel] = r.flags[idx & (r.capacity - 1)];
            }
        }
    }

    // Stages 0-1 of every event and one ring record per event that passed
    // gate 1 (partition-major, stream order) into rec_dev; rec_off receives
    // the per-partition record offsets.  Synchronises `st`.
    void drain_records(const float* ev_dev, const int* off, void* rec_dev, int rec_cap, int* rec_off,
                       uint8_t* flags_dev, cudaStream_t st) {
        if (layout != LAYOUT_HYBRID) throw std::invalid_argument("ring records need the HYBRID layout");
        const int n = off[g.P];
        if (rec_cap < n) throw std::length_error("records_cap below the drain's event count");
        drain(ev_dev, off, flags_dev, st, 1);
        launch_records(st, n, ws.count.as<int>() + 2, ws.E[2].as<StageEntry>(),
                       reinterpret_cast<const float4*>(ev_dev), ws.X.as<float>(), rec_dev);
        check_launch("k_records");
        SSLA_CK(cudaMemcpyAsync(pinned_rec_off, ws.off[2].p, sizeof(int) * (g.P + 1), cudaMemcpyDeviceToHost, st));
        SSLA_CK(cudaStreamSynchronize(st));
        std::memcpy(rec_off, pinned_rec_off, sizeof(int) * (g.P + 1));
    }

    // Uploads the partition offsets into ws.ev_off through the next pinned
    // slot (waits only if that slot's previous copy has not run yet).  The
    // same offsets as the last upload on the same stream are already there
    // (ws.ev_off has no other writer), so the copy is skipped.
    std::vector<int> off_last;
    cudaStream_t off_last_st = nullptr;
    void upload_offsets(const int* off, cudaStream_t st) {
        const int P = g.P;
        if (st == off_last_st && static_cast<int>(off_last.size()) == P + 1 &&
            std::equal(off_last.begin(), off_last.end(), off))
            return;
        off_last.assign(off, off + P + 1);
        off_last_st = st;
        const int slot = off_slot;
        off_slot = (off_slot + 1) % kOffSlots;
        SSLA_CK(cudaEventSynchronize(off_done[slot]));
        int* dst = pinned_off + static_cast<size_t>(slot) * (P + 1);
        std::memcpy(dst, off, sizeof(int) * (P + 1));
        SSLA_CK(cudaMemcpyAsync(ws.ev_off.p, dst, sizeof(int) * (P + 1), cudaMemcpyHostToDevice, st));
        SSLA_CK(cudaEventRecord(off_done[slot], st));
    }

    // s_last = 3: the full path (s0..s3, head, commit).  s_last = 1: stages
    // 0-1 with gates 0-1 only (HYBRID layout), leaving the stage-2 list and
    // its layer-3 output rows for k_records.
    void drain(const float* ev_dev, const int* off, uint8_t* flags_dev, cudaStream_t st, int s_last = 3) {
        DeviceGuard dg(device);
        const int n = drain_front(ev_dev, off, st, s_last);
        if (s_last < 3) {
            run_layers(st, g, ws, parts.as<PartState>(), L, &head, false, record, prof, 2 * (s_last + 1));
            if (flags_dev && n > 0)
                SSLA_CK(cudaMemcpyAsync(flags_dev, ws.rflags.p, n, cudaMemcpyDeviceToDevice, st));
            return;
        }
        run_layers(st, g, ws, parts.as<PartState>(), L, &head, true, record, prof);
        drain_back(n, flags_dev, st);
    }

    // Preprocess, stage-0 tile lists, gates with layer 0, stage lists and
    // their tile lists up to stage s_last; returns the event count.
    int drain_front(const float* ev_dev, const int* off, cudaStream_t st, int s_last) {
        const int P = g.P;
        if (off[0] != 0) throw std::invalid_argument("part_offsets[0] must be 0");
        for (int p = 0; p < P; ++p)
            if (off[p + 1] < off[p]) throw std::invalid_argument("part_offsets must be non-decreasing");
        for (int p = 0; p < P; ++p)
            if (off[p + 1] - off[p] > mpe)
                throw std::length_error("partition holds more events than max_events_per_partition");
        const int n = off[P];
        if (n > max_events) throw std::length_error("more events than max_events");
        ws.n_active = n;
        last_n = n;
        prof.begin(st);
        upload_offsets(off, st);
        const float4* ev = reinterpret_cast<const float4*>(ev_dev);
        launch_prep(st, ev, n, g.W[0], g.H[0], ws.ev_xy.as<uint32_t>(), ws.rflags.as<uint8_t>());
        check_launch("k_prep");
        prof.mark("prep", n > 0 ? 1 : 0, st);
        // stage-0 tile lists
        FilterArgs fa{};
        fa.g = g; fa.stage = 0; fa.ev_xy = ws.ev_xy.as<uint32_t>(); fa.rflags = ws.rflags.as<uint8_t>();
        fa.range = ws.ev_off.as<int>(); fa.tl = ws.tl[0].as<int2>(); fa.tl_cnt = ws.tl_cnt[0].as<int>();
        if (strip.on) {                            // a strip's events: its rows and the bands
            fa.ev_row_lo = std::max(0, strip.lo - strip.band);
            fa.ev_row_hi = std::min(g.H[0], strip.hi + strip.band);
        }
        launch_filter(st, fa);
        check_launch("k_filter s0");
        prof.mark("filter_s0", 1, st);
        // gates + preprocess + layer-0 qvg
        GateArgs ga{};
        ga.g = g; ga.ev = ev; ga.ev_off = ws.ev_off.as<int>(); ga.tl0 = ws.tl[0].as<int2>();
        ga.tl0_cnt = ws.tl_cnt[0].as<int>(); ga.parts = parts.as<PartState>();
        ga.rflags = ws.rflags.as<uint8_t>(); ga.X1 = ws.X.as<float>(); ga.Rcopy = ws.R_B.as<float>();
        ga.L0 = L[0];
        ga.n_gates = (s_last >= 3) ? 4 : 2;
        launch_gates(st, ga);
        check_launch("k_gates");
        fa.zero_work = ws.work.as<int>();
        launch_flag_s0(st, fa);                    // layer-1 output flags into the stage-0 lists
        check_launch("k_flag_s0");
        prof.mark("gates", 2, st);
        // stage lists
        CompactArgs ca{};
        ca.g = g; ca.s_first = 0; ca.tiles_per_part = ws.tiles_per_part; ca.ctile = ws.ctile; ca.ev_off = ws.ev_off.as<int>();
        ca.rflags = ws.rflags.as<uint8_t>(); ca.ev_xy = ws.ev_xy.as<uint32_t>();
        ca.tilecnt = ws.tilecnt.as<int>(); ca.tilebase = ws.tilebase.as<int>();
        for (int s = 0; s <= 4; ++s) { ca.E[s] = ws.E[s].as<StageEntry>(); ca.off[s] = ws.off[s].as<int>(); }
        ca.count = ws.count.as<int>();
        launch_compact(st, ca);
        check_launch("k_compact");
        prof.mark("compact", 3, st);
        for (int s = 1; s <= s_last; ++s) {
            FilterArgs f{};
            f.g = g; f.stage = s; f.E = ws.E[s].as<StageEntry>(); f.rflags = ws.rflags.as<uint8_t>();
            f.range = ws.off[s].as<int>(); f.tl = ws.tl[s].as<int2>(); f.tl_cnt = ws.tl_cnt[s].as<int>();
            f.out_bit = static_cast<uint8_t>(F_R1 << s);
            f.ev_row_lo = fa.ev_row_lo;
            f.ev_row_hi = fa.ev_row_hi;
            launch_filter(st, f);
            check_launch("k_filter");
        }
        prof.mark("filter_s123", s_last, st);
        return n;
    }

    // Last-writer prediction commit and the event flags.
    void drain_back(int n, uint8_t* flags_dev, cudaStream_t st) {
        CommitArgs cm{};
        cm.g = g; cm.E4 = ws.E[4].as<StageEntry>(); cm.off4 = ws.off[4].as<int>();
        cm.head_dec = ws.head_dec.as<float>(); cm.head_raw = ws.head_raw.as<float>();
        cm.parts = parts.as<PartState>();
        launch_commit(st, cm);
        check_launch("k_commit");
        prof.mark("commit", 1, st);
        if (flags_dev && n > 0)
            SSLA_CK(cudaMemcpyAsync(flags_dev, ws.rflags.p, n, cudaMemcpyDeviceToDevice, st));
    }
};

// ---------------------------------------------------------------------------
// drain_n (stage-2 entry) on the reference's HybridS2S3Config buffers.
// A process-wide workspace per device is grown on demand.
// ---------------------------------------------------------------------------
struct DrainN {
    std::mutex mu;
    struct PerDev {
        Workspace ws;
        Geo g{};
        int P = 0, mpe = 0, n_max = 0, H2 = 0, W2 = 0, window = 0;
        DevBuf parts, outs, clks, rec;
        int* pinned = nullptr;
    };
    std::vector<std::unique_ptr<PerDev>> dev;

    int run(const HybridS2S3Config* cfg, const HybridInputRec* const* rings, const int* ns,
            HybridS2S3OutputSlot* const* outs, unsigned long long* const* clks, cudaStream_t st) {
        std::lock_guard<std::mutex> lk(mu);
        int device = 0;
        SSLA_CK(cudaGetDevice(&device));
        if (static_cast<int>(dev.size()) <= device) dev.resize(device + 1);
        if (!dev[device]) dev[device].reset(new PerDev());
        PerDev& d = *dev[device];
        const int P = cfg->n_blocks;
        if (P < 1 || P > SSLA_MAX_BLOCKS) throw std::invalid_argument("cfg->n_blocks must be 1..16");
        if (cfg->H2 <= 0 || cfg->W2 <= 0 || cfg->H3 != cfg->H2 / 2 || cfg->W3 != cfg->W2 / 2)
            throw std::invalid_argument("cfg grid sizes must satisfy H3 = H2/2, W3 = W2/2");
        if ((cfg->H2 % 2) || (cfg->W2 % 2)) throw std::invalid_argument("H2 and W2 must be even");
        for (int b = 1; b < P; ++b)
            for (int li = 0; li < 4; ++li)
                if (std::memcmp(&cfg->layers[b][li], &cfg->layers[0][li], sizeof(LayerWeightsS2S3)) != 0)
                    throw std::invalid_argument("all blocks must share the same layer weights");
        std::vector<int> off(P + 1, 0);
        int mpe = 1;
        for (int b = 0; b < P; ++b) {
            if (ns[b] < 0) throw std::invalid_argument("negative record count");
            off[b + 1] = off[b] + ns[b];
            mpe = std::max(mpe, ns[b]);
        }
        const int n = off[P];
        const int window = cfg->tdrop_window;
        if (d.P != P || d.mpe < mpe || d.n_max < n || d.H2 != cfg->H2 || d.W2 != cfg->W2 ||
            d.window != window) {
            // full-resolution geometry whose stage-2 grid is H2 x W2
            make_geo(d.g, cfg->H2 * 4, cfg->W2 * 4, P, LAYOUT_HYBRID, window, 2);
            d.P = P; d.mpe = std::max(mpe, d.mpe); d.n_max = std::max(n, d.n_max);
            d.H2 = cfg->H2; d.W2 = cfg->W2; d.window = window;
            SSLA_CK(cudaStreamSynchronize(st));
            d.ws.plan(d.g, P, d.mpe, d.n_max, 2, false);
            d.parts.alloc(sizeof(PartState) * P);
            d.outs.alloc(sizeof(void*) * P);
            d.clks.alloc(sizeof(void*) * P);
            d.rec.alloc(sizeof(HybridInputRec) * static_cast<size_t>(std::max(d.n_max, 1)));
            if (d.pinned) cudaFreeHost(d.pinned);
            d.pinned = nullptr;
            SSLA_CK(cudaMallocHost(&d.pinned, sizeof(int) * (P + 1) + sizeof(PartState) * P +
                                                  2 * sizeof(void*) * P));
        }
        Workspace& w = d.ws;
        w.n_active = n;
        // per-block state and parameters (pinned staging, async upload)
        char* pin = reinterpret_cast<char*>(d.pinned);
        int* p_off = reinterpret_cast<int*>(pin);
        PartState* p_parts = reinterpret_cast<PartState*>(pin + sizeof(int) * (P + 1));
        void** p_outs = reinterpret_cast<void**>(pin + sizeof(int) * (P + 1) + sizeof(PartState) * P);
        void** p_clks = p_outs + P;
        std::memcpy(p_off, off.data(), sizeof(int) * (P + 1));
        for (int b = 0; b < P; ++b) {
            PartState ps{};
            for (int li = 0; li < 4; ++li) ps.hidden[4 + li] = cfg->hidden[b][li];
            ps.cnt[2] = cfg->tdrop_s2[b];
            ps.cnt[3] = cfg->tdrop_s3[b];
            ps.own_x0 = cfg->strip[b].owned_lo; ps.own_x1 = cfg->strip[b].owned_hi;
            ps.own_y0 = cfg->strip[b].owned_y_lo; ps.own_y1 = cfg->strip[b].owned_y_hi;
            p_parts[b] = ps;
            p_outs[b] = outs ? outs[b] : nullptr;
            p_clks[b] = clks ? clks[b] : nullptr;
        }
        SSLA_CK(cudaMemcpyAsync(w.ev_off.p, p_off, sizeof(int) * (P + 1), cudaMemcpyHostToDevice, st));
        SSLA_CK(cudaMemcpyAsync(w.off[2].p, p_off, sizeof(int) * (P + 1), cudaMemcpyHostToDevice, st));
        SSLA_CK(cudaMemcpyAsync(d.parts.p, p_parts, sizeof(PartState) * P, cudaMemcpyHostToDevice, st));
        SSLA_CK(cudaMemcpyAsync(d.outs.p, p_outs, sizeof(void*) * P, cudaMemcpyHostToDevice, st));
        SSLA_CK(cudaMemcpyAsync(d.clks.p, p_clks, sizeof(void*) * P, cudaMemcpyHostToDevice, st));
        launch_stamp(st, w.stamps.as<unsigned long long>());
        check_launch("k_stamp");
        for (int b = 0; b < P; ++b)
            if (ns[b] > 0)
                SSLA_CK(cudaMemcpyAsync(d.rec.as<HybridInputRec>() + off[b], rings[b],
                                        sizeof(HybridInputRec) * ns[b], cudaMemcpyDeviceToDevice, st));
        launch_prep_records(st, d.rec.p, n, w.E[2].as<StageEntry>(), w.ev_xy.as<uint32_t>(),
                            w.rflags.as<uint8_t>(), w.X.as<float>());
        check_launch("k_prep_records");
        const Geo& g = d.g;
        FilterArgs f2{};
        f2.g = g; f2.stage = 2; f2.E = w.E[2].as<StageEntry>(); f2.rflags = w.rflags.as<uint8_t>();
        f2.range = w.off[2].as<int>(); f2.tl = w.tl[2].as<int2>(); f2.tl_cnt = w.tl_cnt[2].as<int>();
        f2.out_bit = 0;   // gates not known yet; refiltered below
        launch_filter(st, f2);
        check_launch("k_filter s2");
        Gate2Args ga{};
        ga.g = g; ga.rec_off = w.ev_off.as<int>(); ga.tl2 = w.tl[2].as<int2>(); ga.tl2_cnt = w.tl_cnt[2].as<int>();
        ga.parts = d.parts.as<PartState>(); ga.rflags = w.rflags.as<uint8_t>();
        launch_gates_s2(st, ga);
        check_launch("k_gates_s2");
        CompactArgs ca{};
        ca.g = g; ca.s_first = 2; ca.tiles_per_part = w.tiles_per_part; ca.ctile = w.ctile; ca.ev_off = w.ev_off.as<int>();
        ca.rflags = w.rflags.as<uint8_t>(); ca.ev_xy = w.ev_xy.as<uint32_t>();
        ca.tilecnt = w.tilecnt.as<int>(); ca.tilebase = w.tilebase.as<int>();
        for (int s = 0; s <= 4; ++s) { ca.E[s] = w.E[s].as<StageEntry>(); ca.off[s] = w.off[s].as<int>(); }
        ca.count = w.count.as<int>();
        launch_compact(st, ca);
        check_launch("k_compact");
        for (int s = 2; s < 4; ++s) {     // stage-2 lists again, now with the output bit
            FilterArgs f{};
            f.g = g; f.stage = s; f.E = w.E[s].as<StageEntry>(); f.rflags = w.rflags.as<uint8_t>();
            f.range = w.off[s].as<int>(); f.tl = w.tl[s].as<int2>(); f.tl_cnt = w.tl_cnt[s].as<int>();
            f.out_bit = static_cast<uint8_t>(F_R1 << s);
            launch_filter(st, f);
            check_launch("k_filter");
        }
        // count[2] = n for the entry kernel
        SSLA_CK(cudaMemcpyAsync(w.count.as<int>() + 2, p_off + P, sizeof(int), cudaMemcpyHostToDevice, st));
        DevLayer L[8]{};
        for (int li = 0; li < 4; ++li) {
            const LayerWeightsS2S3& lw = cfg->layers[0][li];
            L[4 + li] = DevLayer{lw.qvgIn, lw.goW, lw.input_proj, lw.ln_gamma, lw.ln_beta};
        }
        // layer-4 residual (input_proj * feat1); the layer's qvg GEMM reads
        // the same X rows inside run_layers
        GemmArgs gr{};
        gr.list = 2; gr.count = w.count.as<int>(); gr.g_cap = n; gr.X = w.X.as<float>(); gr.A2 = 9;
        gr.W = L[4].ipT; gr.R = w.R_A.as<float>(); gr.colmode = COLS_RES; gr.n_cols = gemm_cols(4, COLS_RES);
        launch_gemm(st, 4, gr, n);
        check_launch("k_gemm entry res");
        DevHead nohead{};
        Prof noprof;
        run_layers(st, g, w, d.parts.as<PartState>(), L, &nohead, false, false, noprof);
        if (outs) {
            launch_write_slots(st, n, P, w.ev_off.as<int>(), w.rflags.as<uint8_t>(), w.ev_xy.as<uint32_t>(),
                               d.parts.as<PartState>(), w.slot_feat.as<float>(), d.outs.as<void*>());
            check_launch("k_write_slots");
        }
        launch_stamp(st, w.stamps.as<unsigned long long>() + 1);
        check_launch("k_stamp");
        if (clks) {
            launch_fill_clk(st, P, w.ev_off.as<int>(), w.stamps.as<unsigned long long>(),
                            d.clks.as<unsigned long long*>());
            check_launch("k_fill_clk");
        }
        // the pinned staging buffers are reused by the next call
        SSLA_CK(cudaStreamSynchronize(st));
        return SSLA_OK;
    }
};

DrainN& drain_n_state() {
    static DrainN* d = new DrainN();   // process lifetime
    return *d;
}

template <typename F>
int guarded(F&& f) {
    try {
        return f();
    } catch (const CudaError& e) {
        g_last_error = e.what();
        return SSLA_ERR_CUDA;
    } catch (const std::length_error& e) {
        g_last_error = e.what();
        return SSLA_ERR_CAPACITY;
    } catch (const std::invalid_argument& e) {
        g_last_error = e.what();
        return SSLA_ERR_ARG;
    } catch (const std::bad_alloc&) {
        g_last_error = "host allocation failed";
        return SSLA_ERR_CUDA;
    } catch (const std::exception& e) {
        g_last_error = e.what();
        return SSLA_ERR_LOAD;
    }
}

}  // namespace ssla

// ---------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------
struct SslaEngine {
    ssla::Engine e;
};

extern "C" {

const char* ssla_last_error(void) { return ssla::g_last_error.c_str(); }
const char* ssla_version(void) { return "ssla_b200 0.1.0 (sm_100a)"; }
float ssla_expf_host(float x) { return ssla::ssla_expf(x); }
float ssla_sigmoidf_host(float x) { return ssla::ssla_sigmoidf(x); }

int ssla_engine_create(const char* weights_dir, const SslaEngineConfig* cfg, SslaEngine** out) {
    if (!weights_dir || !cfg || !out) { ssla::g_last_error = "null argument"; return SSLA_ERR_ARG; }
    *out = nullptr;
    if (cfg->n_partitions < 1 || cfg->n_partitions > ssla::kMaxParts || cfg->max_events < 1 ||
        (cfg->layout != SSLA_LAYOUT_DECOMP && cfg->layout != SSLA_LAYOUT_HYBRID)) {
        ssla::g_last_error = "invalid SslaEngineConfig";
        return SSLA_ERR_ARG;
    }
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) {
        cudaGetLastError();
        ssla::g_last_error = "no CUDA device";
        return SSLA_ERR_NO_DEVICE;
    }
    auto* h = new (std::nothrow) SslaEngine();
    if (!h) { ssla::g_last_error = "host allocation failed"; return SSLA_ERR_CUDA; }
    const int rc = ssla::guarded([&] { h->e.create(weights_dir, *cfg); return SSLA_OK; });
    if (rc != SSLA_OK) { delete h; return rc; }
    *out = h;
    return SSLA_OK;
}

void ssla_engine_destroy(SslaEngine* eng) {
    if (!eng) return;
    int prev = -1;
    cudaGetDevice(&prev);
    cudaSetDevice(eng->e.device);
    cudaDeviceSynchronize();
    delete eng;
    if (prev >= 0) cudaSetDevice(prev);
}

int ssla_engine_reset(SslaEngine* eng, void* stream) {
    if (!eng) { ssla::g_last_error = "null engine"; return SSLA_ERR_ARG; }
    return ssla::guarded([&] { eng->e.reset(static_cast<cudaStream_t>(stream)); return SSLA_OK; });
}

int ssla_engine_drain_device(SslaEngine* eng, const float* events_dev, const int* part_offsets,
                             uint8_t* flags_dev, void* stream) {
    if (!eng || !part_offsets || (!events_dev && part_offsets[eng->e.g.P] > 0)) {
        ssla::g_last_error = "null argument";
        return SSLA_ERR_ARG;
    }
    return ssla::guarded([&] {
        eng->e.drain(events_dev, part_offsets, flags_dev, static_cast<cudaStream_t>(stream));
        return SSLA_OK;
    });
}

int ssla_engine_drain_host_async(SslaEngine* eng, const float* events_host, const int* part_offsets,
                                 uint8_t* flags_host, float* preds_host, void* stream) {
    if (!eng || !part_offsets) { ssla::g_last_error = "null argument"; return SSLA_ERR_ARG; }
    return ssla::guarded([&] {
        ssla::DeviceGuard dg(eng->e.device);
        eng->e.drain_host_async(events_host, part_offsets, flags_host, preds_host,
                                static_cast<cudaStream_t>(stream));
        return SSLA_OK;
    });
}

int ssla_engine_drain_host(SslaEngine* eng, const float* events_host, const int* part_offsets,
                           uint8_t* flags_host, void* stream) {
    if (!eng || !part_offsets) { ssla::g_last_error = "null argument"; return SSLA_ERR_ARG; }
    return ssla::guarded([&] {
        ssla::Engine& e = eng->e;
        ssla::DeviceGuard dg(e.device);
        cudaStream_t st = static_cast<cudaStream_t>(stream);
        const int n = part_offsets[e.g.P];
        if (n < 0 || n > e.max_events) throw std::length_error("more events than max_events");
        if (n > 0) {
            if (!events_host) throw std::invalid_argument("null events");
            SSLA_CK(cudaMemcpyAsync(e.ws.ev.p, events_host, sizeof(float) * 4 * n, cudaMemcpyHostToDevice, st));
        }
        e.drain(e.ws.ev.as<float>(), part_offsets, nullptr, st);
        if (flags_host && n > 0)
            SSLA_CK(cudaMemcpyAsync(flags_host, e.ws.rflags.p, n, cudaMemcpyDeviceToHost, st));
        SSLA_CK(cudaStreamSynchronize(st));
        return SSLA_OK;
    });
}

int ssla_engine_step(SslaEngine* eng, int partition, const float* event, uint8_t* flag_out,
                     float* pred_out, void* stream) {
    if (!eng || !event) { ssla::g_last_error = "null argument"; return SSLA_ERR_ARG; }
    return ssla::guarded([&] {
        ssla::Engine& e = eng->e;
        ssla::DeviceGuard dg(e.device);
        e.step(partition, event, flag_out, pred_out, static_cast<cudaStream_t>(stream));
        return SSLA_OK;
    });
}

int ssla_engine_step_latency(SslaEngine* eng, int partition, const float* events_host, int n,
                             double* latency_us, uint8_t* flags_out) {
    if (!eng || !events_host || !latency_us || n < 0) { ssla::g_last_error = "null argument"; return SSLA_ERR_ARG; }
    return ssla::guarded([&] {
        ssla::Engine& e = eng->e;
        ssla::DeviceGuard dg(e.device);
        cudaStream_t st = nullptr;
        uint8_t* flag = nullptr;
        float* pred = nullptr;
        SSLA_CK(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
        SSLA_CK(cudaMallocHost(&flag, 1));
        SSLA_CK(cudaMallocHost(&pred, sizeof(float) * (5 + e.g.ncls)));
        for (int i = 0; i < n; ++i) {
            const auto t0 = std::chrono::steady_clock::now();
            e.step(partition, events_host + 4 * i, flag, pred, st);
            SSLA_CK(cudaStreamSynchronize(st));
            const auto t1 = std::chrono::steady_clock::now();
            latency_us[i] = std::chrono::duration<double, std::micro>(t1 - t0).count();
            if (flags_out) flags_out[i] = *flag;
        }
        cudaFreeHost(pred);
        cudaFreeHost(flag);
        cudaStreamDestroy(st);
        e.check_step_status();
        return SSLA_OK;
    });
}

int ssla_engine_rings_attach(SslaEngine* eng, const SslaLiveRing* rings, int n_rings) {
    if (!eng || !rings) { ssla::g_last_error = "null argument"; return SSLA_ERR_ARG; }
    return ssla::guarded([&] {
        ssla::DeviceGuard dg(eng->e.device);
        eng->e.rings_attach(rings, n_rings);
        return SSLA_OK;
    });
}

int ssla_engine_drain_rings(SslaEngine* eng, int max_per_ring, long long max_total, int* taken, int* n_taken,
                            void* stream) {
    if (!eng) { ssla::g_last_error = "null argument"; return SSLA_ERR_ARG; }
    return ssla::guarded([&] {
        ssla::DeviceGuard dg(eng->e.device);
        const int n = eng->e.drain_rings(max_per_ring, max_total, static_cast<cudaStream_t>(stream), taken);
        if (n_taken) *n_taken = n;
        return SSLA_OK;
    });
}

int ssla_engine_serve_rings(SslaEngine* eng, int max_per_ring, unsigned long long total, unsigned idle_timeout_ms,
                            SslaServeLog* log, unsigned long long* served, void* stream) {
    if (!eng) { ssla::g_last_error = "null argument"; return SSLA_ERR_ARG; }
    return ssla::guarded([&] {
        ssla::DeviceGuard dg(eng->e.device);
        const unsigned long long n =
            eng->e.serve_rings(max_per_ring, total, idle_timeout_ms, log, static_cast<cudaStream_t>(stream));
        if (served) *served = n;
        return SSLA_OK;
    });
}

int ssla_engine_set_owned(SslaEngine* eng, int partition, int x0, int x1, int y0, int y1, void* stream) {
    if (!eng) { ssla::g_last_error = "null argument"; return SSLA_ERR_ARG; }
    return ssla::guarded([&] {
        ssla::DeviceGuard dg(eng->e.device);
        eng->e.set_owned(partition, x0, x1, y0, y1, static_cast<cudaStream_t>(stream));
        return SSLA_OK;
    });
}

int ssla_engine_strip_init(SslaEngine* eng, int lo, int hi, int band_rows, int has_up, int has_down,
                           int cap_rows) {
    if (!eng) { ssla::g_last_error = "null argument"; return SSLA_ERR_ARG; }
    return ssla::guarded([&] {
        ssla::DeviceGuard dg(eng->e.device);
        eng->e.strip_init(lo, hi, band_rows, has_up, has_down, cap_rows);
        return SSLA_OK;
    });
}

int ssla_engine_strip_recv_buffer(SslaEngine* eng, int side, void** dev_ptr, void* ipc_handle) {
    if (!eng) { ssla::g_last_error = "null argument"; return SSLA_ERR_ARG; }
    return ssla::guarded([&] {
        ssla::DeviceGuard dg(eng->e.device);
        eng->e.strip_recv_buffer(side, dev_ptr, ipc_handle);
        return SSLA_OK;
    });
}

int ssla_engine_strip_connect(SslaEngine* eng, int side, void* peer_dev_ptr, const void* peer_ipc_handle) {
    if (!eng) { ssla::g_last_error = "null argument"; return SSLA_ERR_ARG; }
    return ssla::guarded([&] {
        ssla::DeviceGuard dg(eng->e.device);
        eng->e.strip_connect(side, peer_dev_ptr, peer_ipc_handle);
        return SSLA_OK;
    });
}

int ssla_engine_strip_drain(SslaEngine* eng, const float* events_dev, int n, uint8_t* flags_dev, void* stream) {
    if (!eng || n < 0 || (n > 0 && !events_dev)) { ssla::g_last_error = "null argument"; return SSLA_ERR_ARG; }
    return ssla::guarded([&] {
        ssla::DeviceGuard dg(eng->e.device);
        eng->e.strip_drain(events_dev, n, flags_dev, static_cast<cudaStream_t>(stream));
        return SSLA_OK;
    });
}

int ssla_strip_drain_lockstep(SslaEngine* const* engines, int k, const float* const* events_dev, const int* n,
                              uint8_t* const* flags_dev, void* stream) {
    if (!engines || k < 1 || !events_dev || !n) { ssla::g_last_error = "null argument"; return SSLA_ERR_ARG; }
    return ssla::guarded([&] {
        const cudaStream_t st = static_cast<cudaStream_t>(stream);
        for (int i = 0; i < k; ++i) {
            if (!engines[i] || n[i] < 0) throw std::invalid_argument("null engine or negative count");
            if (engines[i]->e.device != engines[0]->e.device)
                throw std::invalid_argument("lockstep strips share one device");
        }
        ssla::DeviceGuard dg(engines[0]->e.device);
        for (int j = 0; j < 7; ++j) {
            for (int i = 0; i < k; ++i)
                engines[i]->e.strip_step(j, events_dev[i], n[i], flags_dev ? flags_dev[i] : nullptr, st);
            if (j < 6) {
                unsigned long long seq = 0;
                for (int i = 0; i < k; ++i) seq = ++engines[i]->e.strip.seq;
                for (int i = 0; i < k; ++i) engines[i]->e.strip_xfer(j, true, seq, false, st);
                for (int i = 0; i < k; ++i) engines[i]->e.strip_xfer(j, false, seq, false, st);
            }
        }
        return SSLA_OK;
    });
}

int ssla_engine_strip_status(SslaEngine* eng, unsigned* status) {
    if (!eng || !status) { ssla::g_last_error = "null argument"; return SSLA_ERR_ARG; }
    return ssla::guarded([&] {
        ssla::DeviceGuard dg(eng->e.device);
        *status = eng->e.strip_status();
        return SSLA_OK;
    });
}

int ssla_engine_live_start(SslaEngine* eng, int partition, const SslaLiveRing* ring, unsigned idle_timeout_ms,
                           void* stream) {
    if (!eng || !ring) { ssla::g_last_error = "null argument"; return SSLA_ERR_ARG; }
    return ssla::guarded([&] {
        ssla::DeviceGuard dg(eng->e.device);
        eng->e.live_start(partition, *ring, idle_timeout_ms, static_cast<cudaStream_t>(stream));
        return SSLA_OK;
    });
}

int ssla_engine_live_join(SslaEngine* eng, unsigned* status) {
    if (!eng) { ssla::g_last_error = "null argument"; return SSLA_ERR_ARG; }
    return ssla::guarded([&] {
        ssla::DeviceGuard dg(eng->e.device);
        const unsigned v = eng->e.live_join(false);
        if (status) *status = v;
        if (v & 0xFFu) {
            ssla::g_last_error = ssla::Engine::live_status_text(v);
            return static_cast<int>(SSLA_ERR_CUDA);
        }
        return static_cast<int>(SSLA_OK);
    });
}

int ssla_engine_fill_s2s3_config(SslaEngine* eng, HybridS2S3Config* cfg, int block) {
    if (!eng || !cfg || block < 0 || block >= SSLA_MAX_BLOCKS) {
        ssla::g_last_error = "bad argument";
        return SSLA_ERR_ARG;
    }
    const ssla::Engine& e = eng->e;
    for (int li = 0; li < 4; ++li) {
        const ssla::DevLayer& L = e.L[4 + li];
        LayerWeightsS2S3& w = cfg->layers[block][li];
        w.qvgIn = L.qvgT;
        w.goW = L.goWT;
        w.input_proj = L.ipT;
        w.ln_gamma = L.gamma;
        w.ln_beta = L.beta;
    }
    const ssla::DevHead& h = e.head;
    cfg->head_W = nullptr;
    cfg->head_b = nullptr;
    cfg->head_cls_conv_W = h.cls_convT;
    cfg->head_cls_conv_b = h.cls_conv_b;
    cfg->head_cls_pred_W = h.cls_predT;
    cfg->head_cls_pred_b = h.cls_pred_b;
    cfg->head_reg_conv_W = h.reg_convT;
    cfg->head_reg_conv_b = h.reg_conv_b;
    cfg->head_reg_pred_W = h.reg_predT;
    cfg->head_reg_pred_b = h.reg_pred_b;
    cfg->head_obj_pred_W = h.obj_predT;
    cfg->head_obj_pred_b = h.obj_pred_b;
    cfg->head_out_dim = 5 + e.g.ncls;
    return SSLA_OK;
}

int ssla_engine_set_head_mode(SslaEngine* eng, int mode) {
    if (!eng || (mode != SSLA_HEAD_EXACT && mode != SSLA_HEAD_TENSOR)) {
        ssla::g_last_error = "bad argument";
        return SSLA_ERR_ARG;
    }
    return ssla::guarded([&] {
        ssla::DeviceGuard dg(eng->e.device);
        SSLA_CK(cudaDeviceSynchronize());           // no drain in flight reads the head selection
        ssla::Engine& e = eng->e;
        e.head.tc_w1 = mode == SSLA_HEAD_TENSOR ? e.head_tc.as<float>() : nullptr;
        e.head.tc_err = mode == SSLA_HEAD_TENSOR ? e.head_tc_err : nullptr;
        return SSLA_OK;
    });
}

int ssla_engine_head_status(SslaEngine* eng, unsigned* status) {
    if (!eng || !status) { ssla::g_last_error = "null argument"; return SSLA_ERR_ARG; }
    return ssla::guarded([&] {
        ssla::DeviceGuard dg(eng->e.device);
        SSLA_CK(cudaDeviceSynchronize());
        *status = eng->e.head_tc_err ? __atomic_exchange_n(eng->e.head_tc_err, 0u, __ATOMIC_ACQ_REL) : 0u;
        return SSLA_OK;
    });
}

int ssla_engine_live_withhold_completion(SslaEngine* eng, long long ring_index) {
    if (!eng || ring_index < -1) { ssla::g_last_error = "bad argument"; return SSLA_ERR_ARG; }
    return ssla::guarded([&] {
        if (eng->e.live_running) throw std::invalid_argument("a live loop is running on this engine");
        eng->e.live_withhold = ring_index < 0 ? ~0ull : static_cast<unsigned long long>(ring_index);
        return SSLA_OK;
    });
}

int ssla_engine_live_latency(SslaEngine* eng, int partition, const float* events_host, int n,
                             double* latency_us, uint8_t* flags_out, float* preds_out) {
    if (!eng || !events_host || !latency_us || n < 0) { ssla::g_last_error = "null argument"; return SSLA_ERR_ARG; }
    return ssla::guarded([&] {
        ssla::Engine& e = eng->e;
        ssla::DeviceGuard dg(e.device);
        constexpr unsigned long long cap = 1024;
        const int cols = 5 + e.g.ncls;
        struct Pinned {
            void* p = nullptr;
            ~Pinned() { if (p) cudaFreeHost(p); }
        } ev, words, fl, pr;
        SSLA_CK(cudaHostAlloc(&ev.p, 16 * cap, cudaHostAllocMapped));
        SSLA_CK(cudaHostAlloc(&words.p, 64, cudaHostAllocMapped));
        SSLA_CK(cudaHostAlloc(&fl.p, cap, cudaHostAllocMapped));
        SSLA_CK(cudaHostAlloc(&pr.p, sizeof(float) * cols * cap, cudaHostAllocMapped));
        std::memset(words.p, 0, 64);
        auto* w = static_cast<unsigned long long*>(words.p);
        SslaLiveRing r{};
        r.events = static_cast<float*>(ev.p);
        r.capacity = cap;
        r.head = w;
        r.tail = w + 1;
        r.events_done = w + 2;
        r.stop_flag = reinterpret_cast<int*>(w + 3);
        r.flags = static_cast<uint8_t*>(fl.p);
        r.preds = static_cast<float*>(pr.p);
        cudaStream_t st = nullptr;
        SSLA_CK(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
        struct StreamGuard {
            cudaStream_t s;
            ~StreamGuard() { cudaStreamDestroy(s); }
        } sg{st};
        e.live_start(partition, r, 2000, st);
        bool timed_out = false;
        for (int i = 0; i < n && !timed_out; ++i) {
            const unsigned long long slot = static_cast<unsigned long long>(i) & (cap - 1);
            std::memcpy(static_cast<float*>(ev.p) + 4 * slot, events_host + 4 * static_cast<size_t>(i), 16);
            __atomic_store_n(r.head, static_cast<unsigned long long>(i) + 1, __ATOMIC_RELEASE);
            const auto t0 = std::chrono::steady_clock::now();
            auto t1 = t0;
            while (__atomic_load_n(r.events_done, __ATOMIC_ACQUIRE) < static_cast<unsigned long long>(i) + 1) {
                t1 = std::chrono::steady_clock::now();
                if (t1 - t0 > std::chrono::seconds(1)) { timed_out = true; break; }
            }
            t1 = std::chrono::steady_clock::now();
            latency_us[i] = std::chrono::duration<double, std::micro>(t1 - t0).count();
            const uint8_t f = r.flags[slot];
            if (flags_out) flags_out[i] = f;
            if (preds_out && (f & SSLA_F_R4))
                std::memcpy(preds_out + static_cast<size_t>(i) * cols, r.preds + slot * cols, sizeof(float) * cols);
        }
        __atomic_store_n(r.stop_flag, 1, __ATOMIC_RELEASE);
        e.live_join();
        if (timed_out) throw ssla::CudaError("live loop: an event was not finished within 1 s");
        return SSLA_OK;
    });
}

int ssla_engine_drain_records(SslaEngine* eng, const float* events_dev, const int* part_offsets,
                              void* records_dev, int records_cap, int* record_offsets,
                              uint8_t* flags_dev, void* stream) {
    if (!eng || !part_offsets || !record_offsets || (!records_dev && records_cap > 0)) {
        ssla::g_last_error = "null argument";
        return SSLA_ERR_ARG;
    }
    return ssla::guarded([&] {
        ssla::Engine& e = eng->e;
        ssla::DeviceGuard dg(e.device);
        e.drain_records(events_dev, part_offsets, records_dev, records_cap, record_offsets, flags_dev,
                        static_cast<cudaStream_t>(stream));
        return SSLA_OK;
    });
}

int ssla_engine_state_bytes(SslaEngine* eng, int kind, int index, size_t* bytes) {
    if (!eng || !bytes) { ssla::g_last_error = "null argument"; return SSLA_ERR_ARG; }
    *bytes = eng->e.state_elems(kind, index) * ssla::Engine::elem_size(kind);
    return *bytes ? SSLA_OK : SSLA_ERR_ARG;
}

static int state_args_ok(SslaEngine* eng, int kind, int partition, int index) {
    if (!eng) return 0;
    // partition -1: every partition's buffer of a per-partition state kind, back to back
    const bool all = partition == -1 && kind <= SSLA_STATE_VERSION;
    if (!all && (partition < 0 || partition >= eng->e.g.P)) return 0;
    if (kind == SSLA_STATE_HIDDEN && (index < 0 || index > 7)) return 0;
    if (kind == SSLA_STATE_COUNTER && (index < 0 || index > 3)) return 0;
    if (kind == SSLA_STATE_STAGE_OUT && (index < 0 || index > 3 || !eng->e.record)) return 0;
    if (kind < 0 || kind > SSLA_STATE_FLAGS) return 0;
    return 1;
}

int ssla_engine_read_state(SslaEngine* eng, int kind, int partition, int index, void* host_dst, size_t bytes) {
    if (!state_args_ok(eng, kind, partition, index) || !host_dst) {
        ssla::g_last_error = "bad state selector";
        return SSLA_ERR_ARG;
    }
    return ssla::guarded([&] {
        ssla::Engine& e = eng->e;
        ssla::DeviceGuard dg(e.device);
        const size_t full = e.state_elems(kind, index) * ssla::Engine::elem_size(kind) *
                            (partition < 0 ? static_cast<size_t>(e.g.P) : 1u);
        if (bytes > full) throw std::invalid_argument("read larger than the state buffer");
        SSLA_CK(cudaDeviceSynchronize());
        SSLA_CK(cudaMemcpy(host_dst, e.state_ptr(kind, partition < 0 ? 0 : partition, index), bytes,
                           cudaMemcpyDeviceToHost));
        return SSLA_OK;
    });
}

int ssla_engine_write_state(SslaEngine* eng, int kind, int partition, int index, const void* host_src,
                            size_t bytes) {
    if (!state_args_ok(eng, kind, partition, index) || !host_src || kind >= SSLA_STATE_STAGE_OUT) {
        ssla::g_last_error = "bad state selector";
        return SSLA_ERR_ARG;
    }
    return ssla::guarded([&] {
        ssla::Engine& e = eng->e;
        ssla::DeviceGuard dg(e.device);
        const size_t full = e.state_elems(kind, index) * ssla::Engine::elem_size(kind);
        if (bytes > full) throw std::invalid_argument("write larger than the state buffer");
        SSLA_CK(cudaDeviceSynchronize());
        SSLA_CK(cudaMemcpy(e.state_ptr(kind, partition, index), host_src, bytes, cudaMemcpyHostToDevice));
        return SSLA_OK;
    });
}

void* ssla_engine_state_ptr(SslaEngine* eng, int kind, int partition, int index) {
    if (!state_args_ok(eng, kind, partition, index)) return nullptr;
    return eng->e.state_ptr(kind, partition, index);
}

int ssla_engine_info(SslaEngine* eng, SslaEngineInfo* info) {
    if (!eng || !info) { ssla::g_last_error = "null argument"; return SSLA_ERR_ARG; }
    return ssla::guarded([&] {
        ssla::Engine& e = eng->e;
        std::memset(info, 0, sizeof *info);
        info->H = e.g.H[0]; info->W = e.g.W[0]; info->ncls = e.g.ncls; info->tdrop_window = e.g.window;
        info->layout = e.layout; info->n_partitions = e.g.P; info->max_events = e.max_events;
        info->device = e.device;
        ssla::DeviceGuard dg(e.device);
        int cnt[5] = {0};
        SSLA_CK(cudaDeviceSynchronize());
        SSLA_CK(cudaMemcpy(cnt, e.ws.count.p, sizeof cnt, cudaMemcpyDeviceToHost));
        info->stage_events[0] = e.last_n;
        info->launches = e.prof.launches;
        for (int s = 1; s < 5; ++s) info->stage_events[s] = cnt[s];
        return SSLA_OK;
    });
}

int ssla_engine_set_profiling(SslaEngine* eng, int enable) {
    if (!eng) { ssla::g_last_error = "null engine"; return SSLA_ERR_ARG; }
    eng->e.prof.on = enable != 0;
    return SSLA_OK;
}

int ssla_engine_phase_times(SslaEngine* eng, SslaPhaseTime* out, int max_n, int* n_out) {
    if (!eng || !out || !n_out) { ssla::g_last_error = "null argument"; return SSLA_ERR_ARG; }
    return ssla::guarded([&] {
        ssla::Engine& e = eng->e;
        ssla::DeviceGuard dg(e.device);
        ssla::Prof& p = e.prof;
        const int n = std::min<int>(static_cast<int>(p.names.size()), max_n);
        *n_out = 0;
        if (!p.on || p.used < 2) return SSLA_OK;
        SSLA_CK(cudaEventSynchronize(p.ev[p.used - 1]));
        for (int i = 0; i < n; ++i) {
            float ms = 0.0f;
            SSLA_CK(cudaEventElapsedTime(&ms, p.ev[i], p.ev[i + 1]));
            std::memset(out[i].name, 0, sizeof out[i].name);
            std::strncpy(out[i].name, p.names[i].c_str(), sizeof out[i].name - 1);
            out[i].ms = ms;
            out[i].launches = p.nl[i];
        }
        *n_out = n;
        return SSLA_OK;
    });
}

int ssla_measure_fp32_peak(int device, double* tflops_out) {
    if (!tflops_out) { ssla::g_last_error = "null argument"; return SSLA_ERR_ARG; }
    return ssla::guarded([&] {
        ssla::DeviceGuard dg(device);
        *tflops_out = ssla::measure_ffma_peak();
        return SSLA_OK;
    });
}

int ssla_selftest_reciprocal(int device, unsigned long long* mismatches, unsigned* first_bad) {
    if (!mismatches) { ssla::g_last_error = "null argument"; return SSLA_ERR_ARG; }
    return ssla::guarded([&] {
        ssla::DeviceGuard dg(device);
        *mismatches = ssla::check_reciprocal(first_bad);
        return SSLA_OK;
    });
}

int ssla_selftest_sigmoid_pair(int device, unsigned long long* mismatches, unsigned* first_bad) {
    if (!mismatches) { ssla::g_last_error = "null argument"; return SSLA_ERR_ARG; }
    return ssla::guarded([&] {
        ssla::DeviceGuard dg(device);
        *mismatches = ssla::check_sigmoid_pair(first_bad);
        return SSLA_OK;
    });
}

int ssla_s2s3_drain_n_multi(const HybridS2S3Config* cfg, const HybridInputRec* const* rings, const int* ns,
                            HybridS2S3OutputSlot* const* outs, unsigned long long* const* batch_clks,
                            void* stream) {
    if (!cfg || !rings || !ns) { ssla::g_last_error = "null argument"; return SSLA_ERR_ARG; }
    return ssla::guarded([&] {
        return ssla::drain_n_state().run(cfg, rings, ns, outs, batch_clks, static_cast<cudaStream_t>(stream));
    });
}

int ssla_s2s3_drain_n(const HybridS2S3Config* cfg, const HybridInputRec* ring0, const HybridInputRec* ring1,
                      int n0, int n1, HybridS2S3OutputSlot* out0, HybridS2S3OutputSlot* out1,
                      unsigned long long* batch_clk0, unsigned long long* batch_clk1, void* stream) {
    if (!cfg) { ssla::g_last_error = "null argument"; return SSLA_ERR_ARG; }
    // The reference kernel runs exactly two blocks (ssla_s2_s3_head_celled.cuh:927).
    HybridS2S3Config two = *cfg;
    two.n_blocks = 2;
    const HybridInputRec* rings[2] = {ring0, ring1};
    const int ns[2] = {n0, n1};
    HybridS2S3OutputSlot* outs[2] = {out0, out1};
    unsigned long long* clks[2] = {batch_clk0, batch_clk1};
    const bool any_clk = batch_clk0 || batch_clk1;
    return ssla_s2s3_drain_n_multi(&two, rings, ns, (out0 || out1) ? outs : nullptr,
                                   any_clk ? clks : nullptr, stream);
}

}  // extern "C"
