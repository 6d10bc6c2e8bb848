// ref_driver.cpp -- TEST INFRASTRUCTURE ONLY.
//
// A C API over the reference's own deploy::SslaSPipeline (built from the
// reference sources by oracle/Makefile into oracle/_ref/libssla_ref.so).
// It drives the pipeline with the reference's public methods only, in the
// two orders the reference uses:
//   layout 0 (decomp): src/legacy/schemes/s2_decomp_st.cpp:138-176
//   layout 1 (hybrid): src/lib_stage01_to_gpu.cpp:210-311 for an owner event
//       (A1 tdrop-before-stage + state-only stage), then the GPU chain of
//       orin/kernels/ssla_s2_s3_head_celled.cuh:1679-1755: tdrop_s2 on the
//       s2 grid gates stage 3, tdrop_s3 on the s3 grid gates the head.  The
//       pipeline has no counter for tdrop_s2 (its three counters are the s1,
//       s2 and s3 grids); the driver keeps that one, with the same uint8 rule
//       (ssla_s2_s3_head_celled.cuh:742-745).  tdrop_s3 reuses the pipeline's
//       s3-grid counter, which the hybrid chain otherwise leaves unused.
// It is the reference arm of bench.py and a pin for the C restatement.

#include <chrono>
#include <cstdint>
#include <cstring>
#include <exception>
#include <memory>
#include <thread>
#include <vector>

#include "oracle.h"
#include "ssla_kernels.h"

namespace {

struct RefHandle {
    deploy::SslaSPipeline pipe;
    std::vector<std::uint8_t> s2_gate;   // GPU tdrop_s2 counter (hybrid)
};

bool own_gate(RefHandle* h, int idx) {
    const std::uint8_t pre = h->s2_gate[idx];
    h->s2_gate[idx] = static_cast<std::uint8_t>(pre + 1u);
    const int w = h->pipe.tdrop_window();
    if (w <= 1) return true;
    return (pre % w) == 0u;
}

enum { F_VALID = 1, F_R1 = 2, F_R2 = 4, F_R3 = 8, F_R4 = 16 };

void run_one(RefHandle* h, int layout, const float* e4, std::uint8_t* flag,
             float* so0, float* so1, float* so2, float* so3) {
    deploy::SslaSPipeline& pipe = h->pipe;
    openeva::Event e{e4[0], e4[1], e4[2], e4[3]};
    const int ex0 = static_cast<int>(e.x);
    const int ey0 = static_cast<int>(e.y);
    std::uint8_t f = 0;
    if (ex0 < 0 || ex0 >= pipe.W() || ey0 < 0 || ey0 >= pipe.H()) {
        if (flag) *flag = 0;
        return;
    }
    f |= F_VALID;
    float feat_in[deploy::kInDim];
    float f0[deploy::kC0], f1[deploy::kC1], f2[deploy::kC2], f3[deploy::kC3];
    pipe.preprocess(e, feat_in);
    int x = ex0, y = ey0;
    if (layout == 0) {
        pipe.stage_forward(0, x, y, feat_in, f0);
        if (!pipe.tdrop_and_pool(0, x, y)) { if (flag) *flag = f; return; }
        f |= F_R1;
        if (so0) std::memcpy(so0, f0, sizeof f0);
        pipe.stage_forward(1, x, y, f0, f1);
        if (!pipe.tdrop_and_pool(1, x, y)) { if (flag) *flag = f; return; }
        f |= F_R2;
        if (so1) std::memcpy(so1, f1, sizeof f1);
        pipe.stage_forward(2, x, y, f1, f2);
        if (!pipe.tdrop_and_pool(2, x, y)) { if (flag) *flag = f; return; }
        f |= F_R3;
        if (so2) std::memcpy(so2, f2, sizeof f2);
        pipe.stage_forward(3, x, y, f2, f3);
        f |= F_R4;
        if (so3) std::memcpy(so3, f3, sizeof f3);
        pipe.head_decode_cell(3, x, y, f3);
        if (flag) *flag = f;
        return;
    }
    // hybrid
    const int x1 = x / 2, y1 = y / 2;
    const bool pass0 = pipe.tdrop_check_at(0, x1, y1);
    if (pass0) pipe.stage_forward(0, x, y, feat_in, f0);
    else       pipe.stage_forward_state_only(0, x, y, feat_in);
    if (!pass0) { if (flag) *flag = f; return; }
    f |= F_R1;
    if (so0) std::memcpy(so0, f0, sizeof f0);
    const int x2 = x1 / 2, y2 = y1 / 2;
    const bool pass1 = pipe.tdrop_check_at(1, x2, y2);
    if (pass1) pipe.stage_forward(1, x1, y1, f0, f1);
    else       pipe.stage_forward_state_only(1, x1, y1, f0);
    if (!pass1) { if (flag) *flag = f; return; }
    f |= F_R2;
    if (so1) std::memcpy(so1, f1, sizeof f1);
    const int W2 = pipe.W() / 4;
    const bool pass2 = own_gate(h, y2 * W2 + x2);
    pipe.stage_forward(2, x2, y2, f1, f2);
    if (!pass2) { if (flag) *flag = f; return; }
    f |= F_R3;
    if (so2) std::memcpy(so2, f2, sizeof f2);
    const int x3 = x2 / 2, y3 = y2 / 2;
    const bool pass3 = pipe.tdrop_check_at(2, x3, y3);
    pipe.stage_forward(3, x3, y3, f2, f3);
    if (pass3) {
        f |= F_R4;
        if (so3) std::memcpy(so3, f3, sizeof f3);
        pipe.head_decode_cell(3, x3, y3, f3);
    }
    if (flag) *flag = f;
}

}  // namespace

extern "C" {

void* ref_create(const char* weights_dir) {
    auto h = std::make_unique<RefHandle>();
    try {
        h->pipe.load(weights_dir);
    } catch (const std::exception&) {
        return nullptr;
    }
    h->pipe.reset();
    h->s2_gate.assign(static_cast<std::size_t>(h->pipe.H() / 4) * (h->pipe.W() / 4), 0);
    return h.release();
}

void ref_destroy(void* p) { delete static_cast<RefHandle*>(p); }

void ref_reset(void* p) {
    auto* h = static_cast<RefHandle*>(p);
    h->pipe.reset();
    std::fill(h->s2_gate.begin(), h->s2_gate.end(), 0);
}

int ref_num_anchors(void* p) { return static_cast<RefHandle*>(p)->pipe.num_anchors_total(); }
int ref_cols(void* p) { return static_cast<RefHandle*>(p)->pipe.cols(); }

// The reference's own OracleRecorder over a run of the n events: after
// event i it records pipe.last_output() (record keeps i % every == 0), the
// way src/legacy/schemes/s2_decomp_st.cpp:195-207 drives it; then save().
int ref_oracle_dump(void* p, int layout, const float* ev, int n, int every, const char* path) {
    auto* h = static_cast<RefHandle*>(p);
    try {
        deploy::OracleRecorder rec(h->pipe.num_anchors_total(), h->pipe.cols(), static_cast<std::size_t>(every),
                                   path);
        for (int i = 0; i < n; ++i) {
            run_one(h, layout, ev + 4 * static_cast<std::size_t>(i), nullptr, nullptr, nullptr, nullptr, nullptr);
            rec.record(static_cast<std::uint64_t>(i), h->pipe.last_output());
        }
        rec.save();
        return static_cast<int>(rec.num_checkpoints());
    } catch (const std::exception&) {
        return -1;
    }
}

// The reference's diff_dumps (include/oracle.h:100-151).
int ref_diff_dumps(const char* a, const char* b, double tol, double* max_abs, int* n_cp, int* n_mismatched) {
    try {
        const deploy::DiffReport r = deploy::diff_dumps(a, b, tol);
        *max_abs = r.max_abs_delta;
        *n_cp = static_cast<int>(r.n_cp);
        *n_mismatched = static_cast<int>(r.n_mismatched_cp);
        return r.ok ? 1 : 0;
    } catch (const std::exception&) {
        return -1;
    }
}

void ref_run_events(void* p, int layout, const float* ev, int n, std::uint8_t* flags,
                    float* so0, float* so1, float* so2, float* so3) {
    auto* h = static_cast<RefHandle*>(p);
    for (int i = 0; i < n; ++i) {
        run_one(h, layout, ev + 4 * static_cast<std::size_t>(i),
                flags ? flags + i : nullptr,
                so0 ? so0 + static_cast<std::size_t>(i) * deploy::kC0 : nullptr,
                so1 ? so1 + static_cast<std::size_t>(i) * deploy::kC1 : nullptr,
                so2 ? so2 + static_cast<std::size_t>(i) * deploy::kC2 : nullptr,
                so3 ? so3 + static_cast<std::size_t>(i) * deploy::kC3 : nullptr);
    }
}

// drain_n records for one block (ssla_s2_s3_head_celled.cuh:986-1094): uses the
// pipeline's s2-grid counter as tdrop_s2 and its s3-grid counter as tdrop_s3,
// and single layer_forward calls so the L4 / L6 outputs left in the slot by
// the reference kernel can be reproduced.
void ref_run_s2_records(void* p, const int* x2, const int* y2, const float* feat1,
                        const int* owner, int n, int* pass2, int* pass3, float* s3_feat) {
    auto* h = static_cast<RefHandle*>(p);
    deploy::SslaSPipeline& pipe = h->pipe;
    float l4[deploy::kC2], l5[deploy::kC2], l6[deploy::kC3], l7[deploy::kC3];
    for (int i = 0; i < n; ++i) {
        const int x = x2[i], y = y2[i];
        const bool p2 = pipe.tdrop_check_at(1, x, y);
        pipe.layer_forward(4, x, y, feat1 + static_cast<std::size_t>(i) * deploy::kC1, l4);
        pipe.layer_forward(5, x, y, l4, l5);
        bool p3 = false;
        if (p2) {
            p3 = pipe.tdrop_check_at(2, x / 2, y / 2);
            pipe.layer_forward(6, x / 2, y / 2, l5, l6);
            pipe.layer_forward(7, x / 2, y / 2, l6, l7);
        }
        pass2[i] = owner[i] ? (p2 ? 1 : 0) : -1;
        pass3[i] = owner[i] ? ((p2 && p3) ? 1 : 0) : -1;
        float* slot = s3_feat + static_cast<std::size_t>(i) * deploy::kC3;
        if (p3) std::memcpy(slot, l7, sizeof l7);
        else if (p2) std::memcpy(slot, l6, sizeof l6);
        else {
            std::memcpy(slot, l4, sizeof l4);
            std::memset(slot + deploy::kC2, 0, sizeof(float) * deploy::kC2);
        }
    }
}

void ref_get_hidden(void* p, int layer, float* out) {
    auto* h = static_cast<RefHandle*>(p);
    const int stage = layer / 2;
    const int C = (stage == 0) ? deploy::kC0 : (stage == 1) ? deploy::kC1
                : (stage == 2) ? deploy::kC2 : deploy::kC3;
    const std::size_t n = static_cast<std::size_t>(h->pipe.bench_Hl(stage)) *
                          h->pipe.bench_Wl(stage) * C;
    std::memcpy(out, h->pipe.bench_hidden(layer), n * sizeof(float));
}

void ref_get_predictions(void* p, float* out) {
    auto* h = static_cast<RefHandle*>(p);
    const auto& v = h->pipe.predictions();
    std::memcpy(out, v.data(), v.size() * sizeof(float));
}

// CPU baseline: n_streams independent pipelines (one per thread, up to
// n_threads at a time), each fed its own event slice; returns wall seconds
// of the run phase.  Streams are independent reference instances, the way
// the reference's own throughput harness splits events across independent
// blocks (orin/perf_celled_multi.py:179-190).
double ref_time_streams(const char* weights_dir, int layout, int n_streams,
                        const float* const* ev, const int* n_ev, int n_threads) {
    std::vector<std::unique_ptr<RefHandle>> hs;
    for (int s = 0; s < n_streams; ++s) {
        auto* raw = static_cast<RefHandle*>(ref_create(weights_dir));
        if (!raw) return -1.0;
        hs.emplace_back(raw);
    }
    if (n_threads < 1) n_threads = 1;
    const auto t0 = std::chrono::steady_clock::now();
    for (int s0 = 0; s0 < n_streams; s0 += n_threads) {
        std::vector<std::thread> th;
        for (int s = s0; s < n_streams && s < s0 + n_threads; ++s) {
            th.emplace_back([&, s]() {
                ref_run_events(hs[s].get(), layout, ev[s], n_ev[s], nullptr,
                               nullptr, nullptr, nullptr, nullptr);
            });
        }
        for (auto& t : th) t.join();
    }
    const auto t1 = std::chrono::steady_clock::now();
    return std::chrono::duration<double>(t1 - t0).count();
}

}  // extern "C"
