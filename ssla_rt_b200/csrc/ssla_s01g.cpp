// libstage01_to_gpu.so ABI (s01g_*) on the GPU engine.
//
// Events enter a single-producer queue (s01g_submit_batch or the synthetic
// producer thread).  One worker thread takes whatever is queued (up to one
// engine batch), runs stages 0-1 with gates 0-1 on the GPU
// (ssla_engine_drain_records) and publishes every returned record into the
// attached rings with the reference's protocol: claim a slot with an atomic
// fetch-add on the ring head, write the record, release-store seq_done =
// slot + 1 (src/lib_stage01_to_gpu.cpp:262-300).
#include "stage01_to_gpu.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#if defined(__linux__)
#include <pthread.h>
#include <sched.h>
#include <time.h>
#endif

#include "ssla_abi_types.h"
#include "ssla_b200.h"

namespace {

constexpr int kMaxRings = SSLA_MAX_BLOCKS;
constexpr int kBatch = 65536;            // events per GPU batch (engine capacity)

std::uint64_t mono_raw_ns() {
#if defined(__linux__)
    timespec ts;
    clock_gettime(CLOCK_MONOTONIC_RAW, &ts);
    return static_cast<std::uint64_t>(ts.tv_sec) * 1000000000ull + static_cast<std::uint64_t>(ts.tv_nsec);
#else
    return 0;
#endif
}

void pin_to_core(int core) {
#if defined(__linux__)
    if (core < 0) return;
    cpu_set_t cs;
    CPU_ZERO(&cs);
    CPU_SET(core, &cs);
    pthread_setaffinity_np(pthread_self(), sizeof(cs), &cs);
#else
    (void)core;
#endif
}

void cpu_relax() {
#if defined(__x86_64__)
    __builtin_ia32_pause();
#elif defined(__aarch64__)
    asm volatile("yield" ::: "memory");
#endif
}

struct QEvent {
    float t, x, y, p;
    std::uint64_t t_emit_ns;
};

struct Ring {
    HybridInputRec* buf = nullptr;
    std::uint64_t* head = nullptr;
    int x_lo = 0, x_hi = 0, y_lo = 0, y_hi = 0;
    std::atomic<std::uint64_t> n_pushed{0};
};

enum Seg { SEG_PRE = 0, SEG_S0, SEG_TD0, SEG_S1, SEG_TD1, SEG_PUSH, NUM_SEGS };

}  // namespace

struct S01gHandle {
    int device = 0;
    SslaEngine* eng = nullptr;
    int W = 0, H = 0, n_shards = 1, halo = 0;
    // input queue (single producer, the worker consumes)
    std::vector<QEvent> q;
    std::uint64_t q_mask = 0;
    alignas(64) std::atomic<std::uint64_t> q_head{0};
    alignas(64) std::atomic<std::uint64_t> q_tail{0};
    // GPU-side batch buffers
    cudaStream_t st = nullptr;
    float* d_ev = nullptr;
    float* h_ev = nullptr;              // pinned
    HybridInputRec* d_rec = nullptr;
    HybridInputRec* h_rec = nullptr;    // pinned
    std::uint8_t* d_flags = nullptr;
    std::uint8_t* h_flags = nullptr;    // pinned
    std::vector<std::uint64_t> emit_ns;
    // rings
    std::atomic<bool> attached{false};
    Ring rings[kMaxRings];
    int n_rings = 0;
    std::uint64_t ring_mask = 0;
    int W2 = 0, H2 = 0;
    // worker
    std::thread worker;
    std::atomic<bool> stop{false};
    std::atomic<std::uint64_t> n_done{0};     // events fully processed
    std::atomic<int> failed{0};
    // statistics
    std::atomic<std::uint64_t> total{0}, pass0{0}, pass1{0}, n_oob{0};
    std::atomic<std::uint64_t> seg_ns[NUM_SEGS]{}, seg_cnt[NUM_SEGS]{};
    std::mutex lat_mu;
    std::vector<double> lat_us;
    std::size_t lat_cap = 1024, lat_idx = 0;
    std::chrono::steady_clock::time_point t0;
    // synthetic producer
    std::atomic<bool> synth_running{false};
    std::thread synth;
    std::atomic<std::uint64_t> synth_n{0};
};

namespace {

// Single-producer enqueue; spins while the queue is full.
void enqueue(S01gHandle* h, const QEvent& e) {
    const std::uint64_t hd = h->q_head.load(std::memory_order_relaxed);
    while (hd - h->q_tail.load(std::memory_order_acquire) > h->q_mask) {
        if (h->failed.load(std::memory_order_relaxed)) return;
        cpu_relax();
    }
    h->q[hd & h->q_mask] = e;
    h->q_head.store(hd + 1, std::memory_order_release);
}

void publish(S01gHandle* h, const HybridInputRec& r, std::uint64_t t_emit) {
    const int sx = r.x, sy = r.y;
    if (sx < 0 || sx >= h->W2 || sy < 0 || sy >= h->H2) return;
    for (int b = 0; b < h->n_rings; ++b) {
        Ring& g = h->rings[b];
        if (sx < g.x_lo || sx >= g.x_hi || sy < g.y_lo || sy >= g.y_hi) continue;
        const std::uint64_t slot = __atomic_fetch_add(g.head, 1ull, __ATOMIC_RELAXED);
        HybridInputRec* dst = g.buf + (slot & h->ring_mask);
        dst->t = r.t;
        dst->x = r.x;
        dst->y = r.y;
        std::memcpy(dst->feat1, r.feat1, sizeof(r.feat1));
        dst->t_push_ns = mono_raw_ns();
        dst->t_emit_ns = t_emit;
        __atomic_store_n(&dst->seq_done, slot + 1ull, __ATOMIC_RELEASE);
        g.n_pushed.fetch_add(1, std::memory_order_relaxed);
    }
}

void worker_main(S01gHandle* h) {
    cudaSetDevice(h->device);
    for (;;) {
        const std::uint64_t tail = h->q_tail.load(std::memory_order_relaxed);
        const std::uint64_t head = h->q_head.load(std::memory_order_acquire);
        if (head == tail) {
            if (h->stop.load(std::memory_order_acquire) &&
                h->q_head.load(std::memory_order_acquire) == tail)
                break;
            std::this_thread::yield();
            continue;
        }
        const int n = static_cast<int>(std::min<std::uint64_t>(head - tail, kBatch));
        for (int i = 0; i < n; ++i) {
            const QEvent& e = h->q[(tail + i) & h->q_mask];
            h->h_ev[4 * i + 0] = e.t;
            h->h_ev[4 * i + 1] = e.x;
            h->h_ev[4 * i + 2] = e.y;
            h->h_ev[4 * i + 3] = e.p;
            h->emit_ns[i] = e.t_emit_ns;
        }
        h->q_tail.store(tail + n, std::memory_order_release);
        const std::uint64_t g0 = mono_raw_ns();
        int rec_off[2] = {0, 0};
        const int off[2] = {0, n};
        bool ok = cudaMemcpyAsync(h->d_ev, h->h_ev, sizeof(float) * 4 * n, cudaMemcpyHostToDevice, h->st) ==
                  cudaSuccess;
        ok = ok && ssla_engine_drain_records(h->eng, h->d_ev, off, h->d_rec, kBatch, rec_off, h->d_flags,
                                             h->st) == SSLA_OK;
        const int nr = ok ? rec_off[1] : 0;
        if (ok && nr > 0)
            ok = cudaMemcpyAsync(h->h_rec, h->d_rec, sizeof(HybridInputRec) * nr, cudaMemcpyDeviceToHost,
                                 h->st) == cudaSuccess;
        ok = ok && cudaMemcpyAsync(h->h_flags, h->d_flags, n, cudaMemcpyDeviceToHost, h->st) == cudaSuccess;
        ok = ok && cudaStreamSynchronize(h->st) == cudaSuccess;
        if (!ok) {
            std::fprintf(stderr, "[s01g] GPU batch failed: %s\n", ssla_last_error());
            h->failed.store(1, std::memory_order_release);
            h->n_done.fetch_add(n, std::memory_order_release);
            continue;
        }
        const std::uint64_t g1 = mono_raw_ns();
        // records follow the events that passed gate 1, in stream order
        std::uint64_t p0 = 0, p1 = 0;
        int k = 0;
        const bool attached = h->attached.load(std::memory_order_acquire);
        for (int i = 0; i < n; ++i) {
            const std::uint8_t f = h->h_flags[i];
            p0 += (f & SSLA_F_R1) ? 1 : 0;
            if (f & SSLA_F_R2) {
                ++p1;
                if (attached && k < nr) publish(h, h->h_rec[k], h->emit_ns[i]);
                ++k;
            }
        }
        const std::uint64_t g2 = mono_raw_ns();
        {
            std::lock_guard<std::mutex> lk(h->lat_mu);
            for (int i = 0; i < n; ++i) {
                h->lat_us[h->lat_idx % h->lat_cap] = static_cast<double>(g2 - h->emit_ns[i]) * 1e-3;
                ++h->lat_idx;
            }
        }
        h->total.fetch_add(n, std::memory_order_relaxed);
        h->pass0.fetch_add(p0, std::memory_order_relaxed);
        h->pass1.fetch_add(p1, std::memory_order_relaxed);
        h->seg_ns[SEG_S0].fetch_add(g1 - g0, std::memory_order_relaxed);
        h->seg_cnt[SEG_S0].fetch_add(n, std::memory_order_relaxed);
        h->seg_ns[SEG_PUSH].fetch_add(g2 - g1, std::memory_order_relaxed);
        h->seg_cnt[SEG_PUSH].fetch_add(p1, std::memory_order_relaxed);
        h->n_done.fetch_add(n, std::memory_order_release);
    }
}

void synth_main(S01gHandle* h, double rate_mev, int pin_core, std::uint64_t seed) {
    pin_to_core(pin_core);
    std::uint64_t state = seed ? seed : 0x9E3779B97F4A7C15ull;
    const double ns_per_event = rate_mev > 0.0 ? 1e3 / rate_mev : 0.0;
    const float dt_us = rate_mev > 0.0 ? static_cast<float>(1.0 / rate_mev) : 1.0f;
    float t_us = 0.0f;
    const std::uint64_t start = mono_raw_ns();
    std::uint64_t i = 0;
    while (h->synth_running.load(std::memory_order_relaxed)) {
        if (ns_per_event > 0.0) {
            const std::uint64_t due = start + static_cast<std::uint64_t>(ns_per_event * static_cast<double>(i));
            while (mono_raw_ns() < due) {
                if (!h->synth_running.load(std::memory_order_relaxed)) return;
                cpu_relax();
            }
        }
        state ^= state << 13;
        state ^= state >> 7;
        state ^= state << 17;
        const std::uint64_t r = state;
        QEvent e;
        e.x = static_cast<float>(static_cast<int>(r % static_cast<std::uint64_t>(h->W)));
        e.y = static_cast<float>(static_cast<int>((r >> 16) % static_cast<std::uint64_t>(h->H)));
        e.p = static_cast<float>((r >> 32) & 1ull);
        t_us += dt_us;
        e.t = t_us;
        e.t_emit_ns = mono_raw_ns();
        enqueue(h, e);
        h->synth_n.fetch_add(1, std::memory_order_relaxed);
        ++i;
    }
}

void release(S01gHandle* h) {
    if (h->d_ev) cudaFree(h->d_ev);
    if (h->d_rec) cudaFree(h->d_rec);
    if (h->d_flags) cudaFree(h->d_flags);
    if (h->h_ev) cudaFreeHost(h->h_ev);
    if (h->h_rec) cudaFreeHost(h->h_rec);
    if (h->h_flags) cudaFreeHost(h->h_flags);
    if (h->st) cudaStreamDestroy(h->st);
    if (h->eng) ssla_engine_destroy(h->eng);
    delete h;
}

}  // namespace

extern "C" {

S01gHandle* s01g_init_full(const char* weights_dir, int n_shards, int halo, int base_core, int sample_cap,
                           unsigned int shard_ring_cap) {
    (void)base_core;
    if (!weights_dir) return nullptr;
    if (n_shards < 1) n_shards = 1;
    if (sample_cap < 1024) sample_cap = 1024;
    if (shard_ring_cap < 4) shard_ring_cap = 4;
    std::uint64_t cap = 1;
    while (cap < static_cast<std::uint64_t>(shard_ring_cap) * static_cast<std::uint64_t>(n_shards)) cap <<= 1;
    auto* h = new S01gHandle();
    if (cudaGetDevice(&h->device) != cudaSuccess) { delete h; return nullptr; }
    SslaEngineConfig cfg{1, kBatch, SSLA_LAYOUT_HYBRID, h->device, 0, kBatch};
    if (ssla_engine_create(weights_dir, &cfg, &h->eng) != SSLA_OK) {
        std::fprintf(stderr, "[s01g_init] %s\n", ssla_last_error());
        h->eng = nullptr;
        release(h);
        return nullptr;
    }
    SslaEngineInfo info{};
    ssla_engine_info(h->eng, &info);
    h->W = info.W;
    h->H = info.H;
    h->n_shards = n_shards;
    h->halo = halo;
    h->q.resize(cap);
    h->q_mask = cap - 1;
    h->emit_ns.resize(kBatch);
    h->lat_cap = static_cast<std::size_t>(sample_cap);
    h->lat_us.assign(h->lat_cap, 0.0);
    bool ok = cudaStreamCreateWithFlags(&h->st, cudaStreamNonBlocking) == cudaSuccess;
    ok = ok && cudaMalloc(&h->d_ev, sizeof(float) * 4 * kBatch) == cudaSuccess;
    ok = ok && cudaMalloc(&h->d_rec, sizeof(HybridInputRec) * kBatch) == cudaSuccess;
    ok = ok && cudaMalloc(&h->d_flags, kBatch) == cudaSuccess;
    ok = ok && cudaMallocHost(&h->h_ev, sizeof(float) * 4 * kBatch) == cudaSuccess;
    ok = ok && cudaMallocHost(&h->h_rec, sizeof(HybridInputRec) * kBatch) == cudaSuccess;
    ok = ok && cudaMallocHost(&h->h_flags, kBatch) == cudaSuccess;
    if (!ok) {
        std::fprintf(stderr, "[s01g_init] CUDA allocation failed\n");
        release(h);
        return nullptr;
    }
    h->t0 = std::chrono::steady_clock::now();
    h->worker = std::thread(worker_main, h);
    return h;
}

S01gHandle* s01g_init(const char* weights_dir, int n_shards, int halo, int base_core, int sample_cap) {
    return s01g_init_full(weights_dir, n_shards, halo, base_core, sample_cap, 1u << 16);
}

void s01g_attach_gpu_rings_multi(S01gHandle* h, int n_blocks, void* const* ring_bufs, void* const* ring_heads,
                                 unsigned long long ring_mask, int W2, int H2, const int* proc_x_los,
                                 const int* proc_x_his, const int* proc_y_los, const int* proc_y_his) {
    if (!h || n_blocks <= 0 || n_blocks > kMaxRings || !ring_bufs || !ring_heads) return;
    h->attached.store(false, std::memory_order_release);
    for (int b = 0; b < n_blocks; ++b) {
        Ring& r = h->rings[b];
        r.buf = static_cast<HybridInputRec*>(ring_bufs[b]);
        r.head = static_cast<std::uint64_t*>(ring_heads[b]);
        r.x_lo = proc_x_los[b];
        r.x_hi = proc_x_his[b];
        r.y_lo = proc_y_los[b];
        r.y_hi = proc_y_his[b];
        r.n_pushed.store(0, std::memory_order_relaxed);
    }
    h->n_rings = n_blocks;
    h->ring_mask = ring_mask;
    h->W2 = W2;
    h->H2 = H2;
    std::atomic_thread_fence(std::memory_order_release);
    h->attached.store(true, std::memory_order_release);
}

void s01g_attach_gpu_rings(S01gHandle* h, void* ring_buf_0, void* ring_head_0, void* ring_buf_1,
                           void* ring_head_1, unsigned long long ring_mask, int W2, int H2, int proc_lo_0,
                           int proc_hi_0, int proc_lo_1, int proc_hi_1) {
    void* bufs[2] = {ring_buf_0, ring_buf_1};
    void* heads[2] = {ring_head_0, ring_head_1};
    const int xlo[2] = {proc_lo_0, proc_lo_1}, xhi[2] = {proc_hi_0, proc_hi_1};
    const int ylo[2] = {0, 0}, yhi[2] = {H2, H2};
    s01g_attach_gpu_rings_multi(h, 2, bufs, heads, ring_mask, W2, H2, xlo, xhi, ylo, yhi);
}

int s01g_submit_batch(S01gHandle* h, const float* events_packed, int n) {
    if (!h || !events_packed || n <= 0) return 0;
    int accepted = 0;
    for (int i = 0; i < n; ++i) {
        const float* e = events_packed + 4 * i;
        const int ex = static_cast<int>(e[1]), ey = static_cast<int>(e[2]);
        if (ex < 0 || ex >= h->W || ey < 0 || ey >= h->H) {
            h->n_oob.fetch_add(1, std::memory_order_relaxed);
            continue;
        }
        enqueue(h, QEvent{e[0], e[1], e[2], e[3], mono_raw_ns()});
        ++accepted;
    }
    return accepted;
}

void s01g_snapshot_stats(S01gHandle* h, double* out) {
    if (!out) return;
    for (int i = 0; i < 32; ++i) out[i] = 0.0;
    if (!h) return;
    out[0] = static_cast<double>(h->total.load(std::memory_order_relaxed));
    out[1] = 0.0;
    out[2] = static_cast<double>(h->pass0.load(std::memory_order_relaxed));
    out[3] = static_cast<double>(h->n_oob.load(std::memory_order_relaxed));
    out[4] = std::chrono::duration<double>(std::chrono::steady_clock::now() - h->t0).count();
    out[5] = static_cast<double>(h->q_head.load(std::memory_order_relaxed) -
                                 h->n_done.load(std::memory_order_relaxed));
    {
        std::lock_guard<std::mutex> lk(h->lat_mu);
        const std::size_t m = std::min(h->lat_idx, h->lat_cap);
        if (m > 0) {
            std::vector<double> v(h->lat_us.begin(), h->lat_us.begin() + static_cast<std::ptrdiff_t>(m));
            std::sort(v.begin(), v.end());
            auto pct = [&](double q) {
                const std::size_t k = static_cast<std::size_t>(std::ceil(q * static_cast<double>(m))) - 1;
                return v[std::min(k, m - 1)];
            };
            double sum = 0.0;
            for (double x : v) sum += x;
            out[6] = pct(0.50);
            out[7] = pct(0.90);
            out[8] = pct(0.99);
            out[9] = pct(0.999);
            out[10] = v.back();
            out[11] = sum / static_cast<double>(m);
            out[12] = static_cast<double>(m);
        }
    }
    out[13] = static_cast<double>(h->pass1.load(std::memory_order_relaxed));
    out[14] = static_cast<double>(h->rings[0].n_pushed.load(std::memory_order_relaxed));
    out[15] = static_cast<double>(h->rings[1].n_pushed.load(std::memory_order_relaxed));
    for (int s = 0; s < NUM_SEGS; ++s) {
        out[16 + s] = static_cast<double>(h->seg_ns[s].load(std::memory_order_relaxed));
        out[22 + s] = static_cast<double>(h->seg_cnt[s].load(std::memory_order_relaxed));
    }
}

void s01g_reset_stats(S01gHandle* h) {
    if (!h) return;
    h->total.store(0);
    h->pass0.store(0);
    h->pass1.store(0);
    h->n_oob.store(0);
    for (int s = 0; s < NUM_SEGS; ++s) {
        h->seg_ns[s].store(0);
        h->seg_cnt[s].store(0);
    }
    for (auto& r : h->rings) r.n_pushed.store(0);
    {
        std::lock_guard<std::mutex> lk(h->lat_mu);
        h->lat_idx = 0;
    }
    h->t0 = std::chrono::steady_clock::now();
}

void s01g_start_synthetic(S01gHandle* h, double rate_mev, int pin_core, std::uint64_t seed) {
    if (!h || h->synth_running.load()) return;
    h->synth_running.store(true, std::memory_order_release);
    h->synth_n.store(0, std::memory_order_relaxed);
    h->synth = std::thread(synth_main, h, rate_mev, pin_core, seed);
}

void s01g_stop_synthetic(S01gHandle* h) {
    if (!h) return;
    h->synth_running.store(false, std::memory_order_release);
    if (h->synth.joinable()) h->synth.join();
}

std::uint64_t s01g_synthetic_n_pushed(S01gHandle* h) {
    return h ? h->synth_n.load(std::memory_order_relaxed) : 0;
}

int s01g_flush(S01gHandle* h, double timeout_s) {
    if (!h) return -1;
    const std::uint64_t target = h->q_head.load(std::memory_order_acquire);
    const auto t_end = std::chrono::steady_clock::now() + std::chrono::duration<double>(timeout_s);
    while (h->n_done.load(std::memory_order_acquire) < target) {
        if (std::chrono::steady_clock::now() > t_end) return -1;
        std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
    return h->failed.load() ? -1 : 0;
}

void s01g_shutdown(S01gHandle* h) {
    if (!h) return;
    s01g_stop_synthetic(h);
    h->stop.store(true, std::memory_order_release);
    if (h->worker.joinable()) h->worker.join();
    release(h);
}

}  // extern "C"
