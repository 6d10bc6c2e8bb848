// Paced replay producer for the pinned event rings (SslaLiveRing).
//
// One host thread publishes the events of every stream into its ring when
// they come due on CLOCK_MONOTONIC: event i of ring r (timestamp t_i in
// microseconds) is due at start_ns + t_i * 1000 * time_scale.  A round
// visits every ring, publishes all of its due events that fit (slots
// written first, then head release-stored -- the single-producer side of
// include/spsc.h:9-11 / orin/orin/ring.py:34-152), and yields when nothing
// was published.  Free space comes from tail, which the consumer (the
// ring-drain gather kernel, or a host reader) release-stores after copying
// the slots.  With time_scale 0 every event is due at start_ns: the rings'
// space alone paces the thread, which measures how fast the consumer
// drains.
//
// The reference's synthetic producer (s01g_start_synthetic,
// src/lib_stage01_to_gpu.cpp:637-672) draws random events at a rate inside
// the library; replaying given arrays instead keeps every published event
// checkable against the oracle.
#include <algorithm>
#include <atomic>
#include <cstdint>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include <time.h>

#include "ssla_b200.h"

namespace ssla {
void set_last_error(const std::string& msg);   // ssla_engine.cu
}

struct SslaReplay {
    std::vector<SslaLiveRing> rings;
    std::vector<const float*> ev;
    std::vector<unsigned long long> count;
    double scale = 0.0;
    unsigned long long start_ns = 0;
    std::atomic<bool> stop{false};
    std::thread th;
    SslaReplayStats st{};
};

namespace {

unsigned long long now_ns() {
    timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return static_cast<unsigned long long>(ts.tv_sec) * 1000000000ull + static_cast<unsigned long long>(ts.tv_nsec);
}

void run(SslaReplay* rp) {
    const int n = static_cast<int>(rp->rings.size());
    std::vector<unsigned long long> head(n);
    for (int r = 0; r < n; ++r) head[r] = __atomic_load_n(rp->rings[r].head, __ATOMIC_ACQUIRE);
    std::vector<unsigned long long> pub(n, 0);     // events of stream r published
    std::vector<unsigned long long> due(n, 0);     // events of stream r due so far
    unsigned long long left = 0;
    for (int r = 0; r < n; ++r) left += rp->count[r];
    long long max_lag = 0;
    unsigned long long full_waits = 0;
    while (now_ns() < rp->start_ns && !rp->stop.load(std::memory_order_relaxed)) std::this_thread::yield();
    while (left > 0 && !rp->stop.load(std::memory_order_relaxed)) {
        const unsigned long long now = now_ns();
        // event time (us) that is due now
        const double due_us = rp->scale > 0.0
                                  ? (now >= rp->start_ns ? static_cast<double>(now - rp->start_ns) / (1000.0 * rp->scale) : -1.0)
                                  : 1e300;
        bool any = false;
        for (int r = 0; r < n; ++r) {
            const SslaLiveRing& ring = rp->rings[r];
            const float* ev = rp->ev[r];
            const unsigned long long cnt = rp->count[r];
            const unsigned long long k = pub[r];
            if (k >= cnt) continue;
            unsigned long long e = due[r];
            if (rp->scale > 0.0) {
                while (e < cnt && static_cast<double>(ev[4 * e]) <= due_us) ++e;
            } else {
                e = cnt;
            }
            due[r] = e;
            if (e == k) continue;
            const unsigned long long tail = __atomic_load_n(ring.tail, __ATOMIC_ACQUIRE);
            const unsigned long long space = ring.capacity - (head[r] - tail);
            const unsigned long long m = std::min(e - k, space);
            if (m < e - k) ++full_waits;
            if (m == 0) continue;
            const unsigned long long mask = ring.capacity - 1;
            float* slots = const_cast<float*>(ring.events);
            unsigned long long done = 0;
            while (done < m) {            // at most two pieces (wrap)
                const unsigned long long s = (head[r] + done) & mask;
                const unsigned long long piece = std::min(m - done, ring.capacity - s);
                std::memcpy(slots + 4 * s, ev + 4 * (k + done), sizeof(float) * 4 * piece);
                done += piece;
            }
            head[r] += m;
            __atomic_store_n(ring.head, head[r], __ATOMIC_RELEASE);
            if (rp->scale > 0.0) {
                const double due_at = static_cast<double>(rp->start_ns) + static_cast<double>(ev[4 * k]) * 1000.0 * rp->scale;
                const long long lag = static_cast<long long>(static_cast<double>(now) - due_at);
                max_lag = std::max(max_lag, lag);
            }
            pub[r] = k + m;
            left -= m;
            any = true;
        }
        if (!any) std::this_thread::yield();
    }
    unsigned long long total = 0;
    for (int r = 0; r < n; ++r) total += pub[r];
    rp->st.published = total;
    rp->st.start_ns = rp->start_ns;
    rp->st.max_lag_ns = max_lag;
    rp->st.full_waits = full_waits;
}

}  // namespace

extern "C" {

SslaReplay* ssla_replay_start(const SslaLiveRing* rings, int n_rings, const float* const* events,
                              const unsigned long long* counts, double time_scale, unsigned long long start_ns) {
    if (!rings || !events || !counts || n_rings < 1 || time_scale < 0.0) {
        ssla::set_last_error("replay: bad argument");
        return nullptr;
    }
    for (int r = 0; r < n_rings; ++r) {
        const SslaLiveRing& g = rings[r];
        if (!g.events || !g.head || !g.tail || g.capacity < 2 || (g.capacity & (g.capacity - 1)) ||
            (counts[r] > 0 && !events[r])) {
            ssla::set_last_error("replay: ring " + std::to_string(r) +
                                 " needs events, head, tail and a power-of-two capacity");
            return nullptr;
        }
    }
    auto* rp = new SslaReplay();
    rp->rings.assign(rings, rings + n_rings);
    rp->ev.assign(events, events + n_rings);
    rp->count.assign(counts, counts + n_rings);
    rp->scale = time_scale;
    rp->start_ns = start_ns ? start_ns : now_ns() + 2000000ull;
    rp->th = std::thread(run, rp);
    return rp;
}

void ssla_replay_stop(SslaReplay* rp) {
    if (rp) rp->stop.store(true, std::memory_order_relaxed);
}

int ssla_replay_join(SslaReplay* rp, SslaReplayStats* stats) {
    if (!rp) {
        ssla::set_last_error("replay: null handle");
        return SSLA_ERR_ARG;
    }
    if (rp->th.joinable()) rp->th.join();
    if (stats) *stats = rp->st;
    delete rp;
    return SSLA_OK;
}

}  // extern "C"
