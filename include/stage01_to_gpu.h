/* stage01_to_gpu.h -- the libstage01_to_gpu.so C ABI (s01g_*), served by
 * libssla_b200.so (also built under the name libstage01_to_gpu.so).
 *
 * Same entry points, argument meaning and ring protocol as the reference
 * library (src/lib_stage01_to_gpu.cpp:341-755, ctypes signatures in
 * orin/orin/hybrid_common.py:470-602): events go in through
 * s01g_submit_batch or the synthetic producer; stages 0-1 and the two CPU
 * tdrop gates run; every event that passes gate 1 is published as a
 * HybridInputRec into each attached GPU ring whose stage-2 range covers it
 * (slot = atomic fetch-add of the ring head, record fields written, then a
 * release-store of seq_done = slot + 1).
 *
 * What differs: stages 0-1 run on the GPU as one exact event stream (the
 * sequential SslaSPipeline semantics), not on n_shards CPU threads that
 * each see only their strip plus the halo; n_shards, halo and base_core
 * are accepted and only shape the statistics.  Records are produced in
 * batches by one worker thread, so a record is published some
 * microseconds after its event is submitted.  Handles are opaque; every
 * call on a NULL handle returns without effect.  s01g_submit_batch and the
 * synthetic producer must not run at the same time (single producer).
 */
#ifndef STAGE01_TO_GPU_H
#define STAGE01_TO_GPU_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct S01gHandle S01gHandle;

/* src/lib_stage01_to_gpu.cpp:345-348.  NULL on a load failure or when no
 * CUDA device is present. */
S01gHandle* s01g_init(const char* weights_dir, int n_shards, int halo,
                      int base_core, int sample_cap);
/* src/lib_stage01_to_gpu.cpp:350-421; shard_ring_cap sizes the input
 * queue (rounded up to a power of two). */
S01gHandle* s01g_init_full(const char* weights_dir, int n_shards, int halo,
                           int base_core, int sample_cap,
                           unsigned int shard_ring_cap);

/* Two rings with full-height stage-2 x ranges (:438-466). */
void s01g_attach_gpu_rings(S01gHandle* h,
                           void* ring_buf_0, void* ring_head_0,
                           void* ring_buf_1, void* ring_head_1,
                           unsigned long long ring_mask,
                           int W2, int H2,
                           int proc_lo_0, int proc_hi_0,
                           int proc_lo_1, int proc_hi_1);
/* Up to 16 rings, x and y ranges per ring (:476-500). */
void s01g_attach_gpu_rings_multi(S01gHandle* h, int n_blocks,
                                 void* const* ring_bufs,
                                 void* const* ring_heads,
                                 unsigned long long ring_mask,
                                 int W2, int H2,
                                 const int* proc_x_los, const int* proc_x_his,
                                 const int* proc_y_los, const int* proc_y_his);

/* n events of 4 floats (t, x, y, p); returns the number accepted (events
 * outside the sensor are counted in stats slot 3) (:502-537). */
int  s01g_submit_batch(S01gHandle* h, const float* events_packed, int n);

/* 32 doubles, slot map of :540-546:
 *   [0] events processed  [1] halo events (0: no replicas are processed)
 *   [2] passed gate 0     [3] out-of-bounds events   [4] seconds since
 *   init / reset          [5] events queued, not yet processed
 *   [6..11] submit -> publish latency p50, p90, p99, p99.9, max, mean (us)
 *   [12] latency samples  [13] passed gate 1
 *   [14], [15] records published to ring 0, 1
 *   [16..21] segment ns: preprocess, s0, tdrop0, s1, tdrop1, push -- the
 *            GPU batches report their whole stage-0/1 time under s0
 *   [22..27] segment counts (same order)  [28..31] reserved */
void s01g_snapshot_stats(S01gHandle* h, double* out);
void s01g_reset_stats(S01gHandle* h);

/* xorshift64 producer at rate_mev Mev/s: x = r % W, y = (r >> 16) % H,
 * p = bit 32 of r, t advancing by 1/rate us (:603-707). */
void s01g_start_synthetic(S01gHandle* h, double rate_mev, int pin_core,
                          uint64_t seed);
void s01g_stop_synthetic(S01gHandle* h);
uint64_t s01g_synthetic_n_pushed(S01gHandle* h);

/* Stops the producer, drains the queue, releases everything (:735-753). */
void s01g_shutdown(S01gHandle* h);

/* No counterpart in the reference: waits until every event submitted so
 * far has been processed and its records published.  Returns 0, or -1
 * after timeout_s seconds. */
int  s01g_flush(S01gHandle* h, double timeout_s);

#ifdef __cplusplus
}
#endif
#endif
