/* ssla_b200.h -- C ABI of the B200-native SSLA-S per-event hot path.
 *
 * libssla_b200.so (ssla_rt_b200/) exports everything declared here: plain
 * C types, pointers and sizes, no torch or C++ types.  Each entry point
 * names the reference interface it replaces (paths relative to the
 * haohq19/ssla-rt checkout).  Device pointers are CUDA global-memory
 * pointers of the engine's device; `stream` is a cudaStream_t (NULL = the
 * legacy default stream).  Every function returns SSLA_OK (0) or an
 * SSLA_ERR_* code and never aborts; ssla_last_error() gives the message.
 */
#ifndef SSLA_B200_H
#define SSLA_B200_H

#include <stddef.h>
#include <stdint.h>

#include "ssla_abi_types.h"

#ifdef __cplusplus
extern "C" {
#endif

enum {
    SSLA_OK = 0,
    SSLA_ERR_ARG = 1,        /* bad argument / shape / layout              */
    SSLA_ERR_CUDA = 2,       /* a CUDA call failed                         */
    SSLA_ERR_LOAD = 3,       /* weights.npz / meta.json missing or invalid */
    SSLA_ERR_CAPACITY = 4,   /* more events than the engine was sized for  */
    SSLA_ERR_NO_DEVICE = 5   /* no CUDA device / kernels not loadable      */
};

/* Temporal-dropout gate layouts.
 * DECOMP: the single-thread reference chain, src/legacy/schemes/
 *   s2_decomp_st.cpp:138-176 (gates after s0, s1, s2 on the s1, s2, s3
 *   grids; head for every event finishing s3).
 * HYBRID: the production chain, src/lib_stage01_to_gpu.cpp:228-311 followed
 *   by orin/kernels/ssla_s2_s3_head_celled.cuh:1679-1755 (gates on the s1,
 *   s2, s2 and s3 grids; the fourth gates the head). */
enum { SSLA_LAYOUT_DECOMP = 0, SSLA_LAYOUT_HYBRID = 1 };

/* Per-event flag bits (ssla_engine_drain_* `flags`). */
enum {
    SSLA_F_VALID = 1,  /* in bounds, entered stage 0     */
    SSLA_F_R1 = 2,     /* passed gate 0, entered stage 1 */
    SSLA_F_R2 = 4,     /* entered stage 2                */
    SSLA_F_R3 = 8,     /* entered stage 3                */
    SSLA_F_R4 = 16,    /* produced a head prediction     */
    SSLA_F_FOREIGN = 32 /* strip mode: a neighbour's band event (its outputs are the neighbour's) */
};

typedef struct SslaEngine SslaEngine;

typedef struct {
    int n_partitions;          /* independent event streams (ring partitions) */
    int max_events;            /* capacity of one drain call, all partitions  */
    int layout;                /* SSLA_LAYOUT_*                                */
    int device;                /* CUDA device ordinal                          */
    int record_stage_outputs;  /* 1: keep per-event stage outputs (tests)     */
    int max_events_per_partition; /* 0: ceil(max_events / n_partitions)      */
} SslaEngineConfig;

typedef struct {
    int H, W, ncls, tdrop_window, layout, n_partitions, max_events;
    int device;
    long long stage_events[5]; /* last drain: events entering s0..s3 / head   */
    int launches;              /* kernels the last drain launched              */
    int _pad;
} SslaEngineInfo;

/* One timed phase of a profiled drain (a kernel or a short kernel group). */
typedef struct {
    char  name[40];
    float ms;
    int   launches;
} SslaPhaseTime;

/* State buffers readable / writable per partition. `index` is the layer
 * (HIDDEN), gate (COUNTER) or stage (STAGE_OUT). STAGE_OUT and FLAGS cover
 * the events of the last drain call (all partitions; partition ignored). */
enum {
    SSLA_STATE_HIDDEN = 0,     /* float [Hs*Ws][C_s]                          */
    SSLA_STATE_COUNTER = 1,    /* uint8 gate counters on the gate's grid      */
    SSLA_STATE_LAST_T = 2,     /* double [H*W], -1 = never seen               */
    SSLA_STATE_PREDS_DEC = 3,  /* float [H3*W3][5+ncls] cx,cy,w,h,obj,cls..   */
    SSLA_STATE_PREDS_RAW = 4,  /* float [H3*W3][5+ncls] reg0..3,obj,cls..     */
    SSLA_STATE_VERSION = 5,    /* uint32 [H3*W3] head writes per cell          */
    SSLA_STATE_STAGE_OUT = 6,  /* float [max_events][C_s]                      */
    SSLA_STATE_FLAGS = 7       /* uint8 [max_events]                           */
};

/* Loads <weights_dir>/meta.json + weights.npz (schema of
 * tools/make_ssla_stub.py:29-144), reshapes the layers into per-position
 * tensors and folds the head's BatchNorm, uploads everything to `device`
 * and allocates per-partition state sized for cfg->max_events.
 * Replaces deploy::SslaSPipeline::load + reset (src/ssla_kernels.cpp:161-286)
 * and the weight half of s01g_init_full (src/lib_stage01_to_gpu.cpp:354-421). */
int  ssla_engine_create(const char* weights_dir, const SslaEngineConfig* cfg,
                        SslaEngine** out);
void ssla_engine_destroy(SslaEngine* eng);

/* Zero hidden state and counters, forget last timestamps, set every
 * prediction row to head(0) (src/ssla_kernels.cpp:276-286, :969-989). */
int  ssla_engine_reset(SslaEngine* eng, void* stream);

/* Runs every event of every partition through s0..s3 and the head, in
 * stream order per partition, with exactly the sequential semantics of the
 * selected layout.  events_dev: float (t, x, y, p) rows (openeva::Event,
 * vendor/openeva/event.h:8-13); partition p owns rows
 * [part_offsets[p], part_offsets[p+1]) (host array, n_partitions+1 ints).
 * flags_dev (may be NULL): uint8 per row, SSLA_F_* bits.  Asynchronous on
 * `stream`.  Replaces the per-event loop of s2_decomp_st.cpp:138-176 and
 * the shard_worker + persistent-kernel chain of the hybrid runtime. */
int  ssla_engine_drain_device(SslaEngine* eng, const float* events_dev,
                              const int* part_offsets, uint8_t* flags_dev,
                              void* stream);

/* Same, from and to host memory (pinned or pageable): copies the events in,
 * drains, copies the flags out and synchronises `stream`.  The analogue of
 * s01g_submit_batch (src/lib_stage01_to_gpu.cpp:501-538) for a batch. */
int  ssla_engine_drain_host(SslaEngine* eng, const float* events_host,
                            const int* part_offsets, uint8_t* flags_host,
                            void* stream);

/* Pipelined form of ssla_engine_drain_host for pinned host buffers: the
 * copy of the events runs on an engine-owned copy stream into one of two
 * device buffers, so it overlaps the previous drain on `stream`.  The drain
 * waits for it, then the flags (flags_host, may be NULL) and every
 * partition's decoded predictions (preds_host, n_partitions x cells x
 * (5+ncls) floats, may be NULL) go back on `stream`: written by a kernel
 * chained to the drain where the buffer is pinned (page-locked, device-
 * mapped), copied where it is pageable.  Returns without waiting: the host
 * buffers belong to the call until `stream` passes it.
 * The shard threads of the reference overlap their ring pushes with the
 * GPU drain the same way (src/lib_stage01_to_gpu.cpp:157-311). */
int  ssla_engine_drain_host_async(SslaEngine* eng, const float* events_host,
                                  const int* part_offsets, uint8_t* flags_host,
                                  float* preds_host, void* stream);

/* One event (t, x, y, p; host memory, passed by value to the kernel) of
 * `partition` through preprocess, the gates, stages 0-3 and the head in a
 * single launch -- the batch-of-1 path.  Leaves exactly the state a drain
 * of that one event leaves.  flag_out (may be NULL) receives the event's
 * SSLA_F_* bits; pred_out (may be NULL, 5+ncls floats) receives the decoded
 * prediction row of the event's stage-3 cell when the event reached the
 * head.  Both may be device memory or pinned host memory (written by the
 * kernel directly).  Asynchronous on `stream`.  Replaces one
 * SslaSPipeline::step (src/ssla_kernels.cpp:927-989) / one ring record of
 * the persistent kernel (ssla_s2_s3_head_celled.cuh:1547-1784). */
int  ssla_engine_step(SslaEngine* eng, int partition, const float* event,
                      uint8_t* flag_out, float* pred_out, void* stream);

/* Batch-of-1 latency: steps the n events (host array of 4-float rows) one
 * at a time with ssla_engine_step -- flags and prediction row written by
 * the kernel into pinned host memory -- and records, per event, the host
 * time from the call to the stream synchronize returning (microseconds).
 * flags_out (may be NULL) receives each event's SSLA_F_* bits.  Measurement
 * support; the engine's state advances as with ssla_engine_step. */
int  ssla_engine_step_latency(SslaEngine* eng, int partition, const float* events_host,
                              int n, double* latency_us, uint8_t* flags_out);

/* Live loop: a resident cluster that takes raw events from a ring in pinned
 * host memory (openeva::Event rows, the SPSC head / tail protocol of
 * include/spsc.h:9-11 and orin/orin/ring.py:34-152) and runs each through
 * preprocess, the gates, stages 0-3 and the head, in ring order, one event
 * at a time -- the full-pipeline counterpart of the reference's polling
 * kernel k_ssla_s2s3_celled_persistent_multi (ssla_s2_s3_head_celled.cuh:
 * 1547-1784) with its tails / events_done / stop_flag words
 * (orin/hybrid_runner_multi.py:445-462).  Every pointer is pinned host
 * memory (cudaHostAlloc / cudaMallocHost / torch pin_memory). */
typedef struct SslaLiveRing {
    const float* events;             /* [capacity][4] t, x, y, p, written by the host          */
    unsigned long long capacity;     /* power of two                                           */
    unsigned long long* head;        /* events published: host release-stores after the slots  */
    unsigned long long* tail;        /* events taken from the ring (device)                    */
    unsigned long long* events_done; /* events finished, outputs and state visible (device)    */
    uint8_t* flags;                  /* [capacity] SSLA_F_* bits of each event, or NULL        */
    float* preds;                    /* [capacity][5+ncls] decoded row of head events, or NULL */
    int* stop_flag;                  /* host sets non-zero to end the loop                      */
} SslaLiveRing;

/* Status bits of a live loop (ssla_engine_live_join). */
enum {
    SSLA_LIVE_ERR_WEIGHTS = 1,   /* a weight copy did not complete in time        */
    SSLA_LIVE_ERR_INPUT = 2,     /* a layer input message did not arrive          */
    SSLA_LIVE_ERR_CONTRIB = 4,   /* contributions did not arrive                  */
    SSLA_LIVE_ERR_EVENT = 8,     /* no event message within the idle bound        */
    SSLA_LIVE_ERR_DONE = 16,     /* an event's completion did not arrive          */
    SSLA_LIVE_EXIT_STOP = 0x100, /* left the loop on the stop flag                */
    SSLA_LIVE_EXIT_IDLE = 0x200  /* left the loop after idle_timeout_ms           */
};

/* Launches the live loop of `partition` on `stream` and returns; events
 * are taken from index *ring->tail on.  The loop ends when *stop_flag is
 * non-zero or after idle_timeout_ms without a new event.  The partition's
 * state belongs to the loop until ssla_engine_live_join returns. */
int  ssla_engine_live_start(SslaEngine* eng, int partition, const SslaLiveRing* ring,
                            unsigned idle_timeout_ms, void* stream);
/* Waits for the loop to end; *status (may be NULL) receives SSLA_LIVE_*
 * bits.  Returns SSLA_ERR_CUDA if a wait inside the loop ran out. */
int  ssla_engine_live_join(SslaEngine* eng, unsigned* status);

/* Head selection of the engine's drains.  SSLA_HEAD_EXACT (the default):
 * the YOLOX head on the CUDA cores in the reference's fmaf order, bit-exact
 * with the CPU oracle.  SSLA_HEAD_TENSOR: its two 1x1 convolutions (cls_conv
 * | reg_conv, 96 -> 192) as one tcgen05 tensor-core GEMM over the drain's head
 * events in three TF32 terms (split TF32), the rest as before; predictions
 * then equal the exact head's within fp32 rounding, not bit for bit.  Flags,
 * hidden state and versions are unaffected.  The single-event step and the
 * live loop always use the exact head.  Replaces the head of the reference's
 * drains (vendor/openeva/heads/async_yolox.h:203-254,
 * orin/kernels/ssla_s2_s3_head_celled.cuh:841-902). */
enum { SSLA_HEAD_EXACT = 0, SSLA_HEAD_TENSOR = 1 };
int  ssla_engine_set_head_mode(SslaEngine* eng, int mode);
/* Status bits of the tensor-core head since the last call (bit 0: a wait
 * for its MMAs ran out); synchronises the device, then clears them. */
int  ssla_engine_head_status(SslaEngine* eng, unsigned* status);

/* Test hook for the loop's timeout path, no reference counterpart: the next
 * live loop started on `eng` withholds the completion message of ring event
 * `ring_index` (-1: none) from its head CTA.  The head CTA's bounded wait
 * then runs out, every CTA leaves through the loop's exit barrier, and
 * ssla_engine_live_join reports SSLA_LIVE_ERR_DONE in *status and returns
 * SSLA_ERR_CUDA; events before `ring_index` are finished normally.  Not
 * allowed while a loop is running. */
int  ssla_engine_live_withhold_completion(SslaEngine* eng, long long ring_index);

/* Batch-of-1 latency through the live loop: publishes the n events (host
 * array of 4-float rows) one at a time into a pinned ring and records, per
 * event, the host time from publishing the event to observing
 * events_done pass it (microseconds).  flags_out (may be NULL) receives
 * each event's SSLA_F_* bits and preds_out (may be NULL, n x (5+ncls))
 * each head event's decoded row (other rows untouched). */
int  ssla_engine_live_latency(SslaEngine* eng, int partition, const float* events_host, int n,
                              double* latency_us, uint8_t* flags_out, float* preds_out);

/* Ring drains: one pinned SslaLiveRing per partition -- independent event
 * streams (camera streams, ring partitions), each with its own producer --
 * drained together by the chunk path.  The reference's shard workers feed
 * GPU rings that its persistent kernel drains in ring order
 * (src/lib_stage01_to_gpu.cpp:157-311, ssla_s2_s3_head_celled.cuh:
 * 1547-1784); here the rings carry raw events and every stage runs on the
 * GPU.  stop_flag is not used.  Attach once (synchronises the device); each
 * ring's tail at attach is where draining starts. */
int  ssla_engine_rings_attach(SslaEngine* eng, const SslaLiveRing* rings, int n_rings);

/* One ring drain on `stream`: takes, from every ring, up to max_per_ring of
 * its published events (head read with acquire; at most max_total events in
 * all, and within max_events / max_events_per_partition), copies them from
 * the rings into the device (releasing each ring's tail once copied), runs
 * the full path over them and then writes each event's SSLA_F_* bits into
 * flags[index & (capacity-1)] and each head event's decoded prediction row
 * into preds[index & (capacity-1)] (either may be NULL) before releasing
 * events_done.  *n_taken receives the events taken (0: nothing published);
 * taken (may be NULL, n_partitions ints) each ring's share.  Asynchronous. */
int  ssla_engine_drain_rings(SslaEngine* eng, int max_per_ring, long long max_total, int* taken,
                             int* n_taken, void* stream);

/* Per-drain record of ssla_engine_serve_rings. */
typedef struct SslaServeLog {
    unsigned long long* done_ns;    /* [cap] CLOCK_MONOTONIC ns when drain k was seen complete, or NULL */
    int* taken;                     /* [cap][n_partitions] events of each ring in drain k, or NULL      */
    int cap;                        /* entries of done_ns / taken                                        */
    int n;                          /* out: entries written, min(drains, cap)                            */
    int drains;                     /* out: drains completed                                              */
    uint8_t* const* flags_hist;     /* [n_partitions] arrays receiving each drained event's flags at
                                       (ring index - the ring's tail at attach), or NULL                  */
    unsigned long long hist_len;    /* length of each flags_hist array                                    */
} SslaServeLog;

/* Serves the rings until `total` events have been drained, or until
 * idle_timeout_ms passes with nothing published and nothing in flight:
 * each drain is formed (ssla_engine_drain_rings) while the previous one
 * runs, and is logged when it completes.  *served receives the events
 * drained.  Synchronises `stream`. */
int  ssla_engine_serve_rings(SslaEngine* eng, int max_per_ring, unsigned long long total,
                             unsigned idle_timeout_ms, SslaServeLog* log, unsigned long long* served,
                             void* stream);

/* Paced replay producer: a host thread that publishes each stream's events
 * into its ring at their timestamps -- event i (t_i microseconds) of ring r
 * is due at start_ns + t_i * 1000 * time_scale on CLOCK_MONOTONIC; with
 * time_scale 0 every event is due at start_ns and only ring space paces
 * the thread.  Slots are written, then head is release-stored; free space is
 * read from tail (acquire).  The synthetic producer of the reference
 * (s01g_start_synthetic, src/lib_stage01_to_gpu.cpp:637-672) draws random
 * events at a rate; this one replays given streams, so the same events can
 * be checked against the oracle.  Host-only; the arrays must stay valid
 * until ssla_replay_join.  start_ns 0 = 2 ms after the call.  NULL on bad
 * arguments (ssla_last_error). */
typedef struct SslaReplay SslaReplay;
typedef struct SslaReplayStats {
    unsigned long long published;   /* events published                                        */
    unsigned long long start_ns;    /* event time 0 on CLOCK_MONOTONIC                          */
    long long max_lag_ns;           /* latest publish after its due time (pacing or full rings) */
    unsigned long long full_waits;  /* rounds in which a due event found its ring full          */
} SslaReplayStats;
SslaReplay* ssla_replay_start(const SslaLiveRing* rings, int n_rings, const float* const* events,
                              const unsigned long long* counts, double time_scale,
                              unsigned long long start_ns);
/* Asks the thread to stop early (it ends after its current round). */
void ssla_replay_stop(SslaReplay* rp);
/* Waits for the thread (every event published, or stopped), fills *stats
 * (may be NULL) and frees the handle. */
int  ssla_replay_join(SslaReplay* rp, SslaReplayStats* stats);

/* Stages 0-1 only (HYBRID layout): preprocess, gates 0-1, layers 0-3 for
 * every event (state of stages 0-1 advances), and one HybridInputRec per
 * event that passed gate 1 -- t, stage-2 x / y, feat1 = the stage-1 output;
 * seq_done, t_push_ns and t_emit_ns zero -- written to records_dev
 * (device memory, room for records_cap >= the drain's event count),
 * partition-major in stream order.  record_offsets (host, n_partitions+1
 * ints) receives each partition's record range.  Synchronises `stream`.
 * Replaces the shard workers' stage-0/1 path that feeds the GPU rings
 * (src/lib_stage01_to_gpu.cpp:157-311). */
int  ssla_engine_drain_records(SslaEngine* eng, const float* events_dev,
                               const int* part_offsets, void* records_dev,
                               int records_cap, int* record_offsets,
                               uint8_t* flags_dev, void* stream);

/* Owned range of `partition` in stage-2 cells, [x0, x1) x [y0, y1) (default:
 * the whole grid).  Events outside it still update state (halo) but commit
 * no prediction -- the owned_lo / owned_hi / owned_y_lo / owned_y_hi bounds
 * of the reference's HybridStrip (ssla_s2_s3_head_celled.cuh:84-127,
 * :1663-1670) for strip-sharded sensors.  Synchronises `stream`. */
int  ssla_engine_set_owned(SslaEngine* eng, int partition, int x0, int x1, int y0, int y1,
                           void* stream);

/* Prediction-tensor checkpoints in the reference's OracleRecorder file
 * format (include/oracle.h:10-19; read by its diff_dumps / oracle_diff,
 * src/oracle_diff.cpp): header {magic 'OEVA', version 1, num_anchors, cols,
 * num_checkpoints}, then per checkpoint {uint64 event_idx, float
 * [num_anchors][cols]}.  Host-only: writes the given checkpoints. */
int  ssla_write_oracle_dump(const char* path, int num_anchors, int cols, int n_checkpoints,
                            const uint64_t* event_idx, const float* preds);
/* Runs the n host events (4-float rows) of one stream through `partition`
 * (drains split after events 0, every, 2*every, ...) and dumps the decoded
 * predictions tensor after each of those events -- OracleRecorder::record
 * (include/oracle.h:43-54) driven the way src/legacy/schemes/
 * s2_decomp_st.cpp:195-207 drives it.  The partition's state advances. */
int  ssla_engine_oracle_dump(SslaEngine* eng, int partition, const float* events_host, int n,
                             int every, const char* path);

/* Exact strip sharding (one partition per engine).  The engine drains its
 * own stage-0 rows [lo, hi) plus `band_rows` (a multiple of 8) of each
 * present neighbour's rows, and after each of layers 1-6 exchanges with its
 * neighbours the next-layer inputs of the events in their bands, so the
 * events it owns get exactly the single-sensor results (no halo drift);
 * only owned events commit predictions.  cap_rows bounds the band rows of
 * one stage list per drain (larger bands set SSLA_STRIP_ERR_CAPACITY).
 * Side 0 is the neighbour above (rows < lo), side 1 the one below. */
enum {
    SSLA_STRIP_ERR_CAPACITY = 1,  /* more band rows than cap_rows            */
    SSLA_STRIP_ERR_TIMEOUT = 2,   /* a neighbour's rows did not arrive       */
    SSLA_STRIP_ERR_MISMATCH = 4   /* a neighbour sent a different row count  */
};
int  ssla_engine_strip_init(SslaEngine* eng, int lo, int hi, int band_rows, int has_up, int has_down,
                            int cap_rows);
/* This engine's receive buffer of `side`: its device address (for a
 * neighbour in the same process) and a cudaIpcMemHandle_t (64 bytes, may be
 * NULL) for a neighbour in another process. */
int  ssla_engine_strip_recv_buffer(SslaEngine* eng, int side, void** dev_ptr, void* ipc_handle);
/* Where this engine's rows for `side` go: the receive buffer of that
 * neighbour for the opposite side, by device address or IPC handle. */
int  ssla_engine_strip_connect(SslaEngine* eng, int side, void* peer_dev_ptr, const void* peer_ipc_handle);
/* One drain of the strip's events (device rows, stream order) with the
 * exchanges; waits for the neighbours' rows on the device (bounded), so
 * each neighbour must drain the chunk with the same global event range on
 * its own GPU concurrently.  The events must lie in rows [lo - band_rows,
 * hi + band_rows) (the routing of ssla_rt_b200/strips.py); the tile lists
 * of a strip engine cover only those rows, so an event outside them is not
 * processed.  Asynchronous on `stream`. */
int  ssla_engine_strip_drain(SslaEngine* eng, const float* events_dev, int n, uint8_t* flags_dev,
                             void* stream);
/* The same for k strips sharing one GPU and one stream: the engines' steps
 * run in lockstep, each exchange after both sides' layers (no device waits). */
int  ssla_strip_drain_lockstep(SslaEngine* const* engines, int k, const float* const* events_dev,
                               const int* n, uint8_t* const* flags_dev, void* stream);
/* SSLA_STRIP_ERR_* bits since the last call (read and cleared; synchronises). */
int  ssla_engine_strip_status(SslaEngine* eng, unsigned* status);

int  ssla_engine_state_bytes(SslaEngine* eng, int kind, int index, size_t* bytes);
/* partition -1 (kinds HIDDEN .. VERSION): every partition's buffer back to
 * back, in partition order, in one copy. */
int  ssla_engine_read_state(SslaEngine* eng, int kind, int partition, int index,
                            void* host_dst, size_t bytes);
int  ssla_engine_write_state(SslaEngine* eng, int kind, int partition, int index,
                             const void* host_src, size_t bytes);
/* Device address of a state buffer (for zero-copy consumers of predictions). */
void* ssla_engine_state_ptr(SslaEngine* eng, int kind, int partition, int index);
int  ssla_engine_info(SslaEngine* eng, SslaEngineInfo* info);

/* drain_n contract of the reference's P1 kernels: each block processes its
 * records in order and writes one HybridS2S3OutputSlot per record; weights,
 * hidden state and tdrop counters are read from / written to the device
 * buffers named in `cfg` (a HOST copy of the HybridS2S3Config the reference
 * kernel receives).  rings / outs / batch_clks: host arrays of device
 * pointers, ns: host array.  batch_clks (may be NULL): every 2-word batch
 * slot of a block receives the %globaltimer ns at drain start and end.
 * Replaces k_ssla_s2s3_celled_drain_n_multi
 * (orin/kernels/ssla_s2_s3_head_celled.cuh:1108-1255). */
int  ssla_s2s3_drain_n_multi(const HybridS2S3Config* cfg,
                             const HybridInputRec* const* rings, const int* ns,
                             HybridS2S3OutputSlot* const* outs,
                             unsigned long long* const* batch_clks,
                             void* stream);
/* Fills the weight and head pointers of cfg->layers[block][0..3] (layers
 * 4-7) and cfg->head_* with this engine's device weights, which are laid out
 * as the reference's GPU kernels read them (qvgIn (9, IN, 3*OUT), goW
 * (9, OUT, OUT) and input_proj (IN, OUT) row-major, the 2-layer head with BN
 * folded, (IN, OUT) row-major) -- the buffers orin/orin/weights_ssla.py:24-88
 * and orin/orin/hybrid_common.py:76-111 build for a HybridS2S3Config.  The
 * pointers stay valid while the engine lives.  block: 0..15. */
int  ssla_engine_fill_s2s3_config(SslaEngine* eng, HybridS2S3Config* cfg, int block);
/* Two-ring form; replaces k_ssla_s2s3_celled_drain_n
 * (orin/kernels/ssla_s2_s3_head_celled.cuh:914-1095). */
int  ssla_s2s3_drain_n(const HybridS2S3Config* cfg,
                       const HybridInputRec* ring0, const HybridInputRec* ring1,
                       int n0, int n1,
                       HybridS2S3OutputSlot* out0, HybridS2S3OutputSlot* out1,
                       unsigned long long* batch_clk0,
                       unsigned long long* batch_clk1, void* stream);

/* Allocation-free gate pass.  No counterpart in the reference: its drain
 * kernels always run the full layer stack.  For callers that cannot allocate
 * device or pinned memory at the call site (a per-batch real-time loop where
 * cudaMalloc / cudaFree may synchronise the device, or a host whose device
 * memory is owned by another runtime's pool): evaluates the stage-2 and
 * stage-3 tdrop gates of ssla_s2s3_drain_n_multi for every record (ring
 * order per block), advances cfg's tdrop counters in place and writes the
 * pass2 / pass3 codes of each output slot exactly as the drain would; hidden
 * state and s3_feat are untouched.  Scratch lives in a fixed file-scope
 * device array of 864 KiB per device: at most SSLA_NOALLOC_MAX_RECORDS
 * records and SSLA_NOALLOC_MAX_CELLS blocks x stage-3 cells per call (larger
 * calls fail with SSLA_ERR_CAPACITY).  Work is linear in the records (they
 * are bucketed by stage-3 cell inside the scratch before the gates).
 * Enqueues on `stream` and returns without synchronising.  The first call on
 * a device (and the first after its context changed) looks the scratch array
 * up and should precede any stream capture on that device; calls that
 * overlap in time on one device share the scratch and race. */
#define SSLA_NOALLOC_MAX_RECORDS 65536
#define SSLA_NOALLOC_MAX_CELLS 65535
int  ssla_s2s3_gate_codes_noalloc(const HybridS2S3Config* cfg,
                                  const HybridInputRec* const* rings, const int* ns,
                                  HybridS2S3OutputSlot* const* outs, void* stream);

/* Per-phase timing (the analogue of the reference's clock64 phase stamps,
 * orin/kernels/ssla_s2_s3_head_celled_profile.cuh:17-40): when enabled,
 * every drain records a CUDA event after each phase on its stream;
 * ssla_engine_phase_times synchronises and returns the elapsed times of the
 * last drain's phases in launch order. */
int  ssla_engine_set_profiling(SslaEngine* eng, int enable);
int  ssla_engine_phase_times(SslaEngine* eng, SslaPhaseTime* out, int max_n, int* n_out);

/* FP32 FMA-pipe peak of `device`, measured with a dependent-chain-free FFMA
 * loop over every SM (the denominator of the engine's roofline). */
int  ssla_measure_fp32_peak(int device, double* tflops_out);

/* Self-test of the device reciprocal inside every sigmoid (hardware
 * approximation + one Newton-Raphson step): compares it on `device` with
 * IEEE round-to-nearest 1/y for every float y in [1, 2^126), the range of
 * the sigmoid's denominator.  *mismatches = 0 means the device sigmoid and
 * ssla_sigmoidf_host (which divides) agree bit for bit; *first_bad (may be
 * null) receives the lowest mismatching bit pattern, 0xFFFFFFFF if none. */
int  ssla_selftest_reciprocal(int device, unsigned long long* mismatches, unsigned* first_bad);

/* Self-test of the packed sigmoid the stage-0/1 scans and the stage-2/3
 * GEMM epilogue use (two sigmoids per call with paired FP32 operations):
 * compares it on `device`, bit for bit, with two calls of the scalar device
 * sigmoid for every float x (pairs (x, -x)).  *mismatches = 0 means the
 * packed form changes no result; *first_bad (may be null) receives the
 * lowest mismatching bit pattern of the first component, 0xFFFFFFFF if none. */
int  ssla_selftest_sigmoid_pair(int device, unsigned long long* mismatches, unsigned* first_bad);

/* Portable exp used by every sigmoid / SiLU / box decode of the engine
 * (the device code's exact twin), for tests on hosts without a GPU. */
float ssla_expf_host(float x);
/* The sigmoid every LRU gate and SiLU of the engine uses (the device code's
 * exact twin): 1 / (1 + exp(-x)) with a degree-6 minimax exp on the clamped
 * range it needs, within 2.3 ulp of the exact value. */
float ssla_sigmoidf_host(float x);

const char* ssla_last_error(void);
const char* ssla_version(void);

#ifdef __cplusplus
}
#endif
#endif
