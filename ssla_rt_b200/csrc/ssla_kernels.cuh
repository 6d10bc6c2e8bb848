// ssla_kernels.cuh -- kernel argument blocks and launch entry points.
#pragma once

#include <cuda_runtime.h>

#include "ssla_device.cuh"

namespace ssla {

struct FilterArgs {
    Geo g;
    int stage;
    const uint32_t* ev_xy;   // stage 0: packed pixel coords per event
    const StageEntry* E;     // stage >= 1: stage list
    const uint8_t* rflags;   // per-event reach flags
    const int* range;        // [P+1] partition ranges in this stage's index space
    int2* tl;                // tile lists
    int* tl_cnt;             // entries per (partition, tile, segment)
    uint8_t out_bit;         // reach bit meaning "second-layer output needed"
    int ev_row_lo, ev_row_hi;  // stage-0 pixel rows holding the drain's events (hi <= lo: all)
    int trow0;               // first tile row of the launch (set by launch_filter)
    int* zero_work;          // k_flag_s0: the stage-0/1 scans' 8 work counters, zeroed (may be null)
};

struct GateArgs {
    Geo g;
    const float4* ev;
    const int* ev_off;       // [P+1]
    const int2* tl0;         // stage-0 tile lists (tile = s3 block)
    const int* tl0_cnt;
    const PartState* parts;
    uint8_t* rflags;
    float* X1;               // [N][12] layer-0 output per event
    float* Rcopy;            // [N][12] layer-1 residual (events entering stage 1)
    DevLayer L0;
    int n_gates;             // gates applied: 4 (full path) or 2 (stages 0-1 only)
};

// Gates for drain_n records entering at stage 2 (tdrop_s2 on the s2 grid,
// tdrop_s3 on the s3 grid).
struct Gate2Args {
    Geo g;
    const int* rec_off;      // [P+1]
    const int2* tl2;         // stage-2 tile lists
    const int* tl2_cnt;
    const PartState* parts;
    uint8_t* rflags;
};

struct CompactArgs {
    Geo g;
    int s_first;             // lists s_first+1 .. 4 are built
    int tiles_per_part;
    int ctile;               // events per compaction tile
    const int* ev_off;       // [P+1]
    const uint8_t* rflags;
    const uint32_t* ev_xy;
    int* tilecnt;            // [P*tiles][4]
    int* tilebase;           // [P*tiles][4]
    StageEntry* E[5];
    int* off[5];             // [P+1] per list
    int* count;              // [5]
};

struct ScanArgs {
    Geo g;
    int stage, layer;
    const int2* tl;
    const int* tl_cnt;
    const int* range;        // [P+1] this stage's partition ranges
    float* S;                // layer's (q, v, a) per (entry, delta); q -> q*h
    const PartState* parts;
    const uint8_t* rflags;   // stage-0 second-layer output flags
    int second;              // 1: second layer of the stage
};

// Rows of a contrib / ln / GEMM launch: the first `count[list]` entries of a
// stage list (list 1..4), or `n_static` chunk events (list 0).
struct ScanFusedArgs {
    Geo g;
    int stage, layer;
    const int2* tl;
    const int* tl_cnt;
    const int* range;        // [P+1] this stage's partition ranges
    const PartState* parts;
    const uint8_t* rflags;   // stage-0 second-layer output flags
    int second;              // 1: second layer of the stage
    const float* X;          // [entry][IN] layer input rows
    const float* W;          // qvgT [9][IN][3*OUT]
    float* QH;               // [(entry * 9 + delta) * OUT] q * h rows
    int* work;               // work-item counter of this launch, zero on entry
    const int* hot;          // hot tiles of the stage: [0] count, [1..] (p * ntiles + tile); null: none
    const uint8_t* hot_flag; // [P * ntiles] 1 = the tile is scanned cell by cell; null: none
    int gpt;                 // group items per tile (scan_fused_groups_per_tile)
};

// When a stage-0/1 scan has fewer 2x2-group work items than resident warps,
// tiles whose event lists exceed this many entries are scanned with one work
// item per cell instead.
constexpr int kHotTileEntries = 4096;

struct HotArgs {
    Geo g;
    int stage;
    int threshold;           // list entries above which a tile is hot
    const int* tl_cnt;
    const int* range;        // [P+1] this stage's partition ranges
    int* hot;                // [0] count, [1..] hot (p * ntiles + tile), ascending
    uint8_t* hot_flag;       // [P * ntiles]
};

void launch_hot_tiles(cudaStream_t st, const HotArgs& a);
// Warps of the stage-0/1 scan kernel of `layer` resident on the device.
int scan_fused_resident_warps(int layer);
// Group work items per 8x8 tile of a stage-0/1 scan layer over tile_count
// (partition, tile) pairs; the launch takes it in ScanFusedArgs::gpt.
int scan_fused_groups_per_tile(int layer, long long tile_count);

struct ContribArgs {
    Geo g;
    int stage;               // stage of the gathered layer
    int second;              // 1: second layer of the stage (rows read S row kprev)
    int list;
    int n_static;
    const int* count;
    const StageEntry* E;     // row entries (list > 0)
    const uint32_t* ev_xy;   // list == 0
    const uint8_t* rflags;
    const float* S;          // qh rows at (k * A + delta) * qstride
    int qstride;             // 3*OUT (GEMM-fed S rows) or OUT (compact QH rows)
    const float* goWT;       // [A][OUT][OUT]
    float* C;                // [row][A][OUT] contributions
    // Stages 0-1: S holds the state after each consumed hit (h, not q * h);
    // q = X row . qvgT[delta][:, 0:OUT] is formed here and multiplied in.
    const float* Xq;         // [row][IN] layer input rows
    const float* Wq;         // qvgT [9][IN][3*OUT]
};

struct LnArgs {
    Geo g;
    int stage;
    int second;
    int list;
    int n_static;
    const int* count;
    const StageEntry* E;
    const uint32_t* ev_xy;
    const uint8_t* rflags;
    uint8_t copyres_bit;     // first layer: R_next = x for events with this bit
    const float* C;          // contributions [row][A][OUT]
    const float* R_in;       // residual rows of the layer (S row index)
    float* X_out;            // [row][OUT] layer output
    float* R_next;           // copy residual of the stage's second layer
    DevLayer L;
    float* stage_out;        // optional [N][OUT] per chunk event (second layers)
    float* slot_feat;        // drain_n: [N][96] the reference's s3_feat slot
    const float* ipT_next;   // next stage's input_proj [OUT][2*OUT] (or null)
    float* R_ipnext;         // its residual rows [row][2*OUT]
};

struct HeadArgs {
    Geo g;
    const int* count;        // count[4] = head events
    const StageEntry* E4;
    const float* X;          // [row][96] stage-3 features in E_4 order
    DevHead head;
    float* head_dec;         // [cap4][5+ncls]
    float* head_raw;
    const float* tc_w1;      // tensor-core head: [cls_conv | reg_conv] rows [192][96], TF32 hi terms then lo terms
    unsigned* err;           // tensor-core head: bit 0 when a wait for its MMAs ran out (host-mapped, or null)
};

enum { COLS_ALL = 0, COLS_VG = 1, COLS_Q = 2, COLS_RES = 3 };


struct GemmArgs {
    int list;
    int n_static;
    const int* count;
    int g_cap;               // capacity of the row list
    const StageEntry* E;     // non-null: row r reads / writes row E[r].kprev
    const float* X;          // [*][K] input features
    const float* W;          // qvgT [A2][K][3*OUT2] or ipT [K][OUT2]
    int colmode;
    int n_cols;
    int A2;
    float* S;                // [*][A2*3*OUT2]
    float* R;                // [*][OUT2]
};

// One event through the whole path (ssla_step.cu).
struct StepArgs {
    Geo g;
    PartState ps;            // the partition's state
    DevLayer L[8];
    DevHead head;
    float4 ev;               // t, x, y, p
    uint8_t* flag_out;       // SSLA_F_* bits of the event (or null)
    float* pred_out;         // decoded prediction row when the event reached the head (or null)
    unsigned* err;           // status bits of waits that ran out (host-mapped, or null)
};

// Strip exchange (ssla_strip.cu).
struct StripSelectArgs {
    const StageEntry* E[5];
    const int* count;
    int g_cap[5];
    int lo, hi, band;        // own stage-0 rows [lo, hi), band rows
    int has[2];              // neighbour above (rows < lo) / below (rows >= hi)
    int cap;                 // rows per index list
    int* idx;                // [3 lists][4: side*2 + kind][cap] entry indices, stream order
    int* cnt;                // [3][4]
    unsigned* err;
};

struct StripXferArgs {
    float* X;                    // layer-input rows of the stage list
    int C;                       // channels of a row
    const int* idx;              // entry indices (send: mine in the band; receive: foreign)
    const int* cnt;
    int cap;
    float* data;                 // packed rows in the receiver's buffer
    unsigned long long* header;  // receiver's header: [0] sequence, [1 + parity] row count
    int parity;
    unsigned long long seq;
    unsigned* done_ctr;          // export: CTA completion counter
    int wait;                    // import: wait for the sequence (bounded) or expect it
    unsigned long long wait_ns;
    unsigned* err;
};

// One ring's share of a ring drain (ssla_engine_drain_rings): events
// [base, base + n) of the ring, chunk rows [off, off + n).
struct RingTake {
    const float4* events;         // ring slots (pinned host memory, device-mapped)
    unsigned long long mask;      // capacity - 1
    unsigned long long base;      // ring index of the first event taken
    unsigned long long* tail;     // released after the slots are copied
    unsigned long long* done;     // released after flags and prediction rows
    uint8_t* flags;               // [capacity] or null
    float* preds;                 // [capacity][cols] or null
    int off, n;
};

struct RingArgs {
    int P, n_total, cols;
    const RingTake* take;         // [P], device copy
    float4* ev;                   // chunk events (gather output)
    const uint8_t* rflags;        // chunk event flags (scatter input)
    const StageEntry* E4;         // head events of the chunk
    const int* count4;
    int cap4;
    const float* head_dec;        // [cap4][cols]
    unsigned* ctr;                // CTA completion counter, zero between launches
};

void launch_ring_gather(cudaStream_t st, const RingArgs& a);
void launch_ring_scatter(cudaStream_t st, const RingArgs& a);

void launch_band_select(cudaStream_t st, const StripSelectArgs& a);
void launch_mark_foreign(cudaStream_t st, int n, const uint32_t* ev_xy, uint8_t* rflags, int lo, int hi);
void launch_strip_export(cudaStream_t st, const StripXferArgs& a);
void launch_strip_import(cudaStream_t st, const StripXferArgs& a);

// Live loop (ssla_live.cu): a resident cluster fed by a pinned host ring.
struct LiveArgs {
    Geo g;
    PartState ps;
    DevLayer L[8];
    DevHead head;
    const float4* events;                // ring slots (pinned host memory)
    unsigned long long mask;             // capacity - 1
    const unsigned long long* head_idx;  // events published (host)
    unsigned long long* tail;            // events taken (device)
    unsigned long long* done;            // events finished (device)
    uint8_t* flags_out;                  // [capacity] or null
    float* preds_out;                    // [capacity][5+ncls] or null
    const int* stop;                     // non-zero ends the loop
    unsigned long long start;            // index of the first event
    unsigned long long idle_ns;          // leave the loop after this long without an event
    unsigned* err;                       // SSLA_LIVE_* status bits (host-mapped)
    unsigned long long withhold_fin;     // test hook: ring index whose completion message is
                                         // withheld from the head CTA (~0: none)
};

struct CommitArgs {
    Geo g;
    const StageEntry* E4;
    const int* off4;         // [P+1]
    const float* head_dec;
    const float* head_raw;
    const PartState* parts;
};

}  // namespace ssla

namespace ssla {

// Host-side launchers (ssla_kernels.cu).  They only enqueue; the caller
// checks cudaGetLastError().
void launch_prep(cudaStream_t st, const float4* ev, int n, int W0, int H0,
                 uint32_t* ev_xy, uint8_t* rflags);
void launch_prep_records(cudaStream_t st, const void* rec, int n, StageEntry* E2,
                         uint32_t* ev_xy, uint8_t* rflags, float* feat);
void launch_filter(cudaStream_t st, const FilterArgs& a);
// Marks the stage-0 tile-list entries whose event reaches stage 1 (after the gates).
void launch_flag_s0(cudaStream_t st, const FilterArgs& a);
// Programmatic dependent launch: a drain kernel is launched while the
// previous one in the stream completes and waits here for it to complete
// (and its memory to be visible) before touching anything it may write.
// No kernel triggers its dependants early: CTAs of the next kernel waiting
// on the SMs slowed the running one (measured), so the dependant is
// released at completion and only the launch latency overlaps.  Without
// the launch attribute the wait is a no-op.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_enter() { pdl_wait(); }

// Launches a drain kernel with programmatic stream serialization: it may be
// scheduled while the previous kernel of the stream drains, and waits for
// it in pdl_enter / pdl_wait.  Errors surface through cudaGetLastError.
template <typename... P, typename... A>
void pdl_launch(void (*kern)(P...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, A... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, kern, static_cast<P>(args)...);
}

cudaError_t launch_live(cudaStream_t st, const LiveArgs& a);
int live_max_ncls();
cudaError_t launch_step(cudaStream_t st, const StepArgs& a);
// One HybridInputRec (t, s2 x / y, feat1) per stage-2 list entry.
void launch_records(cudaStream_t st, int n_cap, const int* count2, const StageEntry* E2,
                    const float4* ev, const float* feat1, void* rec);
void launch_gates(cudaStream_t st, const GateArgs& a);
void launch_gates_s2(cudaStream_t st, const Gate2Args& a);
void launch_compact(cudaStream_t st, const CompactArgs& a);
void launch_scan(cudaStream_t st, int layer, const ScanArgs& a);
void launch_contrib(cudaStream_t st, int layer, const ContribArgs& a, long long max_rows);
void launch_ln(cudaStream_t st, int layer, const LnArgs& a, long long max_rows);
void launch_scan_fused(cudaStream_t st, int layer, const ScanFusedArgs& a);
void launch_head(cudaStream_t st, const HeadArgs& a, long long max_rows);
// The head's convolutions on tcgen05 tensor cores (split TF32, ssla_head_tc.cu).
void launch_head_tc(cudaStream_t st, const HeadArgs& a, long long max_rows);
// GEMM for next layer `layer` (its IN = K, OUT2, A2) with the given columns.
void launch_gemm(cudaStream_t st, int layer, const GemmArgs& a, long long max_rows);
int gemm_cols(int layer, int colmode);
void launch_commit(cudaStream_t st, const CommitArgs& a);
void launch_reset_preds(cudaStream_t st, const Geo& g, const PartState* parts, const DevHead& hd);
void launch_fill_f64(cudaStream_t st, double* p, size_t n, double v);
void launch_write_slots(cudaStream_t st, int n, int P, const int* rec_off, const uint8_t* rflags,
                        const uint32_t* ev_xy, const PartState* parts, const float* slot_feat,
                        void* const* outs);
void launch_fill_clk(cudaStream_t st, int P, const int* rec_off, const unsigned long long* stamps,
                     unsigned long long* const* clks);
void launch_stamp(cudaStream_t st, unsigned long long* dst);
// Copies a drain's flags and decoded predictions into mapped pinned host
// memory from a kernel (either destination may be null): host pointers as
// their device aliases (cudaHostGetDevicePointer).
void launch_results_to_host(cudaStream_t st, const uint8_t* flags, int n_flags, uint8_t* flags_host,
                            const float* preds, int n_preds, float* preds_host);
// Measured FP32 FMA throughput of the current device, TFLOP/s.
double measure_ffma_peak();
// Mismatches of ssla_rcp_rn against IEEE round-to-nearest over every float
// in [1, 2^126) (the first one's bit pattern in *first_bad, 0xFFFFFFFF if none).
unsigned long long check_reciprocal(unsigned* first_bad);
// ssla_sigmoidf2 against two ssla_sigmoidf over every float (first component
// u in [0, 2^31), second u ^ 2^31); mismatches and the first one's u.
unsigned long long check_sigmoid_pair(unsigned* first_bad);

}  // namespace ssla
