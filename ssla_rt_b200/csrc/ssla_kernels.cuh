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
};

struct GateArgs {
    Geo g;
    const float4* ev;
    const int* ev_off;       // [P+1]
    const int2* tl0;         // stage-0 tile lists (tile = s3 block)
    const int* tl0_cnt;
    const PartState* parts;
    uint8_t* rflags;
    float* S0;               // L0 (q, v, sigmoid(g)) per event  [N][36]
    float* R0;               // L0 residual per event            [N][12]
    DevLayer L0;
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

// k_event modes: what produces x (the event's feature) and what follows.
enum {
    MODE_FIRST = 0,   // gather layer 2s -> qvg of layer 2s+1 (same events)
    MODE_SECOND = 1,  // gather layer 2s+1 -> qvg of layer 2s+2 (next stage)
    MODE_HEAD = 2,    // gather layer 7 -> YOLOX head
    MODE_LAST = 3,    // gather layer 7 only (drain_n: no head)
    MODE_ENTRY = 4    // x = stage-1 feature of a record -> qvg of layer 4
};

struct EventArgs {
    Geo g;
    int stage;               // stage of the gathered layer
    int mode;                // MODE_* below
    int n_static;            // stage-0 first layer: list length (all events)
    const int* count;        // device list lengths (index: list id)
    int list;                // list id for count[] (1..4); 0 = all events
    const StageEntry* E;     // iterated list (mode 1/2 and stage >= 1)
    const uint32_t* ev_xy;
    const uint8_t* rflags;
    uint8_t needq_bit;       // mode 0: reach bit of "next layer output needed"
    const float* S_in;
    const float* R_in;
    float* S_out;
    float* R_out;
    DevLayer L;              // gathered layer (goWT, gamma, beta)
    DevLayer N;              // next layer (qvgT, ipT)
    DevHead head;
    float* stage_out;        // optional [N][OUT] per chunk event
    float* head_dec;         // mode 2: [cap4][5+ncls]
    float* head_raw;
    // drain_n (stage-2 entry) path, optional
    const float* entry_feat; // mode 4: [N][24] stage-1 features of the records
    float* slot_feat;        // [N][96] the reference's s3_feat slot contents
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
void launch_filter(cudaStream_t st, const FilterArgs& a, dim3 grid);
void launch_gates(cudaStream_t st, const GateArgs& a);
void launch_gates_s2(cudaStream_t st, const Gate2Args& a);
void launch_compact(cudaStream_t st, const CompactArgs& a);
void launch_scan(cudaStream_t st, int layer, const ScanArgs& a);
void launch_event(cudaStream_t st, int layer, int mode, const EventArgs& a, int grid);
void launch_commit(cudaStream_t st, const CommitArgs& a);
void launch_reset_preds(cudaStream_t st, const Geo& g, const PartState* parts, const DevHead& hd);
void launch_fill_f64(cudaStream_t st, double* p, size_t n, double v);
void launch_write_slots(cudaStream_t st, int n, int P, const int* rec_off, const uint8_t* rflags,
                        const uint32_t* ev_xy, const PartState* parts, const float* slot_feat,
                        void* const* outs);
void launch_fill_clk(cudaStream_t st, int P, const int* rec_off, const unsigned long long* stamps,
                     unsigned long long* const* clks);
void launch_stamp(cudaStream_t st, unsigned long long* dst);
// Measured FP32 FMA throughput of the current device, TFLOP/s.
double measure_ffma_peak();

}  // namespace ssla
