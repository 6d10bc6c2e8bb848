// Prediction-tensor checkpoint dumps in the reference's OracleRecorder file
// format (include/oracle.h:10-19, written by OracleRecorder::save, :57-74):
//
//   uint32 magic = 0x4F455641 ('OEVA'), uint32 version = 1,
//   uint32 num_anchors, uint32 cols (= 5 + num_classes),
//   uint32 num_checkpoints, then per checkpoint
//   uint64 event_idx, float[num_anchors * cols] decoded predictions,
//
// little-endian.  A checkpoint is taken after event i of the recorded
// stream when i % every == 0 (OracleRecorder::record, :43-54), so the
// reference's diff_dumps / oracle_diff (src/oracle_diff.cpp) compares a dump
// of this engine with a dump of any reference scheme directly.
#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <string>
#include <vector>

#include "ssla_b200.h"

namespace ssla {
void set_last_error(const std::string& msg);   // ssla_engine.cu
}

namespace {

bool write_all(std::FILE* f, const void* p, size_t n) { return std::fwrite(p, 1, n, f) == n; }

}  // namespace

extern "C" {

int ssla_write_oracle_dump(const char* path, int num_anchors, int cols, int n_checkpoints,
                           const uint64_t* event_idx, const float* preds) {
    if (!path || num_anchors <= 0 || cols <= 0 || n_checkpoints < 0 ||
        (n_checkpoints > 0 && (!event_idx || !preds))) {
        ssla::set_last_error("oracle dump: bad argument");
        return SSLA_ERR_ARG;
    }
    std::FILE* f = std::fopen(path, "wb");
    if (!f) {
        ssla::set_last_error(std::string("oracle dump: cannot open ") + path);
        return SSLA_ERR_ARG;
    }
    const uint32_t head[5] = {0x4F455641u, 1u, static_cast<uint32_t>(num_anchors), static_cast<uint32_t>(cols),
                              static_cast<uint32_t>(n_checkpoints)};
    bool ok = write_all(f, head, sizeof head);
    const size_t per = static_cast<size_t>(num_anchors) * cols;
    for (int i = 0; ok && i < n_checkpoints; ++i) {
        ok = write_all(f, event_idx + i, 8) && write_all(f, preds + per * i, per * sizeof(float));
    }
    ok = (std::fclose(f) == 0) && ok;
    if (!ok) ssla::set_last_error(std::string("oracle dump: write failed: ") + path);
    return ok ? SSLA_OK : SSLA_ERR_ARG;
}

int ssla_engine_oracle_dump(SslaEngine* eng, int partition, const float* events_host, int n, int every,
                            const char* path) {
    if (!eng || (!events_host && n > 0) || n < 0 || every <= 0 || !path) {
        ssla::set_last_error("oracle dump: bad argument");
        return SSLA_ERR_ARG;
    }
    SslaEngineInfo info{};
    int rc = ssla_engine_info(eng, &info);
    if (rc != SSLA_OK) return rc;
    if (partition < 0 || partition >= info.n_partitions) {
        ssla::set_last_error("oracle dump: partition out of range");
        return SSLA_ERR_ARG;
    }
    const int anchors = (info.H >> 3) * (info.W >> 3);
    const int cols = 5 + info.ncls;
    const size_t per = static_cast<size_t>(anchors) * cols;
    std::vector<uint64_t> idx;
    std::vector<float> preds;
    std::vector<int> off(info.n_partitions + 1, 0);
    const int cap = std::max(1, info.max_events / info.n_partitions);   // within any partition's capacity
    // drains end exactly after the checkpoint events 0, every, 2*every, ...
    int start = 0;
    while (start < n) {
        const int cp = start == 0 ? 0 : ((start - 1) / every + 1) * every;     // next checkpoint >= start
        const int end = std::min(n, std::min(cp + 1, start + cap));
        for (int p = 0; p <= info.n_partitions; ++p) off[p] = p <= partition ? 0 : end - start;
        rc = ssla_engine_drain_host(eng, events_host + 4 * static_cast<size_t>(start), off.data(), nullptr, nullptr);
        if (rc != SSLA_OK) return rc;
        if (end == cp + 1) {
            idx.push_back(static_cast<uint64_t>(cp));
            preds.resize(per * idx.size());
            rc = ssla_engine_read_state(eng, SSLA_STATE_PREDS_DEC, partition, 0, preds.data() + per * (idx.size() - 1),
                                        per * sizeof(float));
            if (rc != SSLA_OK) return rc;
        }
        start = end;
    }
    return ssla_write_oracle_dump(path, anchors, cols, static_cast<int>(idx.size()), idx.data(), preds.data());
}

}  // extern "C"
