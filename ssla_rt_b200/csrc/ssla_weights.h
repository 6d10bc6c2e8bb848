// ssla_weights.h -- host-side model loading for the B200 engine.
//
// Reads meta.json + weights.npz (uncompressed zip of .npy files, as written
// by numpy.savez), reshapes every SSLA layer into per-position tensors
// (src/ssla_kernels.cpp:73-153) and folds the YOLOX head's BatchNorm into its
// 1x1 convolutions (vendor/openeva/heads/async_yolox.h:98-143), producing the
// device layouts the kernels read:
//   qvgT[A][IN][3*OUT]   (row j = part*OUT + o, part 0 q, 1 v, 2 g)
//   goWT[A][OUT][OUT]    (goWT[p][i][o] = goW[p][o][i])
//   ipT[IN][OUT]         (input_proj transposed), gamma[OUT], beta[OUT]
//   head: *_convT[C_in][C_hid], *_predT[C_hid][n], biases
// These are the layouts of the reference's GPU buffers
// (orin/orin/hybrid_common.py:192-199, :386-400).
#pragma once

#include <cstdint>
#include <map>
#include <string>
#include <vector>

namespace ssla {

struct NpyArray {
    std::vector<std::size_t> shape;
    std::vector<float> data;
};

struct Meta {
    std::string model;
    int height = 0, width = 0, num_classes = 0, tdrop_window = 0;
};

// Throws std::runtime_error with a message on any format problem.
Meta read_meta(const std::string& dir);
std::map<std::string, NpyArray> read_npz(const std::string& path);

struct HostLayer {
    int in_dim = 0, out_dim = 0, A = 1;
    std::vector<float> qvgT, goWT, ipT, gamma, beta;   // ipT empty if none
};

struct HostHead {
    int c_in = 96, c_hid = 96, ncls = 2;
    std::vector<float> cls_convT, cls_conv_b, reg_convT, reg_conv_b;
    std::vector<float> cls_predT, cls_pred_b, reg_predT, reg_pred_b;
    std::vector<float> obj_predT, obj_pred_b;
};

struct HostModel {
    Meta meta;
    HostLayer layers[8];
    HostHead head;
};

HostModel load_model(const std::string& dir);

}  // namespace ssla
