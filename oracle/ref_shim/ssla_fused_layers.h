#pragma once
// TEST INFRASTRUCTURE ONLY -- x86 stand-in for the reference's NEON-only
// include/ssla_fused_layers.h, so that the reference's src/ssla_kernels.cpp
// compiles on x86 as the oracle/_ref build (oracle/Makefile puts this
// directory ahead of the reference's include/ on the include path).
//
// The reference header compiles to nothing off ARM (its #if at :23), which
// leaves the six deploy::fused::* calls in src/ssla_kernels.cpp:756-861
// undeclared.  This file declares the same six entry points with the same
// signatures and computes them with the reference's own generic primitives
// (openeva::prim::matvec_ct / lru_step / matvec_accum_ct / add_inplace /
// layernorm_ct), i.e. exactly the math of the generic layer_forward_ct
// (src/ssla_kernels.cpp:315-385) for an interior event: patch order
// delta = 8..0, residual add, fp64 LayerNorm.  The NEON originals differ
// only by their Pade sigmoid and fp32 LayerNorm, which are ARM-only.

#include <array>
#include <cstring>
#include <vector>

#include "openeva/prim/elementwise.h"
#include "openeva/prim/layernorm.h"
#include "openeva/prim/linear.h"
#include "openeva/prim/rnn.h"

namespace deploy {
namespace fused {
namespace shim {

// One interior event through a K=3 layer. W_T selects the goW_T
// (input-major) weight layout that the tiled s1 entry points receive.
template <int IN, int OUT, bool W_T, bool STATE_ONLY>
inline void interior_layer(int ev_x, int ev_y, int Wl, const float* feat_in,
                           const float* input_proj,
                           const std::array<std::vector<float>, 9>& qvg,
                           const std::array<std::vector<float>, 9>* gow,
                           const float* gamma, const float* beta,
                           float* H_all, float* feat_out) {
    float residual[OUT];
    float q_v_g[3 * OUT];
    float qh[OUT];
    if (!STATE_ONLY) {
        if (input_proj) {
            openeva::prim::matvec_ct<IN, OUT>(feat_in, input_proj, nullptr, residual);
        } else {
            std::memcpy(residual, feat_in, sizeof(float) * OUT);
        }
        std::memset(feat_out, 0, sizeof(float) * OUT);
    }
    const int base = ev_y * Wl + ev_x;
    for (int dy = -1; dy <= 1; ++dy) {
        for (int dx = -1; dx <= 1; ++dx) {
            const int pos = (1 - dy) * 3 + (1 - dx);
            openeva::prim::matvec_ct<IN, 3 * OUT>(feat_in, qvg[pos].data(), nullptr, q_v_g);
            float* h = H_all + static_cast<std::ptrdiff_t>(base + dy * Wl + dx) * OUT;
            openeva::prim::lru_step<OUT>(q_v_g + 2 * OUT, q_v_g + OUT, q_v_g, h, qh);
            if (STATE_ONLY) continue;
            const float* w = (*gow)[pos].data();
            if (W_T) {
                // goW_T[i*OUT + o] == goW[o*OUT + i]; same accumulation as
                // matvec_accum_ct (linear.h:92-101).
                for (int o = 0; o < OUT; ++o) {
                    float acc = 0.0f;
                    for (int i = 0; i < OUT; ++i) acc += w[i * OUT + o] * qh[i];
                    feat_out[o] += acc;
                }
            } else {
                openeva::prim::matvec_accum_ct<OUT, OUT>(qh, w, feat_out);
            }
        }
    }
    if (!STATE_ONLY) {
        openeva::prim::add_inplace(OUT, feat_out, residual);
        openeva::prim::layernorm_ct<OUT>(feat_out, gamma, beta);
    }
}

}  // namespace shim

// s0 L0 <2,12>, K=1: single cell at the event.
static inline void s0_l0_interior(int ev_x, int ev_y, int Wl,
                                  const float* feat_in, const float* input_proj,
                                  const float* qvgIn0, const float* goW0,
                                  const float* ln_gamma, const float* ln_beta,
                                  float* H_all, float* feat_out) {
    float residual[12], q_v_g[36], qh[12];
    if (input_proj) {
        openeva::prim::matvec_ct<2, 12>(feat_in, input_proj, nullptr, residual);
    } else {
        std::memcpy(residual, feat_in, sizeof(float) * 2);
    }
    std::memset(feat_out, 0, sizeof(float) * 12);
    openeva::prim::matvec_ct<2, 36>(feat_in, qvgIn0, nullptr, q_v_g);
    float* h = H_all + static_cast<std::ptrdiff_t>(ev_y * Wl + ev_x) * 12;
    openeva::prim::lru_step<12>(q_v_g + 24, q_v_g + 12, q_v_g, h, qh);
    openeva::prim::matvec_accum_ct<12, 12>(qh, goW0, feat_out);
    openeva::prim::add_inplace(12, feat_out, residual);
    openeva::prim::layernorm_ct<12>(feat_out, ln_gamma, ln_beta);
}

static inline void s0_l1_interior(int ev_x, int ev_y, int Wl, const float* feat_in,
                                  const std::array<std::vector<float>, 9>& qvgIn_arr,
                                  const std::array<std::vector<float>, 9>& goW_arr,
                                  const float* ln_gamma, const float* ln_beta,
                                  float* H_all, float* feat_out) {
    shim::interior_layer<12, 12, false, false>(ev_x, ev_y, Wl, feat_in, nullptr,
                                               qvgIn_arr, &goW_arr, ln_gamma,
                                               ln_beta, H_all, feat_out);
}

static inline void s0_l1_interior_state_only(int ev_x, int ev_y, int Wl,
                                             const float* feat_in,
                                             const std::array<std::vector<float>, 9>& qvgIn_arr,
                                             float* H_all) {
    shim::interior_layer<12, 12, false, true>(ev_x, ev_y, Wl, feat_in, nullptr,
                                              qvgIn_arr, nullptr, nullptr,
                                              nullptr, H_all, nullptr);
}

static inline void s1_l0_interior_tiled(int ev_x, int ev_y, int Wl,
                                        const float* feat_in,
                                        const float* input_proj,
                                        const std::array<std::vector<float>, 9>& qvgIn_arr,
                                        const std::array<std::vector<float>, 9>& goW_T_arr,
                                        const float* ln_gamma, const float* ln_beta,
                                        float* H_all, float* feat_out) {
    shim::interior_layer<12, 24, true, false>(ev_x, ev_y, Wl, feat_in, input_proj,
                                              qvgIn_arr, &goW_T_arr, ln_gamma,
                                              ln_beta, H_all, feat_out);
}

static inline void s1_l1_interior_tiled(int ev_x, int ev_y, int Wl,
                                        const float* feat_in,
                                        const std::array<std::vector<float>, 9>& qvgIn_arr,
                                        const std::array<std::vector<float>, 9>& goW_T_arr,
                                        const float* ln_gamma, const float* ln_beta,
                                        float* H_all, float* feat_out) {
    shim::interior_layer<24, 24, true, false>(ev_x, ev_y, Wl, feat_in, nullptr,
                                              qvgIn_arr, &goW_T_arr, ln_gamma,
                                              ln_beta, H_all, feat_out);
}

static inline void s1_l1_interior_tiled_state_only(int ev_x, int ev_y, int Wl,
                                                   const float* feat_in,
                                                   const std::array<std::vector<float>, 9>& qvgIn_arr,
                                                   float* H_all) {
    shim::interior_layer<24, 24, true, true>(ev_x, ev_y, Wl, feat_in, nullptr,
                                             qvgIn_arr, nullptr, nullptr,
                                             nullptr, H_all, nullptr);
}

}  // namespace fused
}  // namespace deploy
