// stability.cu -- the reference's training-stability modes
// (training_stability.h:20-121) as host functions: mode validation, the
// scheduled learning rate, and the init-side modes applied to a flat
// registry-ordered parameter buffer.  The step-side modes (schedules and the
// global-norm gradient clip) run in the LM optimizer step (lm.cu).
#include <algorithm>
#include <cmath>

#include "hx_internal.cuh"

extern "C" {

const char* hx_stability_mode_error(uint32_t mode) {
    // validateTrainingStabilityMode (training_stability.h:77-81)
    if (mode <= 6 && mode != 5) return nullptr;
    if (mode == 5) return "RESIDUAL_BRANCH_SCALING_UNSUPPORTED_ON_DEVICE";
    return "UNKNOWN_TRAINING_STABILITY_MODE";
}

float hx_stability_learning_rate(uint32_t mode, float base, uint32_t step, uint32_t total_steps) {
    // stabilityLearningRate (training_stability.h:88-99): the factor is
    // formed in double and the product rounded once to float.
    if (mode == HX_STABILITY_WARMUP64) {
        const double factor = std::min(1.0, double(step) / 64.0);
        return float(base * factor);
    }
    if (mode == HX_STABILITY_DECAY_LINEAR) {
        const double done = total_steps ? double(total_steps) : 1.0;
        return float(base * (1.0 - double(step - 1) / done));
    }
    return base;
}

int hx_lm_apply_init_stability(const hx_lm_config* cfg, uint32_t mode, float* params) {
    if (!cfg || !params) return HX_ERR_ARGUMENT;
    if (hx_stability_mode_error(mode)) return HX_ERR_UNSUPPORTED;
    if (mode != HX_STABILITY_ZERO_OUTPUT_PROJ_BRANCH_INIT && mode != HX_STABILITY_DEPTH_SCALED_BRANCH_INIT)
        return HX_OK;
    // applyInitStability (training_stability.h:104-121) over the registry
    // layout: token_embedding [V*D], (position_embedding [T*D]), per layer
    // g1 b1 [D], wq wk wv wo [D*D], g2 b2 [D], w1 [D*F], w2 [F*D], output.
    const size_t V = cfg->vocab, T = cfg->tokens, D = cfg->dim, F = cfg->ffn;
    size_t off = V * D + ((cfg->flags & HX_LM_LEARNED_POSITION) ? T * D : 0);
    const float s = 1.0f / std::sqrt(2.0f * float(cfg->layers));
    for (uint32_t l = 0; l < cfg->layers; ++l) {
        const size_t wo = off + 2 * D + 3 * D * D;
        const size_t w1 = off + 4 * D + 4 * D * D;
        const size_t w2 = w1 + D * F;
        if (mode == HX_STABILITY_ZERO_OUTPUT_PROJ_BRANCH_INIT) {
            std::fill(params + wo, params + wo + D * D, 0.0f);
            std::fill(params + w2, params + w2 + F * D, 0.0f);
        } else {
            for (size_t i = 0; i < D * D; ++i) params[wo + i] *= s;
            for (size_t i = 0; i < D * F; ++i) params[w1 + i] *= s;
            for (size_t i = 0; i < F * D; ++i) params[w2 + i] *= s;
        }
        off = w2 + F * D;
    }
    return HX_OK;
}

}  // extern "C"
