// ref_ckpt_adapter.cpp -- C entry points over the reference's own NPRTCKPT
// codec, for the checkpoint parity tests.
//
// TEST INFRASTRUCTURE ONLY (the checker).  The reference keeps its writer
// (nprtSaveCheckpointV2, qnn/qnn_transformer_training.cpp:5171-5252), reader
// (nprtLoadCheckpointForGeneration, :5390-5522), parameter hash
// (nprtParameterHash, :5080-5090), training order (nprtTrainingOrder,
// :4983-4995) and gradient norm (gradientNorm, :920-938) in an anonymous namespace of that driver source.  This file
// includes the source as it lies in the HexaTrain tree (oracle/Makefile
// points the include path there), so those functions are reachable from
// this one translation unit; nothing of the reference is copied here.
#include "qnn/qnn_transformer_training.cpp"

#include <cstring>

namespace {

using phonelm::qnn::TinyTransformerParameters;
namespace tl = phonelm::tiny_lm;

tl::Config make_config(uint32_t V, uint32_t T, uint32_t D, uint32_t F, uint32_t L, uint32_t H) {
    tl::Config c;
    c.vocabularySize = V;
    c.tokens = T;
    c.dimension = D;
    c.feedForwardDimension = F;
    c.numLayers = L;
    c.numHeads = H;
    return c;
}

// Parameters of the reference layout filled from a flat registry-ordered
// buffer (shapes from initialParameters, values overwritten).
TinyTransformerParameters from_flat(const tl::Config& c, const float* flat) {
    TinyTransformerParameters p = tl::initialParameters(c, 1);
    size_t off = 0;
    for (const auto& info : tl::parameterRegistry(p)) {
        auto& values = *const_cast<std::vector<float>*>(info.values);
        std::memcpy(values.data(), flat + off, values.size() * sizeof(float));
        off += values.size();
    }
    return p;
}

void to_flat(const TinyTransformerParameters& p, float* flat) {
    size_t off = 0;
    for (const auto& info : tl::parameterRegistry(p)) {
        std::memcpy(flat + off, info.values->data(), info.values->size() * sizeof(float));
        off += info.values->size();
    }
}

void set_error(char* err, size_t cap, const char* msg) {
    if (err && cap) std::snprintf(err, cap, "%s", msg);
}

}  // namespace

extern "C" {

int hxr_nprt_save(const char* path, uint32_t V, uint32_t T, uint32_t D, uint32_t F, uint32_t L, uint32_t H,
                  uint32_t seed, uint32_t step, const float* params, const float* m, const float* v,
                  const char* kind, const char* hash) {
    try {
        const auto c = make_config(V, T, D, F, L, H);
        return phonelm::qnn::nprtSaveCheckpointV2(path, c, seed, step, from_flat(c, params), from_flat(c, m),
                                                  from_flat(c, v), kind ? kind : "", hash ? hash : "")
                   ? 1
                   : 0;
    } catch (...) {
        return -1;
    }
}

// Returns 1 on success (then fills the outputs), 0 with the reference's
// error code in err.
int hxr_nprt_load(const char* path, uint32_t V, uint32_t T, uint32_t D, uint32_t F, uint32_t L, uint32_t H,
                  uint32_t seed, const char* tokenizer_hash, uint32_t* step, uint32_t* version, int* finite,
                  int* has_adam, float* params, float* m, float* v, char* param_hash, size_t hash_cap, char* err,
                  size_t err_cap) {
    try {
        const auto c = make_config(V, T, D, F, L, H);
        const auto loaded =
            phonelm::qnn::nprtLoadCheckpointForGeneration(path, c, seed, tokenizer_hash ? tokenizer_hash : "");
        *step = loaded.step;
        *version = loaded.v3 ? 3 : loaded.v2 ? 2 : 1;
        *finite = loaded.finite ? 1 : 0;
        *has_adam = loaded.hasAdam ? 1 : 0;
        if (params) to_flat(loaded.parameters, params);
        size_t off = 0;
        for (const auto& e : loaded.adamFirst) {
            if (m) std::memcpy(m + off, e.second.data(), e.second.size() * sizeof(float));
            off += e.second.size();
        }
        off = 0;
        for (const auto& e : loaded.adamSecond) {
            if (v) std::memcpy(v + off, e.second.data(), e.second.size() * sizeof(float));
            off += e.second.size();
        }
        if (param_hash && hash_cap) std::snprintf(param_hash, hash_cap, "%s", loaded.parameterHash.c_str());
        set_error(err, err_cap, "");
        return 1;
    } catch (const std::exception& e) {
        set_error(err, err_cap, e.what());
        return 0;
    }
}

int hxr_nprt_parameter_hash(uint32_t V, uint32_t T, uint32_t D, uint32_t F, uint32_t L, uint32_t H,
                            const float* params, char* out, size_t cap) {
    try {
        const auto c = make_config(V, T, D, F, L, H);
        std::snprintf(out, cap, "%s", phonelm::qnn::nprtParameterHash(from_flat(c, params)).c_str());
        return 1;
    } catch (...) {
        return 0;
    }
}

// gradientNorm (qnn_transformer_training.cpp:920-938) of a flat
// registry-ordered gradient buffer.
double hxr_gradient_norm(uint32_t V, uint32_t T, uint32_t D, uint32_t F, uint32_t L, uint32_t H,
                         const float* grads) {
    try {
        const auto c = make_config(V, T, D, F, L, H);
        return phonelm::qnn::gradientNorm(from_flat(c, grads));
    } catch (...) {
        return -1.0;
    }
}

int hxr_nprt_training_order(uint64_t records, uint32_t steps, uint32_t batch, uint64_t* out) {
    try {
        const auto order = phonelm::qnn::nprtTrainingOrder(records, steps, batch);
        for (size_t i = 0; i < order.size(); ++i) out[i] = order[i];
        return 1;
    } catch (...) {
        return 0;
    }
}

int hxr_nprt_checkpoint_name(uint32_t seed, uint32_t layers, uint32_t T, uint32_t D, uint32_t F, uint32_t step,
                             char* out, size_t cap) {
    std::snprintf(out, cap, "%s", phonelm::qnn::nprtCheckpointName(seed, layers, T, D, F, step).c_str());
    return 1;
}

}  // extern "C"
