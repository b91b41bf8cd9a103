// ref_adapter.cpp -- C-ABI glue over the reference's own CPU code.
//
// TEST INFRASTRUCTURE ONLY.  oracle/Makefile compiles this file together with
// the reference's unmodified app/src/main/cpp/cpu_reference_training.cpp and
// app/src/main/cpp/tiny_language_model_cpu.cpp (read where they lie in the
// HexaTrain tree) into oracle/_ref/libhexaref.so.  Tests use it to pin the C
// restatement in hx_oracle.c, tests/golden/make_golden.py uses it to write
// the committed fixtures, and bench.py's reference arm times it.  The product
// never loads it.
//
// Only glue lives here: flat float buffers in registry order are converted
// to/from the reference's parameter structs, and token ids to its one-hot
// rows.  All arithmetic is the reference's.
#include "cpu_reference_training.h"
#include "tiny_language_model_cpu.h"
#include "training_stability.h"
#include "nicopedia_generation.h"

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <exception>
#include <string>
#include <thread>
#include <vector>

namespace {

using phonelm::cpu::Matrix;
using Params = phonelm::qnn::TinyTransformerParameters;
using LayerParams = phonelm::qnn::TinyTransformerLayerParameters;

struct RefConfig {  // mirrors hxo_lm_config (oracle/hx_oracle.h)
    uint32_t vocab, tokens, dim, ffn, layers, heads;
    float eps;
    int learned_position;
};

phonelm::tiny_lm::Config toConfig(const RefConfig* c) {
    phonelm::tiny_lm::Config r;
    r.vocabularySize = c->vocab;
    r.tokens = c->tokens;
    r.dimension = c->dim;
    r.feedForwardDimension = c->ffn;
    r.epsilon = c->eps;
    r.numLayers = c->layers;
    r.numHeads = c->heads;
    return r;
}

std::vector<std::vector<float>*> layerFields(LayerParams& l) {
    return {&l.gamma1, &l.beta1, &l.wq, &l.wk, &l.wv, &l.wo, &l.gamma2, &l.beta2, &l.w1, &l.w2};
}

// Registry order (tiny_language_model_cpu.cpp parameterRegistry).
std::vector<std::vector<float>*> registryFields(Params& p) {
    std::vector<std::vector<float>*> r{&p.tokenEmbedding};
    for (auto* f : layerFields(p)) r.push_back(f);
    for (auto& l : p.layers)
        for (auto* f : layerFields(l)) r.push_back(f);
    r.push_back(&p.outputProjection);
    return r;
}

std::vector<size_t> registrySizes(const RefConfig* c) {
    const size_t V = c->vocab, D = c->dim, F = c->ffn;
    std::vector<size_t> s{V * D};
    for (uint32_t l = 0; l < c->layers; ++l)
        for (size_t n : {D, D, D * D, D * D, D * D, D * D, D, D, D * F, F * D}) s.push_back(n);
    s.push_back(D * V);
    return s;
}

Params unflatten(const RefConfig* c, const float* flat) {
    Params p;
    p.layers.resize(c->layers - 1);
    auto fields = registryFields(p);
    auto sizes = registrySizes(c);
    size_t off = 0;
    for (size_t i = 0; i < fields.size(); ++i) {
        fields[i]->assign(flat + off, flat + off + sizes[i]);
        off += sizes[i];
    }
    return p;
}

void flatten(Params& p, float* out) {
    size_t off = 0;
    for (auto* f : registryFields(p)) {
        std::memcpy(out + off, f->data(), f->size() * sizeof(float));
        off += f->size();
    }
}

int guard(const char* where, std::string* err, const std::exception& e) {
    if (err) *err = std::string(where) + ": " + e.what();
    return -1;
}

thread_local std::string gLastError;

}  // namespace

extern "C" {

const char* hxr_last_error() { return gLastError.c_str(); }

int hxr_param_count(const RefConfig* c) {
    size_t n = 0;
    for (size_t s : registrySizes(c)) n += s;
    return int(n);
}

// cpu::matMul (cpu_reference_training.cpp:129)
void hxr_matmul(int M, int N, int K, const float* lhs, const float* rhs, float* out) {
    const Matrix a(M, K, std::vector<float>(lhs, lhs + size_t(M) * K));
    const Matrix b(K, N, std::vector<float>(rhs, rhs + size_t(K) * N));
    const auto o = phonelm::cpu::matMul(a, b);
    std::memcpy(out, o.values.data(), o.values.size() * sizeof(float));
}

// cpu::forwardBackward (cpu_reference_training.cpp:172) + sgdUpdate.
float hxr_linear_forward_backward(int B, int D, const float* x, const float* target,
                                  const float* w, float lr, float* prediction, float* error,
                                  float* d_prediction, float* d_weight, float* d_input,
                                  float* w_next) {
    const Matrix X(B, D, std::vector<float>(x, x + size_t(B) * D));
    const Matrix Y(B, D, std::vector<float>(target, target + size_t(B) * D));
    Matrix W(D, D, std::vector<float>(w, w + size_t(D) * D));
    const auto r = phonelm::cpu::forwardBackward(X, Y, W);
    std::memcpy(prediction, r.prediction.values.data(), sizeof(float) * size_t(B) * D);
    std::memcpy(error, r.error.values.data(), sizeof(float) * size_t(B) * D);
    std::memcpy(d_prediction, r.dPrediction.values.data(), sizeof(float) * size_t(B) * D);
    std::memcpy(d_weight, r.dWeight.values.data(), sizeof(float) * size_t(D) * D);
    std::memcpy(d_input, r.dInput.values.data(), sizeof(float) * size_t(B) * D);
    if (lr > 0) phonelm::cpu::sgdUpdate(W, r.dWeight, lr);
    std::memcpy(w_next, W.values.data(), sizeof(float) * size_t(D) * D);
    return r.loss;
}

// The MLP driver's pass() (qnn/qnn_mlp_training.cpp:53-72) sits in an
// anonymous namespace of a file that needs the QNN runtime; its sequence of
// reference primitives is replayed here with the reference's own
// cpu::matMul / transpose / meanSquaredError / sgdUpdate.
int hxr_mlp_step(int B, int I, int H, int O, const float* x, const float* y,
                 const float* w1, const float* w2, float lr, float* loss, float* w1_next,
                 float* w2_next, float* z1, float* h, float* p, float* e, float* dp,
                 float* dw2, float* dh, unsigned char* mask, float* dz1, float* dw1) {
    try {
        using namespace phonelm::cpu;
        const Matrix X(B, I, std::vector<float>(x, x + size_t(B) * I));
        const Matrix Y(B, O, std::vector<float>(y, y + size_t(B) * O));
        Matrix W1(I, H, std::vector<float>(w1, w1 + size_t(I) * H));
        Matrix W2(H, O, std::vector<float>(w2, w2 + size_t(H) * O));
        const Matrix Z1 = matMul(X, W1);
        Matrix Hd(B, H);
        for (size_t i = 0; i < Z1.values.size(); ++i) Hd.values[i] = std::max(0.0f, Z1.values[i]);
        const Matrix P = matMul(Hd, W2);
        const float l = meanSquaredError(P, Y);
        Matrix dP(B, O);
        const float s = 2.0f / static_cast<float>(X.rows * Y.columns);
        for (size_t i = 0; i < dP.values.size(); ++i) dP.values[i] = (P.values[i] - Y.values[i]) * s;
        const Matrix dW2 = matMul(transpose(Hd), dP);
        const Matrix dH = matMul(dP, transpose(W2));
        Matrix dZ1(B, H);
        for (size_t i = 0; i < dZ1.values.size(); ++i)
            dZ1.values[i] = Hd.values[i] > 0 ? dH.values[i] : 0;
        const Matrix dW1 = matMul(transpose(X), dZ1);
        sgdUpdate(W1, dW1, lr);
        sgdUpdate(W2, dW2, lr);
        *loss = l;
        auto put = [](float* dst, const Matrix& m) {
            std::memcpy(dst, m.values.data(), m.values.size() * sizeof(float));
        };
        put(w1_next, W1); put(w2_next, W2); put(z1, Z1); put(h, Hd); put(p, P);
        for (size_t i = 0; i < P.values.size(); ++i) e[i] = P.values[i] - Y.values[i];
        put(dp, dP); put(dw2, dW2); put(dh, dH); put(dz1, dZ1); put(dw1, dW1);
        for (size_t i = 0; i < Hd.values.size(); ++i) mask[i] = Hd.values[i] > 0.0f ? 1 : 0;
        return 0;
    } catch (const std::exception& ex) {
        return guard("hxr_mlp_step", &gLastError, ex);
    }
}

// tiny_lm::fixedPosition (tiny_language_model_cpu.cpp:68)
void hxr_lm_fixed_position(const RefConfig* c, float* out) {
    const auto p = phonelm::tiny_lm::fixedPosition(toConfig(c));
    std::memcpy(out, p.data(), p.size() * sizeof(float));
}

// tiny_lm::initialParameters (tiny_language_model_cpu.cpp:69-70), flattened.
int hxr_lm_initial_parameters(const RefConfig* c, uint32_t seed, float* out) {
    try {
        auto p = phonelm::tiny_lm::initialParameters(toConfig(c), seed);
        flatten(p, out);
        return 0;
    } catch (const std::exception& ex) {
        return guard("hxr_lm_initial_parameters", &gLastError, ex);
    }
}

// tiny_lm::validateConfig
int hxr_lm_validate(const RefConfig* c) {
    std::string e;
    const bool ok = phonelm::tiny_lm::validateConfig(toConfig(c), &e);
    gLastError = e;
    return ok ? 0 : -1;
}

// tiny_lm::forwardBackwardGeneralized (tiny_language_model_cpu.cpp:84) on
// one-hot rows built from token ids.  Optional outputs may be NULL.
int hxr_lm_forward_backward(const RefConfig* c, const uint32_t* input_tokens,
                            const uint32_t* target_tokens, const float* params, float lr,
                            float* loss, float* accuracy, float* grads, float* next,
                            float* logits, float* probs, float* dlogits, float* output,
                            float* layer_input_grads, float* head_probs) {
    try {
        const auto cfg = toConfig(c);
        const std::vector<uint32_t> in(input_tokens, input_tokens + c->tokens);
        const std::vector<uint32_t> tg(target_tokens, target_tokens + c->tokens);
        const auto oh = phonelm::tiny_lm::oneHot(in, c->vocab);
        const auto th = phonelm::tiny_lm::oneHot(tg, c->vocab);
        const Params p = unflatten(c, params);
        auto r = phonelm::tiny_lm::forwardBackwardGeneralized(cfg, oh, th, p, lr);
        *loss = r.loss;
        if (accuracy) *accuracy = r.accuracy;
        flatten(r.gradients, grads);
        if (next) flatten(r.next, next);
        auto put = [](float* dst, const std::vector<float>& v) {
            if (dst) std::memcpy(dst, v.data(), v.size() * sizeof(float));
        };
        put(logits, r.logits);
        put(probs, r.probabilities);
        put(dlogits, r.dLogits);
        put(output, r.transformerOutput);
        if (layer_input_grads)
            for (uint32_t l = 0; l < c->layers; ++l)
                std::memcpy(layer_input_grads + size_t(l) * c->tokens * c->dim,
                            r.layerInputGradients[l].data(),
                            sizeof(float) * size_t(c->tokens) * c->dim);
        if (head_probs) {
            const size_t tt = size_t(c->tokens) * c->tokens;
            for (size_t i = 0; i < r.attentionHeadProbabilities.size(); ++i)
                std::memcpy(head_probs + i * tt, r.attentionHeadProbabilities[i].data(),
                            tt * sizeof(float));
        }
        return 0;
    } catch (const std::exception& ex) {
        return guard("hxr_lm_forward_backward", &gLastError, ex);
    }
}

// tiny_lm::momentumUpdate (tiny_language_model_cpu.cpp:123) over flat
// registry-ordered buffers of configuration c.
int hxr_lm_momentum(const RefConfig* c, const float* w, const float* g, const float* v, float lr, float momentum,
                    float* w_next, float* v_next) {
    try {
        const Params W = unflatten(c, w), G = unflatten(c, g), Vv = unflatten(c, v);
        auto r = phonelm::tiny_lm::momentumUpdate(W, G, Vv, lr, momentum);
        flatten(r.next, w_next);
        flatten(r.velocity, v_next);
        return 0;
    } catch (const std::exception& ex) {
        return guard("hxr_lm_momentum", &gLastError, ex);
    }
}

// nicopedia_gen::greedyArgmax / sampleTopKChecked (nicopedia_generation.h:286-395).
uint32_t hxr_sample_next_token(const float* logits, uint32_t vocab, int greedy, float temperature, uint32_t top_k,
                               uint64_t seed, uint64_t step, int* ok) {
    if (greedy) {
        *ok = 1;
        return phonelm::nicopedia_gen::greedyArgmax(logits, vocab);
    }
    const auto r = phonelm::nicopedia_gen::sampleTopKChecked(logits, vocab, temperature, top_k, seed, step);
    *ok = r.ok ? 1 : 0;
    return r.value;
}

// phonelm::stabilityLearningRate (training_stability.h:88-99).
float hxr_stability_learning_rate(uint32_t mode, float base, uint32_t step, uint32_t total) {
    return phonelm::stabilityLearningRate(mode, base, step, total);
}

// phonelm::applyInitStability (training_stability.h:104-121) on flat params.
int hxr_apply_init_stability(const RefConfig* c, uint32_t mode, float* params) {
    try {
        Params p = phonelm::applyInitStability(toConfig(c), unflatten(c, params), mode);
        flatten(p, params);
        return 0;
    } catch (const std::exception& ex) {
        return guard("hxr_apply_init_stability", &gLastError, ex);
    }
}

// phonelm::validateTrainingStabilityMode (training_stability.h:77-81).
const char* hxr_stability_mode_error(uint32_t mode) {
    const char* e = phonelm::validateTrainingStabilityMode(mode);
    return e ? e : "";
}

// tiny_lm::adamUpdate (tiny_language_model_cpu.cpp:124-145) over flat
// registry-ordered buffers of configuration c.
int hxr_lm_adam(const RefConfig* c, const float* w, const float* g, const float* m,
                const float* v, float lr, float beta1, float beta2, float eps, float c1,
                float c2, float* m_next, float* v_next, float* m_hat, float* v_hat,
                float* w_next) {
    try {
        const Params W = unflatten(c, w), G = unflatten(c, g), Mm = unflatten(c, m),
                     Vv = unflatten(c, v);
        auto r = phonelm::tiny_lm::adamUpdate(W, G, Mm, Vv, lr, beta1, beta2, eps, c1, c2);
        flatten(r.firstMoment, m_next);
        flatten(r.secondMoment, v_next);
        if (m_hat) flatten(r.firstMomentHat, m_hat);
        if (v_hat) flatten(r.secondMomentHat, v_hat);
        flatten(r.next, w_next);
        return 0;
    } catch (const std::exception& ex) {
        return guard("hxr_lm_adam", &gLastError, ex);
    }
}

// One batched Adam step as the reference's driver runs it
// (qnn/qnn_transformer_training.cpp:7295-7345 with the CPU twin of
// :7168-7210): B sequences through forwardBackwardGeneralized (lr 0),
// accum += grad*(1/B) in sequence order, then adamUpdate with the driver's
// double-precision bias corrections.  `threads` spreads the independent
// sequences over host threads; the accumulation order is unchanged.
// tokens: [B, T+1].  params/m/v are updated in place.
int hxr_lm_train_step(const RefConfig* c, int B, const uint32_t* tokens, float* params,
                      float* m, float* v, float lr, int step, int threads, float* mean_loss) {
    try {
        const auto cfg = toConfig(c);
        const uint32_t T = c->tokens;
        const Params current = unflatten(c, params);
        std::vector<phonelm::tiny_lm::StepResult> results(B);
        auto work = [&](int first, int stride) {
            for (int b = first; b < B; b += stride) {
                const uint32_t* seq = tokens + size_t(b) * (T + 1);
                const auto oh = phonelm::tiny_lm::oneHot(std::vector<uint32_t>(seq, seq + T), c->vocab);
                const auto th = phonelm::tiny_lm::oneHot(std::vector<uint32_t>(seq + 1, seq + 1 + T), c->vocab);
                results[b] = phonelm::tiny_lm::forwardBackwardGeneralized(cfg, oh, th, current, 0.0f);
            }
        };
        threads = std::max(1, std::min(threads, B));
        std::vector<std::thread> pool;
        for (int t = 1; t < threads; ++t) pool.emplace_back(work, t, threads);
        work(0, threads);
        for (auto& th : pool) th.join();
        Params accum = current;
        for (auto* f : registryFields(accum)) std::fill(f->begin(), f->end(), 0.0f);
        double lossSum = 0;
        for (int b = 0; b < B; ++b) {
            auto acc = registryFields(accum);
            auto grd = registryFields(results[b].gradients);
            for (size_t i = 0; i < acc.size(); ++i)
                for (size_t j = 0; j < acc[i]->size(); ++j)
                    (*acc[i])[j] += (*grd[i])[j] * (1.0f / float(B));
            lossSum += results[b].loss;
        }
        const float c1 = float(1.0 / (1.0 - std::pow(0.9, double(step))));
        const float c2 = float(1.0 / (1.0 - std::pow(0.999, double(step))));
        const Params Mm = unflatten(c, m), Vv = unflatten(c, v);
        auto r = phonelm::tiny_lm::adamUpdate(current, accum, Mm, Vv, lr, .9f, .999f, 1e-8f, c1, c2);
        flatten(r.next, params);
        flatten(r.firstMoment, m);
        flatten(r.secondMoment, v);
        *mean_loss = float(lossSum / B);
        return 0;
    } catch (const std::exception& ex) {
        return guard("hxr_lm_train_step", &gLastError, ex);
    }
}

// tiny_lm::gradientCheck (finite differences on the reference's tiny case)
int hxr_lm_gradient_check(uint32_t seed, float epsilon, float* max_abs, float* max_rel) {
    const auto r = phonelm::tiny_lm::gradientCheck(seed, epsilon);
    *max_abs = r.maximumAbsoluteError;
    *max_rel = r.maximumRelativeError;
    return r.passed ? 1 : 0;
}

}  // extern "C"
