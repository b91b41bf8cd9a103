// qnn_runtime_hexatrain.cpp -- phonelm::qnn::Runtime over libhexatrain_b200.
//
// The reference selects its Runtime implementation at link time
// (app/src/main/cpp/CMakeLists.txt:86-99: qnn_runtime_qairt.cpp with the
// QAIRT SDK, qnn_runtime_stub.cpp without).  This file is a third choice: the
// same class, declared by the reference's own header qnn/qnn_runtime.h
// (:250-451), implemented on the C ABI of include/hexatrain.h, so that the
// reference's drivers (TrainingEngine::run and the experiment runners it
// dispatches to) train on a B200 without any other change.  A maintainer
// compiles it in place of qnn_runtime_stub.cpp and links
// libhexatrain_b200.so; runtime_adapter/Makefile is the recipe.
//
// Served on the GPU (the training-step hot path):
//   initialize, prepare/executeMlpFullStep, prepare/executeTinyTransformer-
//   Training (generalized graph, FULL variant, no taps),
//   executeTinyTransformerForwardOnly (FORWARD_ONLY variant),
//   prepare/executeAdamOptimizer, prepare/executeMomentumOptimizer.
// Every other graph of the reference (per-op diagnostic graphs, the legacy
// MLP split graphs, single-op checks) answers like the stub runtime:
// false with "QNN_DISABLED: <graph> unavailable ..." -- they are outside the
// hot path.  Failure injection follows RuntimeOptions as the QAIRT runtime
// does (failGraphExecuteAt, failGraphFinalize; qnn_runtime_full_step.inc:
// 309-320, 378-399).  The CUDA device is HEXATRAIN_CUDA_DEVICE (default 0).
#include "qnn_runtime.h"

#include <chrono>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <sstream>

#include "hexatrain.h"

namespace phonelm::qnn {

namespace {
using Clock = std::chrono::steady_clock;
double us_since(Clock::time_point t0) {
    return std::chrono::duration<double, std::micro>(Clock::now() - t0).count();
}
const char* yes(bool b) { return b ? "true" : "false"; }
}  // namespace

const char* backendKindName(QnnBackendKind kind) {
    switch (kind) {
        case QnnBackendKind::CPU: return "CPU";
        case QnnBackendKind::HTP: return "HTP";
    }
    return "UNKNOWN";
}

struct Runtime::Impl {
    hx_runtime* rt = nullptr;
    // prepared MLP full step
    uint32_t B = 0, I = 0, H = 0, O = 0;
    bool mlp_diag = false, mlp_ready = false;
    // prepared generalized LM graph
    hx_lm_config lm{};
    bool lm_diag = false, lm_ready = false, lm_forward_only = false;
    size_t lm_params = 0;
    uint32_t adam_n = 0, momentum_n = 0;
    uint64_t execute_calls = 0;
    ~Impl() {
        if (rt) hx_runtime_destroy(rt);
    }
    std::string last() const { return rt ? hx_runtime_last_error(rt) : "runtime not initialized"; }
};

Runtime::Runtime() : info_(queryBackendInfo()), impl_(new Impl) {}
Runtime::~Runtime() { delete impl_; }

const BackendInfo& Runtime::info() const { return info_; }
const std::string& Runtime::diagnostics() const { return diagnostics_; }
const RuntimeMetrics& Runtime::metrics() const { return metrics_; }
const ApiTrace& Runtime::apiTrace() const { return apiTrace_; }
std::uint32_t Runtime::tinyTransformerTrainingSourceTensorCreateSuccessCount() const { return 0; }
std::uint32_t Runtime::tinyTransformerTrainingSourceGraphAddNodeSuccessCount() const { return 0; }
std::uint32_t Runtime::tinyTransformerTrainingLastInputTensorCount() const {
    return impl_->lm_ready ? 3 + 10 * impl_->lm.layers : 0;  // one-hot, target, E, 10 per layer, head
}
std::uint32_t Runtime::tinyTransformerTrainingLastOutputTensorCount() const { return 0; }
bool Runtime::tinyTransformerTrainingLastLearningRateBytesUnchanged() const { return true; }
void Runtime::setOptions(const RuntimeOptions& options) { options_ = options; }

std::string Runtime::apiTraceSummary() const {
    const auto& t = apiTrace_;
    std::ostringstream s;
    s << "api_trace_version=1\n"
      << "api_trace_backend_requested=" << t.backendRequested << '\n'
      << "api_trace_backend_library=" << t.backendLibrary << '\n'
      << "api_trace_backend_library_load_result=" << t.backendLibraryLoadResult << '\n'
      << "api_trace_backend_create_called=" << yes(t.backendCreateCalled) << '\n'
      << "api_trace_backend_create_result=" << t.backendCreateResult << '\n'
      << "api_trace_full_step_graph_create_called=" << yes(t.fullStepGraphCreateCalled) << '\n'
      << "api_trace_full_step_graph_create_result=" << t.fullStepGraphCreateResult << '\n'
      << "api_trace_full_step_graph_finalize_called=" << yes(t.fullStepGraphFinalizeCalled) << '\n'
      << "api_trace_full_step_graph_finalize_result=" << t.fullStepGraphFinalizeResult << '\n'
      << "api_trace_graph_execute_attempt_count=" << t.graphExecuteAttemptCount << '\n'
      << "api_trace_graph_execute_success_count=" << t.graphExecuteSuccessCount << '\n'
      << "api_trace_graph_execute_failure_count=" << t.graphExecuteFailureCount << '\n'
      << "api_trace_graph_execute_first_failure_call=" << t.graphExecuteFirstFailureCall << '\n'
      << "api_trace_failure_injection_enabled=" << yes(t.failureInjectionEnabled) << '\n'
      << "api_trace_failure_injection_point=" << t.failureInjectionPoint << '\n'
      << "api_trace_failure_injection_call=" << t.failureInjectionCall << '\n'
      << "api_trace_effective_result=" << t.effectiveResult << '\n'
      << "api_trace_fallback_attempted=" << yes(t.fallbackAttempted) << '\n';
    return s.str();
}

std::string Runtime::qnnCallbackCaptureSummary() const { return "qnn_callback_capture_enabled=false\n"; }

void Runtime::recordGraphExecuteResult(int qnnResult, int effectiveResult, bool success) {
    auto& t = apiTrace_;
    const auto call = static_cast<std::int64_t>(t.graphExecuteAttemptCount);
    ++t.graphExecuteAttemptCount;
    if (t.graphExecuteFirstCallIndex < 0) {
        t.graphExecuteFirstCallIndex = call;
        t.graphExecuteFirstResult = effectiveResult;
    }
    t.graphExecuteLastCallIndex = call;
    t.graphExecuteLastResult = effectiveResult;
    t.lastQnnResult = qnnResult;
    t.effectiveResult = effectiveResult;
    if (success) {
        ++t.graphExecuteSuccessCount;
    } else {
        ++t.graphExecuteFailureCount;
        if (t.graphExecuteFirstFailureCall < 0) t.graphExecuteFirstFailureCall = call;
    }
}

bool Runtime::initialize(QnnBackendKind requestedBackend, std::string& error) {
    apiTrace_.backendRequested = backendKindName(requestedBackend);
    apiTrace_.backendLibrary = "libhexatrain_b200.so";
    apiTrace_.backendCreateCalled = true;
    const char* dev = std::getenv("HEXATRAIN_CUDA_DEVICE");
    const int device = dev ? std::atoi(dev) : 0;
    const auto t0 = Clock::now();
    char err[512] = {0};
    if (impl_->rt) {
        hx_runtime_destroy(impl_->rt);
        impl_->rt = nullptr;
    }
    const int rc = hx_runtime_create(device, &impl_->rt, err, sizeof err);
    metrics_.backendCreateUs = us_since(t0);
    apiTrace_.backendLibraryLoadResult = 0;
    apiTrace_.backendCreateResult = rc;
    apiTrace_.backendHandleNonnull = impl_->rt != nullptr;
    if (rc != HX_OK) {
        error = err;
        return false;
    }
    diagnostics_ = "runtime=hexatrain_b200\ncuda_device=" + std::to_string(device) + "\n";
    return true;
}

bool Runtime::recreateContext(std::string& error) {
    error = "QNN_DISABLED: context recreation unavailable on the CUDA runtime";
    return false;
}

// ---- graphs outside the training-step hot path --------------------------------
namespace {
bool disabled(std::string& e, const char* what) {
    e = std::string("QNN_DISABLED: ") + what + " unavailable on the CUDA runtime (outside the training-step path)";
    return false;
}
}  // namespace

bool Runtime::prepareMatMul(uint32_t, uint32_t, uint32_t, bool, std::string& e) { return disabled(e, "MatMul"); }
bool Runtime::executeMatMul(const std::vector<float>&, const std::vector<float>&, std::vector<float>&,
                            std::string& e) { return disabled(e, "MatMul"); }
bool Runtime::setInitialWeight(const std::vector<float>&, std::string& e) { return disabled(e, "weight binding"); }
bool Runtime::updateWeight(const std::vector<float>&, std::string& e) { return disabled(e, "weight update"); }
bool Runtime::executePrepared(const std::vector<float>&, std::vector<float>&, std::string& e) {
    return disabled(e, "MatMul");
}
bool Runtime::prepareDWeightMatMul(uint32_t, uint32_t, uint32_t, std::string& e) { return disabled(e, "dW MatMul"); }
bool Runtime::executeDWeight(const std::vector<float>&, const std::vector<float>&, std::vector<float>&,
                             std::string& e) { return disabled(e, "dW MatMul"); }
bool Runtime::prepareInputGradientMatMul(uint32_t, uint32_t, uint32_t, std::string& e) { return disabled(e, "dX"); }
bool Runtime::executeInputGradient(const std::vector<float>&, const std::vector<float>&, std::vector<float>&,
                                   std::string& e) { return disabled(e, "dX"); }
bool Runtime::prepareMlp(uint32_t, uint32_t, uint32_t, uint32_t, std::string& e, bool) { return disabled(e, "MLP"); }
bool Runtime::prepareReluBackward(uint32_t, uint32_t, std::string& e) { return disabled(e, "ReLU backward"); }
bool Runtime::executeReluBackward(const std::vector<float>&, const std::vector<float>&, std::vector<std::uint8_t>&,
                                  std::vector<float>&, std::string& e) { return disabled(e, "ReLU backward"); }
bool Runtime::prepareMlpFusedBackward(bool, std::string& e) { return disabled(e, "fused backward"); }
bool Runtime::executeMlpFusedBackward(const std::vector<float>&, const std::vector<float>&, const std::vector<float>&,
                                      std::vector<float>&, std::vector<float>&, std::vector<std::uint8_t>&,
                                      std::vector<float>&, std::vector<float>&, std::string& e) {
    return disabled(e, "fused backward");
}
bool Runtime::setMlpWeights(const std::vector<float>&, const std::vector<float>&, std::string& e) {
    return disabled(e, "MLP");
}
bool Runtime::executeMlpForward(const std::vector<float>&, std::vector<float>&, std::vector<float>&,
                                std::string& e) { return disabled(e, "MLP"); }
bool Runtime::executeMlpSecondBackward(const std::vector<float>&, const std::vector<float>&, std::vector<float>&,
                                       std::vector<float>&, std::string& e) { return disabled(e, "MLP"); }
bool Runtime::executeMlpFirstBackward(const std::vector<float>&, const std::vector<float>&, std::vector<float>&,
                                      std::string& e) { return disabled(e, "MLP"); }
bool Runtime::prepareTrainingOpsMicro(uint32_t, uint32_t, uint32_t, uint32_t, std::string& e) {
    return disabled(e, "training ops micro");
}
bool Runtime::executeTrainingOpsMicro(const std::vector<float>&, const std::vector<float>&, const std::vector<float>&,
                                      const std::vector<float>&, float, float&, std::vector<float>&,
                                      std::vector<float>&, std::string& e) { return disabled(e, "training ops micro"); }
bool Runtime::prepareLayerNorm(uint32_t, uint32_t, uint32_t, float, std::string& e) { return disabled(e, "LayerNorm"); }
bool Runtime::executeLayerNorm(const std::vector<float>&, std::vector<float>&, std::string& e) {
    return disabled(e, "LayerNorm");
}
bool Runtime::prepareElementwiseSquare(uint32_t, std::string& e) { return disabled(e, "elementwise square"); }
bool Runtime::executeElementwiseSquare(const std::vector<float>&, std::vector<float>&, std::string& e) {
    return disabled(e, "elementwise square");
}
bool Runtime::prepareLayerNormBackward(uint32_t, uint32_t, float, std::string& e) {
    return disabled(e, "LayerNorm backward");
}
bool Runtime::executeLayerNormBackward(const std::vector<float>&, const std::vector<float>&, const std::vector<float>&,
                                       const std::vector<float>&, LayerNormBackwardOutputs&, std::string& e) {
    return disabled(e, "LayerNorm backward");
}
bool Runtime::prepareSoftmax(uint32_t, uint32_t, std::string& e) { return disabled(e, "Softmax"); }
bool Runtime::executeSoftmax(const std::vector<float>&, std::vector<float>&, std::string& e) {
    return disabled(e, "Softmax");
}
bool Runtime::prepareSoftmaxBackward(uint32_t, uint32_t, std::string& e) { return disabled(e, "Softmax backward"); }
bool Runtime::executeSoftmaxBackward(const std::vector<float>&, const std::vector<float>&, std::vector<float>&,
                                     std::string& e) { return disabled(e, "Softmax backward"); }
bool Runtime::prepareCrossEntropyGradient(uint32_t, uint32_t, std::string& e) {
    return disabled(e, "cross entropy gradient");
}
bool Runtime::executeCrossEntropyGradient(const std::vector<float>&, const std::vector<float>&,
                                          CrossEntropyGradientOutputs&, std::string& e) {
    return disabled(e, "cross entropy gradient");
}
bool Runtime::prepareAttention(uint32_t, uint32_t, std::string& e) { return disabled(e, "attention"); }
bool Runtime::executeAttention(const std::vector<float>&, const std::vector<float>&, const std::vector<float>&,
                               const std::vector<float>&, std::vector<float>&, std::vector<float>&, std::string& e) {
    return disabled(e, "attention");
}
bool Runtime::prepareAttentionBackward(uint32_t, uint32_t, std::string& e) { return disabled(e, "attention backward"); }
bool Runtime::executeAttentionBackward(const std::vector<float>&, const std::vector<float>&, const std::vector<float>&,
                                       const std::vector<float>&, const std::vector<float>&,
                                       AttentionBackwardOutputs&, std::string& e) {
    return disabled(e, "attention backward");
}
bool Runtime::prepareTinyTransformer(uint32_t, uint32_t, uint32_t, float, std::string& e) {
    return disabled(e, "tiny transformer forward graph");
}
bool Runtime::executeTinyTransformer(const std::vector<float>&, std::vector<float>&, std::string& e) {
    return disabled(e, "tiny transformer forward graph");
}

// ---- the MLP full step (qnn_runtime_full_step.inc:209-400) --------------------

bool Runtime::prepareMlpFullStep(uint32_t batchSize, uint32_t inputDimension, uint32_t hiddenDimension,
                                 uint32_t outputDimension, bool diagnosticOutputs, std::string& e) {
    Impl& im = *impl_;
    if (!im.rt) {
        e = "full step invalid runtime or shape";
        return false;
    }
    const auto t0 = Clock::now();
    apiTrace_.fullStepGraphCreateCalled = true;
    const int rc = hx_mlp_prepare(im.rt, batchSize, inputDimension, hiddenDimension, outputDimension,
                                  diagnosticOutputs ? 1 : 0);
    apiTrace_.fullStepGraphCreateResult = rc;
    apiTrace_.fullStepGraphHandleNonnull = rc == HX_OK;
    metrics_.graphCreateUs += us_since(t0);
    if (rc != HX_OK) {
        e = im.last();
        return false;
    }
    ++metrics_.graphCreateCount;
    // The step's CUDA graph is captured on first use; "finalize" is the
    // prepare's success here.
    apiTrace_.fullStepGraphFinalizeCalled = true;
    apiTrace_.fullStepGraphFinalizeResult = 0;
    ++metrics_.graphFinalizeCount;
    if (options_.failGraphFinalize) {
        apiTrace_.failureInjectionEnabled = true;
        apiTrace_.failureInjectionPoint = "graphFinalize";
        apiTrace_.failureInjectionCall = 0;
        apiTrace_.lastQnnResult = 0;
        apiTrace_.effectiveResult = -9002;
        e = "injected graphFinalize failure after QNN success";
        return false;
    }
    im.B = batchSize; im.I = inputDimension; im.H = hiddenDimension; im.O = outputDimension;
    im.mlp_diag = diagnosticOutputs;
    im.mlp_ready = true;
    return true;
}

bool Runtime::executeMlpFullStep(const std::vector<float>& input, const std::vector<float>& target,
                                 const std::vector<float>& w1Current, const std::vector<float>& w2Current,
                                 float learningRate, MlpFullStepOutputs& out, std::string& e) {
    Impl& im = *impl_;
    if (!im.rt || !im.mlp_ready) {
        e = "full step graph not prepared";
        return false;
    }
    const size_t B = im.B, I = im.I, H = im.H, O = im.O;
    out.w1Next.resize(I * H);
    out.w2Next.resize(H * O);
    hx_mlp_outputs o{};
    o.loss = &out.loss;
    o.w1_next = out.w1Next.data();
    o.w2_next = out.w2Next.data();
    if (im.mlp_diag) {
        out.prediction.resize(B * O); out.error.resize(B * O); out.dPrediction.resize(B * O);
        out.dW2.resize(H * O); out.dHidden.resize(B * H); out.mask.resize(B * H); out.dZ1.resize(B * H);
        out.dW1.resize(I * H); out.hidden.resize(B * H);
        o.prediction = out.prediction.data(); o.error = out.error.data(); o.d_prediction = out.dPrediction.data();
        o.d_w2 = out.dW2.data(); o.d_hidden = out.dHidden.data(); o.mask = out.mask.data();
        o.d_z1 = out.dZ1.data(); o.d_w1 = out.dW1.data(); o.hidden = out.hidden.data();
    }
    const auto callIndex = apiTrace_.graphExecuteAttemptCount;
    const auto t0 = Clock::now();
    const int rc = hx_mlp_execute(im.rt, input.data(), input.size(), target.data(), target.size(), w1Current.data(),
                                  w1Current.size(), w2Current.data(), w2Current.size(), learningRate, &o);
    metrics_.executeUs.push_back(us_since(t0));
    ++metrics_.graphExecuteCount;
    hx_metrics m{};
    hx_runtime_metrics(im.rt, &m);
    metrics_.inputBindUs.push_back(m.last_input_bind_us);
    metrics_.outputBindUs.push_back(m.last_output_bind_us);
    const bool injected =
        rc == HX_OK && options_.failGraphExecuteAt >= 0 && callIndex == std::uint64_t(options_.failGraphExecuteAt);
    if (injected) {
        apiTrace_.failureInjectionEnabled = true;
        apiTrace_.failureInjectionPoint = "graphExecute";
        apiTrace_.failureInjectionCall = std::int64_t(callIndex);
    }
    recordGraphExecuteResult(rc, injected ? -9001 : rc, rc == HX_OK && !injected);
    if (injected) {
        e = "injected graphExecute failure after QNN success";
        return false;
    }
    if (rc != HX_OK) {
        e = im.last().find("buffer size mismatch") != std::string::npos
                ? im.last()
                : "full step graphExecute=" + std::to_string(rc) + ": " + im.last();
        return false;
    }
    return true;
}

// ---- optimizer graphs (qnn_runtime_transformer.inc:799-1218) ----------------

bool Runtime::prepareAdamOptimizer(uint32_t elements, std::string& e) {
    Impl& im = *impl_;
    if (!im.rt || hx_adam_prepare(im.rt, elements) != HX_OK) {
        e = im.rt ? im.last() : "Adam optimizer invalid runtime or shape";
        return false;
    }
    im.adam_n = elements;
    ++metrics_.graphCreateCount;
    ++metrics_.graphFinalizeCount;
    return true;
}

bool Runtime::executeAdamOptimizer(const std::vector<float>& current, const std::vector<float>& gradient,
                                   const std::vector<float>& firstMoment, const std::vector<float>& secondMoment,
                                   float learningRate, float gradientScale, float firstCorrection,
                                   float secondCorrection, AdamOptimizerOutputs& out, std::string& e) {
    Impl& im = *impl_;
    const size_t n = im.adam_n;
    if (!im.rt || !n || current.size() != n || gradient.size() != n || firstMoment.size() != n ||
        secondMoment.size() != n) {
        e = "Adam optimizer buffer size or scalar";
        return false;
    }
    for (auto* v : {&out.firstMomentNext, &out.secondMomentNext, &out.firstMomentHat, &out.secondMomentHat,
                    &out.secondRoot, &out.denominator, &out.dividedUpdate, &out.normalizedUpdate,
                    &out.scaledUpdate, &out.weightNext})
        v->resize(n);
    hx_adam_outputs o{out.firstMomentNext.data(), out.secondMomentNext.data(), out.firstMomentHat.data(),
                      out.secondMomentHat.data(), out.secondRoot.data(), out.denominator.data(),
                      out.dividedUpdate.data(), out.normalizedUpdate.data(), out.scaledUpdate.data(),
                      out.weightNext.data()};
    const auto t0 = Clock::now();
    const int rc = hx_adam_execute(im.rt, current.data(), gradient.data(), firstMoment.data(), secondMoment.data(),
                                   learningRate, gradientScale, firstCorrection, secondCorrection, &o);
    metrics_.executeUs.push_back(us_since(t0));
    ++metrics_.graphExecuteCount;
    recordGraphExecuteResult(rc, rc, rc == HX_OK);
    if (rc != HX_OK) {
        e = im.last();
        return false;
    }
    return true;
}

bool Runtime::prepareMomentumOptimizer(uint32_t elements, std::string& e) {
    Impl& im = *impl_;
    if (!im.rt || hx_momentum_prepare(im.rt, elements) != HX_OK) {
        e = im.rt ? im.last() : "momentum optimizer invalid runtime or shape";
        return false;
    }
    im.momentum_n = elements;
    ++metrics_.graphCreateCount;
    ++metrics_.graphFinalizeCount;
    return true;
}

bool Runtime::executeMomentumOptimizer(const std::vector<float>& current, const std::vector<float>& gradient,
                                       const std::vector<float>& velocity, float learningRate, float momentum,
                                       MomentumOptimizerOutputs& out, std::string& e) {
    Impl& im = *impl_;
    const size_t n = im.momentum_n;
    if (!im.rt || !n || current.size() != n || gradient.size() != n || velocity.size() != n) {
        e = "momentum optimizer buffer size or scalar";
        return false;
    }
    out.velocityNext.resize(n);
    out.weightNext.resize(n);
    const auto t0 = Clock::now();
    const int rc = hx_momentum_execute(im.rt, current.data(), gradient.data(), velocity.data(), learningRate, momentum,
                                       out.velocityNext.data(), out.weightNext.data());
    metrics_.executeUs.push_back(us_since(t0));
    ++metrics_.graphExecuteCount;
    recordGraphExecuteResult(rc, rc, rc == HX_OK);
    if (rc != HX_OK) {
        e = im.last();
        return false;
    }
    return true;
}

// ---- the generalized L-layer / H-head LM graph --------------------------------
// (qnn_runtime_transformer_training_generalized.inc, its execute companion)

namespace {
// Registry order of the flat parameter buffer (qnn_transformer_training.cpp:
// 1164-1180): token embedding, layer 0 (the base struct), layers[0..],
// output projection.
std::vector<TinyTransformerLayerParameters*> layer_list(TinyTransformerParameters& p) {
    std::vector<TinyTransformerLayerParameters*> v{&p};
    for (auto& l : p.layers) v.push_back(&l);
    return v;
}
template <class F>
void for_each_tensor(TinyTransformerParameters& p, F&& f) {
    f(p.tokenEmbedding);
    for (TinyTransformerLayerParameters* l : layer_list(p))
        for (std::vector<float>* t : {&l->gamma1, &l->beta1, &l->wq, &l->wk, &l->wv, &l->wo, &l->gamma2, &l->beta2,
                                      &l->w1, &l->w2})
            f(*t);
    f(p.outputProjection);
}
bool flatten(const TinyTransformerParameters& p, size_t count, std::vector<float>& flat) {
    flat.clear();
    flat.reserve(count);
    for_each_tensor(const_cast<TinyTransformerParameters&>(p),
                    [&](std::vector<float>& t) { flat.insert(flat.end(), t.begin(), t.end()); });
    return flat.size() == count;
}
void unflatten(const std::vector<float>& flat, TinyTransformerParameters& p) {
    size_t off = 0;
    for_each_tensor(p, [&](std::vector<float>& t) {
        std::copy(flat.begin() + long(off), flat.begin() + long(off + t.size()), t.begin());
        off += t.size();
    });
}
}  // namespace

bool Runtime::prepareTinyTransformerTraining(uint32_t tokens, uint32_t dimension, uint32_t feedForwardDimension,
                                             float epsilon, bool diagnosticOutputs, std::string& e,
                                             uint32_t vocabularySize, TinyTransformerTrainingVariant variant,
                                             TinyTransformerTrainingTapSet tapSet, uint32_t numLayers,
                                             uint32_t numHeads) {
    return prepareTinyTransformerTrainingGeneralized(tokens, dimension, feedForwardDimension, epsilon,
                                                     diagnosticOutputs, e, vocabularySize, variant, tapSet,
                                                     numLayers, numHeads);
}

bool Runtime::prepareTinyTransformerTrainingGeneralized(uint32_t tokens, uint32_t dimension,
                                                        uint32_t feedForwardDimension, float epsilon,
                                                        bool diagnosticOutputs, std::string& e,
                                                        uint32_t vocabularySize,
                                                        TinyTransformerTrainingVariant variant,
                                                        TinyTransformerTrainingTapSet tapSet, uint32_t numLayers,
                                                        uint32_t numHeads) {
    Impl& im = *impl_;
    if (!im.rt) {
        e = "generalized tiny training invalid runtime";
        return false;
    }
    if (vocabularySize == 0) return disabled(e, "vocabulary-free tiny transformer training graph");
    if (tapSet != TinyTransformerTrainingTapSet::NONE) return disabled(e, "graph tap sets");
    if (variant == TinyTransformerTrainingVariant::STOP_AFTER_DINPUT ||
        variant == TinyTransformerTrainingVariant::STOP_AFTER_DEMBEDDING)
        return disabled(e, "truncated tiny transformer training graphs");
    hx_lm_config c{vocabularySize, tokens, dimension, feedForwardDimension, numLayers, numHeads, epsilon, 0u};
    const auto t0 = Clock::now();
    const bool forward_only = variant == TinyTransformerTrainingVariant::FORWARD_ONLY;
    if (hx_lm_prepare(im.rt, &c, 1, (diagnosticOutputs && !forward_only) ? 1 : 0) != HX_OK) {
        e = im.last();
        return false;
    }
    metrics_.graphCreateUs += us_since(t0);
    ++metrics_.graphCreateCount;
    ++metrics_.graphFinalizeCount;
    im.lm = c;
    im.lm_diag = diagnosticOutputs && !forward_only;
    im.lm_forward_only = forward_only;
    im.lm_params = hx_lm_param_count(&c);
    im.lm_ready = true;
    return true;
}

bool Runtime::executeTinyTransformerTraining(const std::vector<float>& input, const std::vector<float>& target,
                                             const TinyTransformerParameters& current, float learningRate,
                                             TinyTransformerTrainingOutputs& outputs, std::string& e) {
    return executeTinyTransformerTrainingGeneralized(input, target, current, learningRate, outputs, e);
}

bool Runtime::executeTinyTransformerTrainingGeneralized(const std::vector<float>& input,
                                                        const std::vector<float>& target,
                                                        const TinyTransformerParameters& current,
                                                        float learningRate, TinyTransformerTrainingOutputs& outputs,
                                                        std::string& e) {
    Impl& im = *impl_;
    if (!im.rt || !im.lm_ready || im.lm_forward_only) {
        e = "generalized tiny training graph not prepared";
        return false;
    }
    const hx_lm_config& c = im.lm;
    const size_t T = c.tokens, V = c.vocab, D = c.dim, L = c.layers, H = c.heads;
    std::vector<float> flat;
    if (input.size() != T * V || target.size() != T * V || !flatten(current, im.lm_params, flat)) {
        e = "generalized tiny training buffer schema";
        return false;
    }
    std::vector<float> grads(im.lm_params), lig, hp;
    hx_lm_outputs o{};
    o.loss = &outputs.loss;
    o.grads = grads.data();
    outputs.logits.clear(); outputs.probabilities.clear(); outputs.dLogits.clear();
    outputs.output.clear(); outputs.dOutput.clear();
    if (im.lm_diag) {
        outputs.logits.resize(T * V);
        outputs.probabilities.resize(T * V);
        outputs.dLogits.resize(T * V);
        outputs.output.resize(T * D);
        outputs.dOutput.resize(T * D);
        lig.resize(L * T * D);
        hp.resize(L * H * T * T);
        o.logits = outputs.logits.data();
        o.probabilities = outputs.probabilities.data();
        o.d_logits = outputs.dLogits.data();
        o.output = outputs.output.data();
        o.d_output = outputs.dOutput.data();
        o.layer_input_grads = lig.data();
        o.head_probabilities = hp.data();
    }
    const auto callIndex = apiTrace_.graphExecuteAttemptCount;
    const auto t0 = Clock::now();
    const int rc = hx_lm_execute(im.rt, input.data(), target.data(), flat.data(), flat.size(), learningRate, &o);
    metrics_.executeUs.push_back(us_since(t0));
    ++metrics_.graphExecuteCount;
    const bool injected =
        rc == HX_OK && options_.failGraphExecuteAt >= 0 && callIndex == std::uint64_t(options_.failGraphExecuteAt);
    recordGraphExecuteResult(rc, injected ? -9001 : rc, rc == HX_OK && !injected);
    if (injected) {
        apiTrace_.failureInjectionEnabled = true;
        apiTrace_.failureInjectionPoint = "graphExecute";
        apiTrace_.failureInjectionCall = std::int64_t(callIndex);
        e = "injected graphExecute failure after QNN success";
        return false;
    }
    if (rc != HX_OK) {
        e = im.last();
        return false;
    }
    // The generalized execute's results (..._generalized_execute.inc:193-239):
    // gradients in the parameters' shapes, per-layer input gradients, the
    // per-head attention probabilities as taps when H > 1, no SGD "next"
    // (the graph stops at gradients) and no embedded-input terminal.
    outputs.taps.clear();
    outputs.next = {};
    outputs.gradients = current;
    unflatten(grads, outputs.gradients);
    outputs.layerInputGradients.clear();
    outputs.embeddedInput.clear();
    outputs.dEmbeddedInput.clear();
    if (im.lm_diag) {
        for (size_t l = 0; l < L; ++l)
            outputs.layerInputGradients.emplace_back(lig.begin() + long(l * T * D), lig.begin() + long((l + 1) * T * D));
        if (H > 1)
            for (size_t l = 0; l < L; ++l)
                for (size_t h = 0; h < H; ++h) {
                    char name[64];
                    std::snprintf(name, sizeof name, "layer_%03zu_head_%03zu_probabilities", l, h);
                    const auto b = hp.begin() + long((l * H + h) * T * T);
                    outputs.taps.push_back({name, std::vector<float>(b, b + long(T * T))});
                }
        outputs.dEmbeddedInput = outputs.layerInputGradients.front();
    }
    return true;
}

bool Runtime::executeTinyTransformerForwardOnly(const std::vector<float>& input,
                                                const TinyTransformerParameters& current,
                                                TinyTransformerTrainingOutputs& outputs, std::string& e) {
    Impl& im = *impl_;
    if (!im.rt || !im.lm_ready) {
        e = "generalized tiny training forward-only graph not prepared";
        return false;
    }
    const hx_lm_config& c = im.lm;
    const size_t T = c.tokens, V = c.vocab;
    std::vector<float> flat;
    if (input.size() != T * V || !flatten(current, im.lm_params, flat)) {
        e = "generalized tiny training forward-only buffer schema";
        return false;
    }
    // one-hot rows to ids; a row that is not exactly one-hot is rejected
    std::vector<uint32_t> ids(T);
    for (size_t t = 0; t < T; ++t) {
        int hot = -1;
        for (size_t v = 0; v < V; ++v) {
            const float x = input[t * V + v];
            if (x == 1.0f && hot < 0) hot = int(v);
            else if (x != 0.0f) hot = -2;
        }
        if (hot < 0) {
            e = "INVALID_TINY_LM_ONE_HOT: every input row must hold exactly one 1.0 and zeros elsewhere";
            return false;
        }
        ids[t] = uint32_t(hot);
    }
    outputs.logits.resize(T * V);
    const auto t0 = Clock::now();
    const int rc = hx_lm_forward_tokens(im.rt, ids.data(), flat.data(), flat.size(), outputs.logits.data());
    metrics_.executeUs.push_back(us_since(t0));
    ++metrics_.graphExecuteCount;
    recordGraphExecuteResult(rc, rc, rc == HX_OK);
    if (rc != HX_OK) {
        e = im.last();
        return false;
    }
    outputs.taps.clear();
    outputs.next = {};
    outputs.output.clear(); outputs.dOutput.clear(); outputs.dEmbeddedInput.clear();
    outputs.embeddedInput.clear(); outputs.layerInputGradients.clear();
    outputs.probabilities.clear(); outputs.dLogits.clear();
    return true;
}

}  // namespace phonelm::qnn
