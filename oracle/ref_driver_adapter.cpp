// ref_driver_adapter.cpp -- runs the reference's own experiment drivers on
// this repository's Runtime adapter.
//
// TEST INFRASTRUCTURE ONLY (the checker).  oracle/Makefile compiles the
// reference's driver sources where they lie in the HexaTrain tree
// (qnn/qnn_mlp_training.cpp with trainFullStep, qnn/qnn_transformer_training.cpp
// with languageModelAdam, training_engine.cpp, ...) together with
// hexatrain_b200/runtime_adapter/qnn_runtime_hexatrain.cpp in place of the
// reference's qnn_runtime_stub.cpp / qnn_runtime_qairt.cpp, and links
// libhexatrain_b200.so.  The drivers then run unchanged: they prepare and
// execute their graphs on the B200 through the adapter and gate the results
// against their own CPU code, and their KEY=VALUE report comes back here.
//
// The MNN experiment runner (mnn_training_test.cpp) needs the MNN library,
// which is absent; training_engine.cpp refers to four of its functions, so
// this file defines them for the link.  The driver modes run here never
// reach them.
#include <atomic>
#include <cstdio>
#include <cstring>
#include <string>

#include "qnn/qnn_mlp_training.h"
#include "qnn/qnn_transformer.h"
#include "training_engine.h"

namespace phonelm {
const char* backendName(BackendKind) { return "MNN_UNAVAILABLE"; }
bool validateTrainingConfig(const TrainingConfig&, std::string& error) {
    error = "MNN experiment runner not built (MNN library absent)";
    return false;
}
TrainingOutcome runMnnTraining(const TrainingConfig&, std::atomic_bool&, const LogSink&) { return TrainingOutcome{}; }
std::string mnnEnvironmentReport() { return "mnn_available=false\n"; }
}  // namespace phonelm

extern "C" {

// Runs execution mode `mode` of the reference's drivers with the given
// TrainingConfig fields; writes the report (truncated to cap) and returns its
// full length.  MLP modes (26-36) go to runMlpExperiment, LM modes (44-102)
// to runTinyTransformerTrainingExperiment -- what TrainingEngine::run
// dispatches to for those modes.
long hxd_run_mode(int mode, int batch, int dimension, int hidden, int output, int steps, int epochs,
                  int sample_count, int measured_steps, int correctness_interval, float learning_rate,
                  unsigned long long seed, int benchmark, int feed_forward, char* report, size_t cap)
{
    phonelm::TrainingConfig c;
    c.batchSize = batch;
    c.dimension = dimension;
    c.hiddenDimension = hidden;
    c.outputDimension = output;
    c.feedForwardDimension = feed_forward;
    c.steps = steps;
    c.epochs = epochs;
    c.sampleCount = sample_count;
    c.measuredSteps = measured_steps;
    c.correctnessInterval = correctness_interval;
    c.learningRate = learning_rate;
    c.seed = seed;
    c.benchmarkMode = benchmark != 0;
    std::atomic_bool stop{false};
    const auto m = static_cast<phonelm::ExecutionMode>(mode);
    std::string r;
    if (mode >= 26 && mode <= 36)
        r = phonelm::qnn::runMlpExperiment(m, c, stop, phonelm::LogSink{});
    else if (mode >= 44 && mode <= 102)
        r = phonelm::qnn::runTinyTransformerTrainingExperiment(m, c, phonelm::LogSink{}, &stop);
    else
        r = "status=FAILED\nerror=mode not routed by this harness\n";
    if (report && cap) std::snprintf(report, cap, "%s", r.c_str());
    return long(r.size());
}

}  // extern "C"
