// bridge.cu -- the JNI-free core of the host-app bridge
// (include/hexatrain_bridge.h): the reference's NativeBridge entry points
// (app/src/main/cpp/native_bridge.cpp) over this library's C ABI, with its
// KEY=VALUE reports.  Host code only; every step runs through hx_*.
//
// Data is the library's seeded synthetic set (the generators of
// hexatrain_b200/data.py, restated here so a run is reproducible from any
// host): MLP X, Y ~ U(-1,1), W1 ~ U(+-1/sqrt(I)), W2 ~ U(+-1/sqrt(H)) from a
// counter-based splitmix64 stream; LM token ids ~ Zipf(1.1) by inverse CDF,
// step s of seed k drawing from stream k*1000003 + s.
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdio>
#include <mutex>
#include <sstream>
#include <string>
#include <vector>

#include "../../include/hexatrain.h"
#include "../../include/hexatrain_bridge.h"

namespace {

constexpr uint64_t kGolden = 0x9E3779B97F4A7C15ull;

uint64_t splitmix(uint64_t x) {
    x += kGolden;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

// Word i of stream (seed, tag): key = splitmix(seed ^ splitmix(tag)).
uint64_t stream_word(uint64_t seed, uint64_t tag, uint64_t i) {
    return splitmix(splitmix(seed ^ splitmix(tag)) + i * kGolden);
}

void uniform(uint64_t seed, uint64_t tag, size_t n, double lo, double hi, std::vector<float>& out) {
    out.resize(n);
    for (size_t i = 0; i < n; ++i) {
        const double u = double(stream_word(seed, tag, i) >> 40) * (1.0 / double(1 << 24));
        out[i] = float(lo + (hi - lo) * u);
    }
}

void zipf(uint64_t seed, size_t n, uint32_t vocab, double s, std::vector<uint32_t>& out) {
    std::vector<double> cdf(vocab);
    double acc = 0.0;
    for (uint32_t k = 0; k < vocab; ++k) {
        acc += std::pow(double(k + 1), -s);
        cdf[k] = acc;
    }
    for (double& c : cdf) c /= acc;
    out.resize(n);
    for (size_t i = 0; i < n; ++i) {
        const double u = double(stream_word(seed, 7, i) >> 11) * (1.0 / 9007199254740992.0);
        const size_t id = size_t(std::upper_bound(cdf.begin(), cdf.end(), u) - cdf.begin());
        out[i] = uint32_t(std::min<size_t>(id, vocab - 1));
    }
}

std::atomic<bool> g_running{false};
std::atomic<bool> g_stop{false};
thread_local std::string g_report;

const char* keep(std::string s) {
    g_report = std::move(s);
    return g_report.c_str();
}

const char* mode_name(int mode) {
    switch (mode) {
        case 32: return "QNN_HTP_MLP_FULL_STEP";
        case 33: return "QNN_HTP_MLP_FULL_STEP_BENCHMARK";
        case 35: return "QNN_HTP_MLP_FULL_STEP_FAIL_EXECUTE";
        case 99: return "QNN_HTP_TINY_LANGUAGE_MODEL_GENERIC";
    }
    return "UNSUPPORTED";
}

struct Stats {
    std::vector<double> v;
    void emit(std::ostringstream& s, const char* name) const {
        if (v.empty()) return;
        std::vector<double> w = v;
        std::sort(w.begin(), w.end());
        double sum = 0;
        for (double x : w) sum += x;
        s << '\n' << name << "_count=" << w.size() << '\n' << name << "_mean_us=" << sum / w.size() << '\n' << name
          << "_p50_us=" << w[w.size() / 2] << '\n' << name << "_max_us=" << w.back();
    }
};

void progress(const hx_bridge_run* r, const std::string& line) {
    if (r->progress) r->progress(r->progress_context, line.c_str());
}

struct Runtime {
    hx_runtime* rt = nullptr;
    ~Runtime() { if (rt) hx_runtime_destroy(rt); }
};

std::string failed(const char* head, const hx_bridge_run* r, const char* api, const std::string& error) {
    std::ostringstream s;
    s << head << "\nexecution_mode=" << mode_name(r->execution_mode) << "\nstatus=FAILED\nfailed_api=" << api
      << "\nerror=" << error << "\ncpu_fallback=false\nbackend=CUDA_B200\n";
    return s.str();
}

// Mean squared error of the whole sample set under (w1, w2), on the device:
// one full step over every sample with learning rate 0.
bool full_loss(hx_runtime* rt, const std::vector<float>& x, const std::vector<float>& y, const std::vector<float>& w1,
               const std::vector<float>& w2, float* loss) {
    std::vector<float> n1(w1.size()), n2(w2.size());
    hx_mlp_outputs o{};
    o.loss = loss;
    o.w1_next = n1.data();
    o.w2_next = n2.data();
    return hx_mlp_execute(rt, x.data(), x.size(), y.data(), y.size(), w1.data(), w1.size(), w2.data(), w2.size(),
                          0.0f, &o) == HX_OK;
}

std::string run_mlp(const hx_bridge_run* r) {
    const char* head = "MLP_FULL_STEP";
    const int B = r->batch_size, I = r->dimension, H = r->hidden_dimension, O = r->output_dimension;
    const int N = r->sample_count;
    if (B <= 0 || I <= 0 || H <= 0 || O <= 0 || N < B)
        return failed(head, r, "configuration", "invalid MLP shape or sample count");
    const int steps = r->epochs > 0 ? (N / B) * r->epochs : r->steps;
    const uint64_t seed = uint64_t(r->seed);
    std::vector<float> x, y, w1, w2;
    uniform(seed, 1, size_t(N) * I, -1.0, 1.0, x);
    uniform(seed, 2, size_t(N) * O, -1.0, 1.0, y);
    const double a1 = 1.0 / std::sqrt(double(I)), a2 = 1.0 / std::sqrt(double(H));
    uniform(seed, 3, size_t(I) * H, -a1, a1, w1);
    uniform(seed, 4, size_t(H) * O, -a2, a2, w2);

    Runtime train, eval;
    char msg[512] = {};
    if (hx_runtime_create(0, &train.rt, msg, sizeof msg) != HX_OK) return failed(head, r, "runtime_create", msg);
    if (hx_runtime_create(0, &eval.rt, msg, sizeof msg) != HX_OK) return failed(head, r, "runtime_create", msg);
    if (hx_mlp_prepare(train.rt, B, I, H, O, 0) != HX_OK)
        return failed(head, r, "prepare", hx_runtime_last_error(train.rt));
    if (hx_mlp_prepare(eval.rt, N, I, H, O, 0) != HX_OK)
        return failed(head, r, "prepare", hx_runtime_last_error(eval.rt));
    if (r->execution_mode == 35) hx_runtime_inject_execute_failure(train.rt, 37);
    float initial = 0, final_loss = 0;
    if (!full_loss(eval.rt, x, y, w1, w2, &initial)) return failed(head, r, "loss", hx_runtime_last_error(eval.rt));

    std::vector<float> w1n(w1.size()), w2n(w2.size()), xb(size_t(B) * I), yb(size_t(B) * O);
    Stats exec;
    bool nan = false, stopped = false;
    int done = 0;
    for (int st = 0; st < steps; ++st) {
        if (g_stop.load()) {
            stopped = true;
            break;
        }
        for (int b = 0; b < B; ++b) {
            const int row = (st * B + b) % N;  // cyclic batch (qnn_mlp_training.cpp:98-104)
            std::copy(x.begin() + size_t(row) * I, x.begin() + size_t(row + 1) * I, xb.begin() + size_t(b) * I);
            std::copy(y.begin() + size_t(row) * O, y.begin() + size_t(row + 1) * O, yb.begin() + size_t(b) * O);
        }
        float loss = 0;
        hx_mlp_outputs o{};
        o.loss = &loss;
        o.w1_next = w1n.data();
        o.w2_next = w2n.data();
        if (hx_mlp_execute(train.rt, xb.data(), xb.size(), yb.data(), yb.size(), w1.data(), w1.size(), w2.data(),
                           w2.size(), r->learning_rate, &o) != HX_OK)
            return failed(head, r, "full_step_execute", hx_runtime_last_error(train.rt));
        hx_metrics m{};
        hx_runtime_metrics(train.rt, &m);
        exec.v.push_back(m.last_execute_us);
        std::swap(w1, w1n);  // ping-pong handoff (qnn_mlp_training.cpp:748-749)
        std::swap(w2, w2n);
        nan = nan || !std::isfinite(loss);
        ++done;
        if (done == 1 || done % 16 == 0 || done == steps)
            progress(r, "phase=training\nstep=" + std::to_string(done) + "\nloss=" + std::to_string(loss));
        if (nan) break;
    }
    if (!full_loss(eval.rt, x, y, w1, w2, &final_loss)) return failed(head, r, "loss", hx_runtime_last_error(eval.rt));
    const bool ok = !nan && !stopped && std::isfinite(final_loss) && final_loss < initial;
    hx_metrics m{};
    hx_runtime_metrics(train.rt, &m);
    std::ostringstream s;
    s.precision(9);
    s << head << "\nexecution_mode=" << mode_name(r->execution_mode) << "\nseed=" << r->seed
      << "\nsample_count=" << N << "\nbatch_size=" << B << "\ninput_dim=" << I << "\nhidden_dim=" << H
      << "\noutput_dim=" << O << "\nepochs=" << r->epochs << "\nsteps=" << done << "\nlearning_rate="
      << r->learning_rate << "\ninitial_loss=" << initial << "\nfinal_loss=" << final_loss
      << "\nloss_reduction_ratio=" << final_loss / initial << "\ntraining_graph_create_count="
      << m.graph_create_count << "\ntraining_graph_execute_count=" << m.graph_execute_count
      << "\nexecute_count_per_step=1\nweight_handoff_method=PING_PONG_BINDING\ninput_output_alias=false";
    exec.emit(s, "training_graph_execute");
    s << "\ncpu_fallback=false\nbackend=CUDA_B200\nnan_detected=" << (nan ? "true" : "false")
      << "\nstopped=" << (stopped ? "true" : "false") << "\nstatus=" << (ok ? "SUCCESS" : "FAILED") << '\n';
    return s.str();
}

const char* stability_name(int mode) {
    static const char* names[] = {"LEGACY", "WARMUP64", "DECAY_LINEAR", "ZERO_OUTPUT_PROJ_BRANCH_INIT",
                                  "DEPTH_SCALED_BRANCH_INIT", "RESIDUAL_BRANCH_SCALING", "GRADIENT_CLIP_1"};
    return mode >= 0 && mode <= 6 ? names[mode] : "UNKNOWN";
}

std::string run_lm(const hx_bridge_run* r) {
    const char* head = "TINY_LANGUAGE_MODEL";
    hx_lm_config c{uint32_t(r->output_dimension), uint32_t(r->sample_count), uint32_t(r->dimension),
                   uint32_t(r->hidden_dimension), uint32_t(r->epochs), uint32_t(r->measured_steps), 1e-5f, 0};
    char msg[512] = {};
    if (hx_lm_validate(&c, msg, sizeof msg) != HX_OK) return failed(head, r, "configuration", msg);
    if (r->batch_size <= 0 || r->steps <= 0) return failed(head, r, "configuration", "batch size and steps must be > 0");
    if (const char* bad = hx_stability_mode_error(uint32_t(r->training_stability_mode)))
        return failed(head, r, "training_stability_mode", bad);
    const uint32_t B = uint32_t(r->batch_size), T = c.tokens, V = c.vocab;
    const uint64_t seed = uint64_t(r->seed);
    Runtime rt;
    if (hx_runtime_create(0, &rt.rt, msg, sizeof msg) != HX_OK) return failed(head, r, "runtime_create", msg);
    if (hx_lm_prepare(rt.rt, &c, B, 0) != HX_OK) return failed(head, r, "prepare", hx_runtime_last_error(rt.rt));
    hx_optimizer_config opt{};
    opt.kind = HX_OPT_ADAM;
    opt.adam_lr = r->learning_rate > 0 ? r->learning_rate : 1e-3f;
    opt.beta1 = 0.9f;
    opt.beta2 = 0.999f;
    opt.adam_eps = 1e-8f;
    if (hx_lm_set_optimizer(rt.rt, &opt) != HX_OK ||
        hx_lm_set_stability(rt.rt, uint32_t(r->training_stability_mode), uint32_t(r->steps), 0.0f) != HX_OK)
        return failed(head, r, "optimizer", hx_runtime_last_error(rt.rt));
    const size_t P = hx_lm_param_count(&c);
    std::vector<float> p(P);
    hx_lm_init_reference(&c, uint32_t(seed), p.data());
    hx_lm_apply_init_stability(&c, uint32_t(r->training_stability_mode), p.data());
    if (hx_lm_state_upload(rt.rt, p.data(), nullptr, nullptr, nullptr, P) != HX_OK)
        return failed(head, r, "state_upload", hx_runtime_last_error(rt.rt));
    const std::string dir = r->diagnostic_checkpoint_dir ? r->diagnostic_checkpoint_dir : "";
    uint32_t first = 1;
    std::string resume = "n/a";
    if (r->diagnostic_resume_step > 0) {
        char name[160];
        hx_nprt_checkpoint_name(uint32_t(seed), c.layers, T, c.dim, c.ffn, uint32_t(r->diagnostic_resume_step), name,
                                sizeof name);
        hx_nprt_info info{};
        if (hx_lm_checkpoint_resume(rt.rt, (dir + "/" + name).c_str(), uint32_t(seed),
                                    uint32_t(r->diagnostic_resume_step), nullptr, &info) != HX_OK)
            return failed(head, r, "resume", hx_runtime_last_error(rt.rt));
        first = info.step + 1;
        resume = info.parameter_hash;
    }
    Stats exec;
    std::vector<uint32_t> tokens;
    float first_loss = NAN, last_loss = NAN;
    bool stopped = false, nan = false;
    uint32_t last_step = first - 1;
    for (uint32_t step = first; step <= uint32_t(r->steps); ++step) {
        if (g_stop.load()) {
            stopped = true;
            break;
        }
        zipf(seed * 1000003ull + (step - 1), size_t(B) * (T + 1), V, 1.1, tokens);
        float loss = 0;
        if (hx_lm_train_step(rt.rt, tokens.data(), step, &loss) != HX_OK)
            return failed(head, r, "train_step", hx_runtime_last_error(rt.rt));
        hx_metrics m{};
        hx_runtime_metrics(rt.rt, &m);
        exec.v.push_back(m.last_execute_us);
        if (step == first) first_loss = loss;
        last_loss = loss;
        last_step = step;
        nan = nan || !std::isfinite(loss);
        progress(r, "phase=training\nstep=" + std::to_string(step) + "\nloss=" + std::to_string(loss));
        if (nan) break;
    }
    std::string ckpt = "n/a";
    if (!dir.empty() && last_step > 0 && !nan) {
        char name[160];
        hx_nprt_checkpoint_name(uint32_t(seed), c.layers, T, c.dim, c.ffn, last_step, name, sizeof name);
        if (V == 1024) {
            ckpt = "SKIPPED_NO_TOKENIZER_IDENTITY";  // V3 files need the tokenizer hash
        } else if (hx_lm_checkpoint_save(rt.rt, (dir + "/" + name).c_str(), uint32_t(seed), last_step, nullptr,
                                         nullptr) == HX_OK) {
            ckpt = name;
        } else {
            return failed(head, r, "checkpoint_write", hx_runtime_last_error(rt.rt));
        }
    }
    const bool ok = !nan && !stopped && last_step == uint32_t(r->steps);
    std::ostringstream s;
    s.precision(9);
    s << head << "\nexecution_mode=" << mode_name(r->execution_mode) << "\nseed=" << r->seed << "\nvocabulary=" << V
      << "\ntokens=" << T << "\ndimension=" << c.dim << "\nffn=" << c.ffn << "\nlayers=" << c.layers
      << "\nheads=" << c.heads << "\nbatch_size=" << B << "\nsteps=" << last_step << "\nfirst_step=" << first
      << "\noptimizer=ADAM\nadam_learning_rate=" << opt.adam_lr << "\ntraining_stability_mode="
      << stability_name(r->training_stability_mode) << "\nfirst_loss=" << first_loss << "\nfinal_loss=" << last_loss
      << "\nresume_checkpoint_hash=" << resume << "\ncheckpoint_written=" << ckpt;
    exec.emit(s, "train_step_execute");
    s << "\ncpu_fallback=false\nbackend=CUDA_B200\nnan_detected=" << (nan ? "true" : "false")
      << "\nstopped=" << (stopped ? "true" : "false") << "\nstatus=" << (ok ? "SUCCESS" : "FAILED") << '\n';
    return s.str();
}

}  // namespace

extern "C" {

const char* hx_bridge_environment_report(void) {
    std::ostringstream s;
    int n = 0;
    const cudaError_t e = cudaGetDeviceCount(&n);
    s << "ENVIRONMENT\nbackend=CUDA_B200\nlibrary=libhexatrain_b200\ncuda_device_count=" << (e == cudaSuccess ? n : 0);
    int rtv = 0, drv = 0;
    cudaRuntimeGetVersion(&rtv);
    cudaDriverGetVersion(&drv);
    s << "\ncuda_runtime_version=" << rtv << "\ncuda_driver_version=" << drv;
    for (int d = 0; e == cudaSuccess && d < n; ++d) {
        cudaDeviceProp p{};
        if (cudaGetDeviceProperties(&p, d) != cudaSuccess) continue;
        s << "\ndevice_" << d << "_name=" << p.name << "\ndevice_" << d << "_compute_capability=" << p.major << '.'
          << p.minor << "\ndevice_" << d << "_sm_count=" << p.multiProcessorCount << "\ndevice_" << d
          << "_memory_bytes=" << p.totalGlobalMem;
    }
    s << '\n';
    cudaGetLastError();  // a missing device is reported above, not left pending
    return keep(s.str());
}

const char* hx_bridge_status_report(void) {
    std::ostringstream s;
    hx_runtime* rt = nullptr;
    char msg[512] = {};
    const int rc = hx_runtime_create(0, &rt, msg, sizeof msg);
    s << "RUNTIME_STATUS\nbackend=CUDA_B200\nstatus=" << (rc == HX_OK ? "AVAILABLE" : "UNAVAILABLE");
    if (rc != HX_OK) s << "\nerror=" << msg;
    s << "\nserved_execution_modes=32,33,35,99\ncpu_fallback=false\n";
    if (rt) hx_runtime_destroy(rt);
    return keep(s.str());
}

const char* hx_bridge_run_execution_mode(const hx_bridge_run* r) {
    if (!r) return keep("EXECUTION\nstatus=FAILED\nerror=null run\n");
    const int mode = r->execution_mode;
    if (mode != 32 && mode != 33 && mode != 35 && mode != 99) {
        std::ostringstream s;
        s << "EXECUTION\nexecution_mode=" << mode
          << "\nstatus=FAILED\nfailure_classification=UNSUPPORTED_EXECUTION_MODE\ncpu_fallback=false\n";
        return keep(s.str());
    }
    bool expected = false;
    if (!g_running.compare_exchange_strong(expected, true))
        return keep("EXECUTION\nstatus=FAILED\nerror=a benchmark is already running\n");
    std::string out;
    try {
        out = mode == 99 ? run_lm(r) : run_mlp(r);
    } catch (const std::exception& e) {
        out = failed("EXECUTION", r, "exception", e.what());
    }
    g_running.store(false);
    return keep(std::move(out));
}

void hx_bridge_request_stop(void) { g_stop.store(true); }

void hx_bridge_clear_stop(void) {
    if (!g_running.load()) g_stop.store(false);
}

}  // extern "C"
