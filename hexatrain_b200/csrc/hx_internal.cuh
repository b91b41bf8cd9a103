// hx_internal.cuh -- shared internals of libhexatrain_b200.so.
//
// Error convention: internal code throws hx::Error; every extern "C" entry
// point catches it, stores the message in the runtime (hx_runtime_last_error)
// and returns the status code.  Nothing throws across the C ABI, matching the
// reference's bool + std::string& error convention (qnn/qnn_runtime.h:250-451).
#pragma once

#include "pdl.cuh"

#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cstdint>
#include <cstring>
#include <memory>
#include <string>
#include <utility>
#include <vector>

#include "../../include/hexatrain.h"

namespace hx {

struct Error {
    int code;
    std::string message;
};

[[noreturn]] inline void fail(int code, const std::string& msg) { throw Error{code, msg}; }

inline void check_cuda(cudaError_t e, const char* what) {
    if (e != cudaSuccess) fail(HX_ERR_CUDA, std::string(what) + ": " + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ")");
}
#define HX_CUDA(call) ::hx::check_cuda((call), #call)
// After a kernel launch: catches launch-configuration errors immediately.
#define HX_LAUNCHED(rt) do { ::hx::check_cuda(cudaGetLastError(), "kernel launch"); ++(rt)->metrics.kernel_launches; } while (0)

// Launches `kernel` on `stream` with programmatic stream serialisation: the
// kernel may be launched as the previous kernel of the stream drains,
// and its HX_PDL_PROLOGUE() holds it until that kernel has completed.
// Arguments are converted to the kernel's parameter types.
template <class... KArgs, class... Args>
inline void pdl_launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    check_cuda(cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...), "kernel launch");
}

inline void require(bool ok, int code, const std::string& msg) {
    if (!ok) fail(code, msg);
}

using Clock = std::chrono::steady_clock;
inline double us_since(Clock::time_point t0) {
    return std::chrono::duration<double, std::micro>(Clock::now() - t0).count();
}

// One device allocation owned by a runtime.
struct DeviceBuffer {
    void* ptr = nullptr;
    size_t bytes = 0;
    DeviceBuffer() = default;
    DeviceBuffer(const DeviceBuffer&) = delete;
    DeviceBuffer& operator=(const DeviceBuffer&) = delete;
    ~DeviceBuffer() { release(); }
    void release() {
        if (ptr) cudaFree(ptr);
        ptr = nullptr;
        bytes = 0;
    }
    void allocate(size_t n) {
        release();
        if (n == 0) n = 16;
        const cudaError_t e = cudaMalloc(&ptr, n);
        if (e != cudaSuccess) {
            ptr = nullptr;
            fail(HX_ERR_MEMORY, "device allocation of " + std::to_string(n) + " bytes failed: " + cudaGetErrorString(e));
        }
        bytes = n;
    }
    template <class T> T* as() const { return static_cast<T*>(ptr); }
};

// Bump allocator over one device allocation: all per-plan tensors are carved
// out of a single cudaMalloc at prepare time (256-byte aligned sub-buffers).
struct Arena {
    DeviceBuffer block;
    size_t used = 0;
    struct Slot { size_t offset; };
    std::vector<size_t> pending;
    size_t reserve(size_t bytes) {
        const size_t off = (used + 255) & ~size_t(255);
        used = off + bytes;
        return off;
    }
    void commit() { block.allocate(used); }
    template <class T> T* at(size_t offset) const { return reinterpret_cast<T*>(static_cast<char*>(block.ptr) + offset); }
};

// Kernel classes for the event profiler (hx_runtime_profile).
enum ProfTag { kTagGemm = 0, kTagAttnFwd, kTagAttnBwd, kTagLayerNorm, kTagSoftmaxCe, kTagOptimizer, kTagEmbed,
               kTagReduce, kTagCount };
inline const char* prof_tag_name(int t) {
    static const char* n[] = {"gemm", "attention_fwd", "attention_bwd", "layernorm", "softmax_ce", "optimizer",
                              "embedding", "reduce"};
    return (t >= 0 && t < kTagCount) ? n[t] : "other";
}

struct ProfRecord {
    int tag;
    cudaEvent_t a, b;
    double flops, bytes;
};

struct Profiler {
    bool on = false;
    std::vector<cudaEvent_t> pool;
    size_t used = 0;
    std::vector<ProfRecord> recs;
    ~Profiler() {
        for (cudaEvent_t e : pool) cudaEventDestroy(e);
    }
    cudaEvent_t next() {
        if (used == pool.size()) {
            cudaEvent_t e;
            check_cuda(cudaEventCreate(&e), "cudaEventCreate");
            pool.push_back(e);
        }
        return pool[used++];
    }
};

// Error-word codes of the bounded waits: GEMM roles 1-4, attention roles
// 11-14, the Muon kernel 16, and the wait self-test
// (hx_runtime_check_wait_timeout).
constexpr int kWaitProbeCode = 21;

struct MlpPlan;
struct LmPlan;
struct AdamPlan;
struct MomentumPlan;
// LmPlan is defined in lm.cu; its deleter is too.
struct LmPlanDeleter {
    void operator()(LmPlan* p) const;
};

}  // namespace hx

struct hx_runtime {
    int device = 0;
    cudaStream_t own_stream = nullptr;
    cudaStream_t stream = nullptr;
    std::string last_error;
    hx_metrics metrics{};
    int64_t inject_execute_at = -1;
    int sm_count = 148;
    std::unique_ptr<hx::MlpPlan> mlp;
    std::unique_ptr<hx::LmPlan, hx::LmPlanDeleter> lm;
    std::unique_ptr<hx::AdamPlan> adam;
    std::unique_ptr<hx::MomentumPlan> momentum;
    hx::DeviceBuffer scratch;  // generic device workspace (grows on demand)
    // Second stream for work that runs beside the main stream's (the weight
    // gradients of the LM backward) and its own workspace.
    cudaStream_t side_stream = nullptr;
    hx::DeviceBuffer side_scratch;
    hx::DeviceBuffer err_flag; // device-side error word of bounded waits
    hx::Profiler prof;
    int gemm_backend = 0;      // HX_GEMM_AUTO / HX_GEMM_CUDA_CORES / HX_GEMM_TENSOR_CORES
    int attention_backend = 0; // HX_ATTN_AUTO / HX_ATTN_CUDA_CORES

    ~hx_runtime();
    void activate() const { hx::check_cuda(cudaSetDevice(device), "cudaSetDevice"); }
    // Bumped by everything that changes what a captured CUDA graph would
    // launch or where it reads: a workspace reallocation (graphs hold its
    // address) and an engine switch.  Cached graphs of an older epoch are
    // dropped before their next replay.
    uint64_t graph_epoch = 0;
    // Grow-only device workspace for split-K partials and reductions, one
    // per stream so that launches on the two streams never share one.
    float* workspace(size_t bytes) {
        hx::DeviceBuffer& b = (side_stream && stream == side_stream) ? side_scratch : scratch;
        if (b.bytes < bytes) {
            b.allocate(bytes);
            ++graph_epoch;
        }
        return b.as<float>();
    }
    int* device_error() {
        if (!err_flag.ptr) {
            err_flag.allocate(16);
            hx::check_cuda(cudaMemset(err_flag.ptr, 0, 16), "cudaMemset");
        }
        return err_flag.as<int>();
    }
    // Reads (and clears) the device error word; fails if a kernel reported
    // a timed-out pipeline wait.  Synchronises the stream.
    void check_device_error() {
        if (!err_flag.ptr) {
            hx::check_cuda(cudaStreamSynchronize(stream), "cudaStreamSynchronize");
            return;
        }
        int code = 0;
        hx::check_cuda(cudaMemcpyAsync(&code, err_flag.ptr, sizeof(int), cudaMemcpyDeviceToHost, stream),
                       "cudaMemcpyAsync");
        hx::check_cuda(cudaStreamSynchronize(stream), "cudaStreamSynchronize");
        if (code) {
            hx::check_cuda(cudaMemsetAsync(err_flag.ptr, 0, sizeof(int), stream), "cudaMemsetAsync");
            hx::check_cuda(cudaStreamSynchronize(stream), "cudaStreamSynchronize");
            const char* where = code >= hx::kWaitProbeCode ? "wait self-test"
                                : code >= 16               ? "tensor-core Muon"
                                : code >= 10               ? "tensor-core attention"
                                                           : "tensor-core GEMM";
            hx::fail(HX_ERR_CUDA, std::string("DEVICE_WAIT_TIMEOUT: a bounded pipeline wait in the ") + where +
                                      " gave up (role " + std::to_string(code) + "); results of this call are invalid");
        }
    }
    // Record the outcome of an execute call (ApiTrace counters).
    void record_execute(bool ok, double us) {
        ++metrics.execute_attempt_count;
        if (ok) {
            ++metrics.graph_execute_count;
            metrics.last_execute_us = us;
            metrics.total_execute_us += us;
        } else {
            if (metrics.first_failure_call < 0) metrics.first_failure_call = int64_t(metrics.execute_attempt_count - 1);
            ++metrics.execute_failure_count;
        }
    }
    // Host-side failure injection at a given execute attempt index.
    bool injected_now() const {
        return inject_execute_at >= 0 && uint64_t(inject_execute_at) == metrics.execute_attempt_count;
    }
};

namespace hx {
// Records CUDA events around the launches issued in its scope when the
// runtime's profiler is on; no-op otherwise.
struct ProfScope {
    hx_runtime* rt;
    ProfRecord rec{};
    ProfScope(hx_runtime* r, int tag, double flops, double bytes) : rt(r) {
        if (!rt->prof.on) return;
        rec.tag = tag;
        rec.flops = flops;
        rec.bytes = bytes;
        rec.a = rt->prof.next();
        rec.b = rt->prof.next();
        check_cuda(cudaEventRecord(rec.a, rt->stream), "cudaEventRecord");
    }
    // Closes the timed region (idempotent; the destructor calls it too).
    void end() {
        if (!rt->prof.on || !rec.a) return;
        if (cudaEventRecord(rec.b, rt->stream) == cudaSuccess) rt->prof.recs.push_back(rec);
        rec.a = nullptr;
    }
    ~ProfScope() { end(); }
};
}  // namespace hx

// Runs `body` and converts any failure to a status code + stored message.
template <class F>
inline int hx_guard(hx_runtime* rt, F&& body) {
    if (!rt) return HX_ERR_ARGUMENT;
    try {
        rt->activate();
        body();
        rt->last_error.clear();
        return HX_OK;
    } catch (const hx::Error& e) {
        rt->last_error = e.message;
        return e.code;
    } catch (const std::bad_alloc&) {
        rt->last_error = "host allocation failed";
        return HX_ERR_MEMORY;
    } catch (const std::exception& e) {
        rt->last_error = e.what();
        return HX_ERR_ARGUMENT;
    }
}
