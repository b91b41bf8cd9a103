// plans.cuh -- prepared per-graph state (the CUDA counterpart of a finalized
// QNN graph): shapes, device tensors carved from one arena, and cached CUDA
// graphs for replay.
#pragma once

#include <algorithm>
#include <array>
#include <map>

#include "hx_internal.cuh"

namespace hx {

// Cache of instantiated CUDA graphs keyed by the device pointers a step was
// captured with.  The ping-pong weight swap of the reference driver
// (qnn/qnn_mlp_training.cpp:748-749) produces two keys that alternate.
struct GraphCache {
    using Key = std::array<uintptr_t, 24>;
    struct Entry {
        cudaGraphExec_t exec;
        uint64_t kernels;  // kernel launches the graph replays
    };
    std::map<Key, Entry> execs;
    std::map<Key, int> seen;     // keys run eagerly once, not yet captured
    uint64_t epoch = 0;          // the runtime's graph_epoch when the cached graphs were captured
    bool capture_failed = false; // a capture failed once: run eagerly from then on
    ~GraphCache() { clear(); }
    void clear() {
        for (auto& kv : execs) cudaGraphExecDestroy(kv.second.exec);
        execs.clear();
        seen.clear();
    }
};

// Runs the work `enqueue` puts on the runtime stream: eagerly the first two
// times `key` is seen (the first run also sizes the runtime workspace), with
// a CUDA graph captured right after the second eager run and replayed on
// every later call.  A caller whose pointers change on every call therefore
// never pays for a capture.  Graphs of an older runtime graph epoch are
// dropped.  A stream that cannot be captured
// (the legacy default stream), or a capture that fails, leaves the work to
// run eagerly; the eager run has already done this call's work.
// A plan keeps at most this many captured graphs (the MLP driver's cyclic
// batches over 512 samples at B = 8 bind 64 distinct input slices).
constexpr size_t kGraphCacheMax = 256;

template <class F>
void run_cached(hx_runtime* rt, GraphCache& c, const GraphCache::Key& key, F&& enqueue)
{
    if (c.epoch != rt->graph_epoch) {
        c.clear();
        c.epoch = rt->graph_epoch;
    }
    auto it = c.execs.find(key);
    if (it != c.execs.end()) {
        check_cuda(cudaGraphLaunch(it->second.exec, rt->stream), "cudaGraphLaunch");
        rt->metrics.kernel_launches += it->second.kernels;
        return;
    }
    enqueue();  // eager run
    if (c.capture_failed) return;
    if (c.seen.size() >= 4 * kGraphCacheMax) c.seen.clear();
    if (c.seen.emplace(key, 1).second) return;  // first sighting: no capture yet
    c.seen.erase(key);
    if (c.epoch != rt->graph_epoch) {
        c.clear();
        c.epoch = rt->graph_epoch;
    }
    if (c.execs.size() >= kGraphCacheMax) c.clear();
    if (cudaStreamBeginCapture(rt->stream, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
        (void)cudaGetLastError();
        c.capture_failed = true;
        return;
    }
    cudaGraph_t g = nullptr;
    const uint64_t launches = rt->metrics.kernel_launches;
    bool ok = true;
    try {
        enqueue();
    } catch (...) {
        ok = false;
    }
    const uint64_t kernels = rt->metrics.kernel_launches - launches;
    rt->metrics.kernel_launches = launches;  // captured, not launched
    const cudaError_t ec = cudaStreamEndCapture(rt->stream, &g);
    cudaGraphExec_t exec = nullptr;
    if (ok && ec == cudaSuccess && g && cudaGraphInstantiate(&exec, g, 0) == cudaSuccess) {
        c.execs.emplace(key, GraphCache::Entry{exec, kernels});
        ++rt->metrics.graph_finalize_count;
    } else {
        c.capture_failed = true;
    }
    if (g) cudaGraphDestroy(g);
    (void)cudaGetLastError();
}

struct MlpPlan {
    uint32_t B = 0, I = 0, H = 0, O = 0;
    bool diag = false;
    Arena arena;
    // arena offsets
    size_t x, y, w1, w2, w1n, w2n, h, p, e, dp, dw2, dh, mask, dz1, dw1, loss;
    size_t mse_part, mse_done;  // per-block loss sums and the finished-block counter
    GraphCache graphs;
    bool use_graphs = true;
};

struct AdamPlan {
    uint32_t n = 0;
    Arena arena;
    size_t w, g, m, v, out[10];
};

struct MomentumPlan {
    uint32_t n = 0;
    Arena arena;
    size_t w, g, vel, vel_next, w_next;
};

struct LmPlan;  // lm.cu
size_t lm_plan_bytes(const LmPlan* p);
// The configuration and optimizer kind of the prepared LM plan; false if
// no LM is prepared.
bool lm_prepared_config(const hx_runtime* rt, hx_lm_config* cfg, uint32_t* optimizer_kind);

inline size_t plan_device_bytes(const hx_runtime* rt) {
    size_t n = 0;
    if (rt->mlp) n += rt->mlp->arena.block.bytes;
    if (rt->adam) n += rt->adam->arena.block.bytes;
    if (rt->momentum) n += rt->momentum->arena.block.bytes;
    if (rt->lm) n += lm_plan_bytes(rt->lm.get());
    return n;
}

// ---- shared kernels --------------------------------------------------------

// Sum of squares in double over n floats, divided by n, rounded to float:
// the reference's meanSquaredError (cpu_reference_training.cpp:163-170)
// with fixed-shape trees instead of a sequential sum.  Each block sums one
// contiguous chunk into part[block]; the last block to finish adds the
// block sums in index order and re-zeroes *done, which must be zero when the
// kernel starts.  part holds at least kMseMaxBlocks doubles.
constexpr size_t kMseMaxBlocks = 512;
__global__ void mse_reduce_kernel(const float* __restrict__ e, size_t n, size_t chunk, double* __restrict__ part,
                                  unsigned int* __restrict__ done, float* __restrict__ loss);
void launch_mse_reduce(hx_runtime* rt, const float* e, size_t n, double* part, unsigned int* done, float* loss);

// Copies `count` floats, used for D2D staging inside captured graphs.
void copy_d2d(hx_runtime* rt, void* dst, const void* src, size_t bytes);

}  // namespace hx

