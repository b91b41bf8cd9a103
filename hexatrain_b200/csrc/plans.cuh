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
    std::map<Key, cudaGraphExec_t> execs;
    ~GraphCache() { clear(); }
    void clear() {
        for (auto& kv : execs) cudaGraphExecDestroy(kv.second);
        execs.clear();
    }
};

struct MlpPlan {
    uint32_t B = 0, I = 0, H = 0, O = 0;
    bool diag = false;
    Arena arena;
    // arena offsets
    size_t x, y, w1, w2, w1n, w2n, h, p, e, dp, dw2, dh, mask, dz1, dw1, loss;
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
// with a fixed-shape tree instead of a sequential sum.  One block.
__global__ void mse_reduce_kernel(const float* __restrict__ e, size_t n, float* __restrict__ loss);

// Copies `count` floats, used for D2D staging inside captured graphs.
void copy_d2d(hx_runtime* rt, void* dst, const void* src, size_t bytes);

}  // namespace hx

