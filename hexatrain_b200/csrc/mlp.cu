// mlp.cu -- phonelm_mlp_training_step on B200.
//
// The reference builds a 16-node QNN graph (qnn/qnn_runtime_full_step.inc:209-330).
// Here the same dataflow is five GEMM launches whose epilogues carry every
// elementwise node, plus one deterministic loss reduction:
//   1. Z1 = X W1           epilogue: H = ReLU(Z1), mask = H > 0
//   2. P  = H W2           epilogue: E = P - Y, dP = E * 2/(B*O)
//   3. loss = mean(E^2)    double-precision block sums, added in block order
//   4. dW2 = H^T dP        epilogue: W2_next = W2 - lr*dW2
//   5. dH = dP W2^T        epilogue: dZ1 = (H > 0) ? dH : 0   (pre-update W2)
//   6. dW1 = X^T dZ1       epilogue: W1_next = W1 - lr*dW1
// The whole sequence is captured once per distinct set of bound pointers into
// a CUDA graph and replayed, so a step costs one graph launch.  Small shapes
// (the reference's 8/128/128/64 and 32/256/256/128) run instead as one
// kernel on one cluster of CTAs (mlp_fused.cuh).
#include <cmath>

#include "gemm.cuh"
#include "mlp_fused.cuh"
#include "plans.cuh"

namespace hx {

__global__ void mse_reduce_kernel(const float* __restrict__ e, size_t n, size_t chunk, double* __restrict__ part,
                                  unsigned int* __restrict__ done, float* __restrict__ loss)
{
    HX_PDL_PROLOGUE();
    __shared__ double wsum[32];
    __shared__ bool last;
    const int w = threadIdx.x / 32, l = threadIdx.x % 32, nw = blockDim.x / 32;
    // this block's contiguous chunk, strided over the block's threads
    const size_t lo = size_t(blockIdx.x) * chunk, hi = lo + chunk < n ? lo + chunk : n;
    double s = 0.0;
    for (size_t i = lo + threadIdx.x; i < hi; i += blockDim.x) {
        const double v = e[i];
        s += v * v;
    }
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (l == 0) wsum[w] = s;
    __syncthreads();
    if (w == 0) {
        s = l < nw ? wsum[l] : 0.0;
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if (l == 0) {
            part[blockIdx.x] = s;
            __threadfence();
            last = atomicAdd(done, 1u) == gridDim.x - 1;
        }
    }
    __syncthreads();
    if (!last) return;
    // The last block to finish: the per-block sums in a fixed tree by index.
    __threadfence();
    s = 0.0;
    for (unsigned int b = threadIdx.x; b < gridDim.x; b += blockDim.x) s += __ldcg(part + b);
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (l == 0) wsum[w] = s;
    __syncthreads();
    if (w == 0) {
        s = l < nw ? wsum[l] : 0.0;
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if (l == 0) {
            *loss = (float)(s / (double)n);
            *done = 0u;  // ready for the next launch
        }
    }
}

void launch_mse_reduce(hx_runtime* rt, const float* e, size_t n, double* part, unsigned int* done, float* loss)
{
    // Chunks of at least 16K elements, at most two blocks per SM: the grid,
    // and with it the summation order, depends only on n and the SM count.
    const size_t min_chunk = 16384;
    size_t blocks = (n + min_chunk - 1) / min_chunk;
    blocks = std::max<size_t>(1, std::min<size_t>(blocks, std::min<size_t>(kMseMaxBlocks, 2 * size_t(rt->sm_count))));
    const size_t chunk = (n + blocks - 1) / blocks;
    blocks = std::max<size_t>(1, (n + chunk - 1) / chunk);
    ::hx::pdl_launch(mse_reduce_kernel, (unsigned)blocks, 1024, 0, rt->stream, e, n, chunk, part, done, loss);
    HX_LAUNCHED(rt);
}

void copy_d2d(hx_runtime* rt, void* dst, const void* src, size_t bytes) {
    if (bytes) HX_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, rt->stream));
}

namespace {

struct MlpBinding {
    const float *x, *y, *w1, *w2;
    float *loss, *w1n, *w2n;
    float *h, *p, *e, *dp, *dw2, *dh, *dz1, *dw1;
    uint8_t* mask;
    float lr;
};

// Whether the fused MLP step can run as a 16-CTA cluster on this device (a
// non-portable cluster size: opted in per kernel, then checked by the
// occupancy query); sets the kernels' shared-memory limits either way.
bool mlp_fused_cluster16(hx_runtime* rt)
{
    static int answer[64] = {};  // per device: 0 unknown, 1 yes, 2 no
    int& a = answer[rt->device & 63];
    if (a == 0) {
        HX_CUDA(cudaFuncSetAttribute(mlp_fused_step_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)kMlpFusedSmemBytes));
        a = 2;
        if (cudaFuncSetAttribute(mlp_fused_step_kernel<16>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) ==
                cudaSuccess &&
            cudaFuncSetAttribute(mlp_fused_step_kernel<16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)kMlpFusedSmemBytes) == cudaSuccess) {
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3(16);
            cfg.blockDim = dim3(kMlpFusedThreads);
            cfg.dynamicSmemBytes = kMlpFusedSmemBytes;
            int clusters = 0;
            if (cudaOccupancyMaxActiveClusters(&clusters, mlp_fused_step_kernel<16>, &cfg) == cudaSuccess &&
                clusters >= 1)
                a = 1;
        }
        (void)cudaGetLastError();
    }
    return a == 1;
}

void mlp_enqueue(hx_runtime* rt, const MlpPlan& pl, const MlpBinding& b)
{
    const int B = pl.B, I = pl.I, H = pl.H, O = pl.O;
    if (rt->gemm_backend == HX_GEMM_AUTO && mlp_fused_eligible(pl.B, pl.I, pl.H, pl.O)) {
        // the whole step in one cluster launch (small shapes)
        ProfScope prof(rt, kTagGemm, 2.0 * B * (2.0 * I * H + 3.0 * H * O),
                       4.0 * (2.0 * (double(I) * H + double(H) * O) + double(B) * I + double(B) * O));
        const MlpFusedArgs fa{b.x, b.y, b.w1, b.w2, b.loss, b.w1n, b.w2n, b.h, b.p, b.e, b.dp, b.dw2, b.dh, b.dz1,
                              b.dw1, b.mask, pl.arena.at<double>(pl.mse_part), b.lr, B, I, H, O};
        if (mlp_fused_cluster16(rt))
            ::hx::pdl_launch(mlp_fused_step_kernel<16>, 16, kMlpFusedThreads, kMlpFusedSmemBytes, rt->stream, fa);
        else
            ::hx::pdl_launch(mlp_fused_step_kernel<8>, 8, kMlpFusedThreads, kMlpFusedSmemBytes, rt->stream, fa);
        HX_LAUNCHED(rt);
        return;
    }
    const float s = 2.0f / float(B * O);
    gemm<false, false>(rt, B, H, I, b.x, I, b.w1, H, EpiRelu{b.h, b.mask, H});
    gemm<false, false>(rt, B, O, H, b.h, H, b.w2, O, EpiError{b.y, b.p, b.e, b.dp, s, O});
    {
        ProfScope prof(rt, kTagReduce, 2.0 * B * O, 4.0 * B * O);
        launch_mse_reduce(rt, b.e, size_t(B) * O, pl.arena.at<double>(pl.mse_part), pl.arena.at<unsigned int>(pl.mse_done),
                          b.loss);
    }
    gemm<true, false>(rt, H, O, B, b.h, H, b.dp, O, EpiSgd{b.w2, b.dw2, b.w2n, b.lr, O});
    gemm<false, true>(rt, B, H, O, b.dp, O, b.w2, O, EpiReluBackward{b.h, b.dz1, b.dh, H});
    gemm<true, false>(rt, I, H, B, b.x, I, b.dz1, H, EpiSgd{b.w1, b.dw1, b.w1n, b.lr, H});
}

GraphCache::Key key_of(const MlpBinding& b) {
    GraphCache::Key k{};
    const void* ptrs[] = {b.x, b.y, b.w1, b.w2, b.loss, b.w1n, b.w2n, b.h, b.p, b.e, b.dp,
                          b.dw2, b.dh, b.dz1, b.dw1, b.mask};
    size_t i = 0;
    for (const void* p : ptrs) k[i++] = reinterpret_cast<uintptr_t>(p);
    uint32_t bits;
    std::memcpy(&bits, &b.lr, 4);
    k[i++] = bits;
    return k;
}

// Runs the step: eagerly the first time a binding is seen (this also sizes
// the workspace), from a captured CUDA graph afterwards.
void mlp_run(hx_runtime* rt, MlpPlan& pl, const MlpBinding& b)
{
    if (!pl.use_graphs || rt->prof.on) {
        mlp_enqueue(rt, pl, b);
        return;
    }
    run_cached(rt, pl.graphs, key_of(b), [&] { mlp_enqueue(rt, pl, b); });
}

MlpPlan& need_mlp(hx_runtime* rt) {
    require(rt->mlp != nullptr, HX_ERR_STATE, "full step graph not prepared");
    return *rt->mlp;
}

}  // namespace
}  // namespace hx

using namespace hx;

extern "C" {

int hx_mlp_prepare(hx_runtime* rt, uint32_t B, uint32_t I, uint32_t H, uint32_t O, int diagnostic) {
    return hx_guard(rt, [&] {
        require(B && I && H && O, HX_ERR_ARGUMENT, "full step invalid runtime or shape");
        const uint64_t lim = uint64_t(1) << 31;
        require(uint64_t(B) * I < lim && uint64_t(I) * H < lim && uint64_t(B) * H < lim && uint64_t(H) * O < lim &&
                    uint64_t(B) * O < lim,
                HX_ERR_ARGUMENT, "full step shape exceeds 2^31 elements per tensor");
        auto pl = std::make_unique<MlpPlan>();
        pl->B = B; pl->I = I; pl->H = H; pl->O = O;
        pl->diag = diagnostic != 0;
        const size_t f = sizeof(float);
        Arena& a = pl->arena;
        pl->x = a.reserve(f * B * I);
        pl->y = a.reserve(f * B * O);
        pl->w1 = a.reserve(f * I * H);
        pl->w2 = a.reserve(f * H * O);
        pl->w1n = a.reserve(f * I * H);
        pl->w2n = a.reserve(f * H * O);
        pl->h = a.reserve(f * B * H);
        pl->p = a.reserve(f * B * O);
        pl->e = a.reserve(f * B * O);
        pl->dp = a.reserve(f * B * O);
        pl->dw2 = a.reserve(f * H * O);
        pl->dh = a.reserve(f * B * H);
        pl->mask = a.reserve(size_t(B) * H);
        pl->dz1 = a.reserve(f * B * H);
        pl->dw1 = a.reserve(f * I * H);
        pl->loss = a.reserve(f * 4);
        pl->mse_part = a.reserve(sizeof(double) * kMseMaxBlocks);
        pl->mse_done = a.reserve(sizeof(unsigned int));
        a.commit();
        HX_CUDA(cudaMemsetAsync(a.at<unsigned int>(pl->mse_done), 0, sizeof(unsigned int), rt->stream));
        HX_CUDA(cudaStreamSynchronize(rt->stream));
        rt->mlp = std::move(pl);
        ++rt->metrics.graph_create_count;
    });
}

int hx_mlp_execute(hx_runtime* rt, const float* x, size_t xn, const float* y, size_t yn, const float* w1,
                   size_t w1c, const float* w2, size_t w2c, float lr, const hx_mlp_outputs* out) {
    const auto t0 = Clock::now();
    const int rc = hx_guard(rt, [&] {
        MlpPlan& pl = need_mlp(rt);
        require(x && y && w1 && w2 && out && out->loss && out->w1_next && out->w2_next, HX_ERR_ARGUMENT,
                "full step null buffer");
        require(xn == size_t(pl.B) * pl.I && yn == size_t(pl.B) * pl.O && w1c == size_t(pl.I) * pl.H &&
                    w2c == size_t(pl.H) * pl.O,
                HX_ERR_ARGUMENT, "full step buffer size mismatch");
        require(std::isfinite(lr), HX_ERR_ARGUMENT, "full step learning rate must be finite");
        const Arena& a = pl.arena;
        const auto tb = Clock::now();
        HX_CUDA(cudaMemcpyAsync(a.at<float>(pl.x), x, xn * 4, cudaMemcpyHostToDevice, rt->stream));
        HX_CUDA(cudaMemcpyAsync(a.at<float>(pl.y), y, yn * 4, cudaMemcpyHostToDevice, rt->stream));
        HX_CUDA(cudaMemcpyAsync(a.at<float>(pl.w1), w1, w1c * 4, cudaMemcpyHostToDevice, rt->stream));
        HX_CUDA(cudaMemcpyAsync(a.at<float>(pl.w2), w2, w2c * 4, cudaMemcpyHostToDevice, rt->stream));
        rt->metrics.last_input_bind_us = us_since(tb);
        MlpBinding b{a.at<float>(pl.x), a.at<float>(pl.y), a.at<float>(pl.w1), a.at<float>(pl.w2),
                     a.at<float>(pl.loss), a.at<float>(pl.w1n), a.at<float>(pl.w2n), a.at<float>(pl.h),
                     a.at<float>(pl.p), a.at<float>(pl.e), a.at<float>(pl.dp),
                     pl.diag ? a.at<float>(pl.dw2) : nullptr, pl.diag ? a.at<float>(pl.dh) : nullptr,
                     a.at<float>(pl.dz1), pl.diag ? a.at<float>(pl.dw1) : nullptr,
                     pl.diag ? a.at<uint8_t>(pl.mask) : nullptr, lr};
        mlp_run(rt, pl, b);
        const auto to = Clock::now();
        auto get = [&](void* dst, size_t off, size_t bytes) {
            if (dst) HX_CUDA(cudaMemcpyAsync(dst, a.at<char>(off), bytes, cudaMemcpyDeviceToHost, rt->stream));
        };
        const size_t f = 4, B = pl.B, I = pl.I, H = pl.H, O = pl.O;
        get(out->loss, pl.loss, f);
        get(out->w1_next, pl.w1n, f * I * H);
        get(out->w2_next, pl.w2n, f * H * O);
        if (pl.diag) {
            get(out->prediction, pl.p, f * B * O);
            get(out->error, pl.e, f * B * O);
            get(out->d_prediction, pl.dp, f * B * O);
            get(out->d_w2, pl.dw2, f * H * O);
            get(out->d_hidden, pl.dh, f * B * H);
            get(out->mask, pl.mask, B * H);
            get(out->d_z1, pl.dz1, f * B * H);
            get(out->d_w1, pl.dw1, f * I * H);
            get(out->hidden, pl.h, f * B * H);
        }
        rt->check_device_error();
        rt->metrics.last_output_bind_us = us_since(to);
        if (rt->injected_now()) fail(HX_ERR_CUDA, "injected execute failure after device success");
    });
    if (rt) rt->record_execute(rc == HX_OK, us_since(t0));
    return rc;
}

int hx_mlp_execute_device(hx_runtime* rt, const float* x, const float* y, const float* w1, const float* w2,
                          float lr, const hx_mlp_outputs* out) {
    const auto t0 = Clock::now();
    const int rc = hx_guard(rt, [&] {
        MlpPlan& pl = need_mlp(rt);
        require(x && y && w1 && w2 && out && out->loss && out->w1_next && out->w2_next, HX_ERR_ARGUMENT,
                "full step null buffer");
        require(std::isfinite(lr), HX_ERR_ARGUMENT, "full step learning rate must be finite");
        require(w1 != out->w1_next && w2 != out->w2_next, HX_ERR_ARGUMENT,
                "full step in-place alias: next weights must not alias current weights");
        const Arena& a = pl.arena;
        auto pick = [&](float* user, size_t off) { return user ? user : a.at<float>(off); };
        MlpBinding b{x, y, w1, w2, out->loss, out->w1_next, out->w2_next,
                     pick(out->hidden, pl.h), pick(out->prediction, pl.p), pick(out->error, pl.e),
                     pick(out->d_prediction, pl.dp), out->d_w2, out->d_hidden, pick(out->d_z1, pl.dz1),
                     out->d_w1, out->mask, lr};
        mlp_run(rt, pl, b);
        if (rt->injected_now()) {
            HX_CUDA(cudaStreamSynchronize(rt->stream));
            fail(HX_ERR_CUDA, "injected execute failure after device success");
        }
    });
    if (rt) rt->record_execute(rc == HX_OK, us_since(t0));
    return rc;
}

}  // extern "C"
