// optim.cu -- C entry points of the standalone optimizers: the reference's
// phonelm_adam_optimizer graph (qnn/qnn_runtime_transformer.inc:926-1218)
// and Muon (no reference counterpart).
#include <cmath>

#include "muon_tc.cuh"
#include "optim.cuh"
#include "plans.cuh"

namespace hx {

// One CTA per matrix.  Shared memory: X [R][C] (R <= C, the shorter side
// first), A [R][R], Bm [R][R].  Limits: R <= 128, R*C <= 16384.
__global__ void muon_kernel(const MuonMatrix* __restrict__ mats, MuonScalars s, const float* __restrict__ lr_dev)
{
    HX_PDL_PROLOGUE();
    if (lr_dev) s.lr = *lr_dev;
    extern __shared__ float sm[];
    const MuonMatrix mt = mats[blockIdx.x];
    const int rows = mt.rows, cols = mt.cols;
    const bool tr = rows > cols;
    const int R = tr ? cols : rows, C = tr ? rows : cols;
    const int n = rows * cols;
    float* X = sm;
    float* A = X + R * C;
    float* Bm = A + R * R;
    __shared__ double red[32];

    // momentum, Nesterov, Frobenius norm
    double ss = 0.0;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float bn = __fadd_rn(__fmul_rn(s.momentum, mt.buf[i]), mt.g[i]);
        mt.buf[i] = bn;
        const float u = s.nesterov ? __fadd_rn(mt.g[i], __fmul_rn(s.momentum, bn)) : bn;
        const int r = i / cols, c = i % cols;
        if (tr) X[c * C + r] = u; else X[r * C + c] = u;
        ss += (double)u * u;
    }
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x < 32) {
        double t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0;
        for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
        if (threadIdx.x == 0) red[0] = t;
    }
    __syncthreads();
    const float inv = (float)(1.0 / (sqrt(red[0]) + 1e-7));
    for (int i = threadIdx.x; i < n; i += blockDim.x) X[i] = __fmul_rn(X[i], inv);
    __syncthreads();

    for (int it = 0; it < s.steps; ++it) {
        // A = X X^T
        for (int i = threadIdx.x; i < R * R; i += blockDim.x) {
            const int r = i / R, q = i % R;
            float acc = 0.f;
            for (int k = 0; k < C; ++k) acc = fmaf(muon_operand(X[r * C + k], s.bf16), muon_operand(X[q * C + k], s.bf16), acc);
            A[i] = acc;
        }
        __syncthreads();
        // Bm = b A + c A A
        for (int i = threadIdx.x; i < R * R; i += blockDim.x) {
            const int r = i / R, q = i % R;
            float acc = 0.f;
            for (int k = 0; k < R; ++k) acc = fmaf(muon_operand(A[r * R + k], s.bf16), muon_operand(A[k * R + q], s.bf16), acc);
            Bm[i] = s.b * A[i] + s.c * acc;
        }
        __syncthreads();
        // X = a X + Bm X   (each thread owns whole output elements; write
        // after a barrier so the product reads the old X)
        float newv[16];
        int cnt = 0;
        for (int i = threadIdx.x; i < R * C; i += blockDim.x) {
            const int r = i / C, q = i % C;
            float acc = 0.f;
            for (int k = 0; k < R; ++k) acc = fmaf(muon_operand(Bm[r * R + k], s.bf16), muon_operand(X[k * C + q], s.bf16), acc);
            newv[cnt++] = s.a * X[i] + acc;
        }
        __syncthreads();
        cnt = 0;
        for (int i = threadIdx.x; i < R * C; i += blockDim.x) X[i] = newv[cnt++];
        __syncthreads();
    }
    const float sc = sqrtf(fmaxf(1.f, (float)rows / (float)cols));
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const int r = i / cols, c = i % cols;
        const float xo = tr ? X[c * C + r] : X[r * C + c];
        mt.w[i] = __fsub_rn(mt.w[i], __fmul_rn(s.lr, __fmul_rn(sc, xo)));
    }
}

AdamScalars adam_scalars(float lr, float gradient_scale, float c1, float c2) {
    AdamScalars s;
    s.lr = lr;
    s.gradient_scale = gradient_scale;
    s.c1 = c1;
    s.c2 = c2;
    s.beta1 = 0.9f;
    s.beta2 = 0.999f;
    // (1 - beta) is formed in float, as tiny_lm::adamUpdate does.
    s.one_minus_beta1 = 1.0f - s.beta1;
    s.one_minus_beta2 = 1.0f - s.beta2;
    s.eps = 1e-8f;
    return s;
}

void launch_adam(hx_runtime* rt, bool graph_order, size_t n, const float* w, const float* g, const float* m,
                 const float* v, float* wn, float* mn, float* vn, const AdamScalars& s, const AdamTaps& t,
                 const float* scale_dev = nullptr, const AdamScalars* s_dev = nullptr)
{
    if (n == 0) return;
    ProfScope prof(rt, kTagOptimizer, 12.0 * n, 28.0 * n);
    const int threads = 256;
    const size_t work = graph_order ? n : (n + 3) / 4;
    const int blocks = (int)std::min<size_t>((work + threads - 1) / threads, size_t(rt->sm_count) * 16);
    if (graph_order)
        ::hx::pdl_launch(adam_kernel<true>, blocks, threads, 0, rt->stream, n, w, g, m, v, wn, mn, vn, s, t, scale_dev, s_dev);
    else
        ::hx::pdl_launch(adam_kernel<false>, blocks, threads, 0, rt->stream, n, w, g, m, v, wn, mn, vn, s, t, scale_dev, s_dev);
    HX_LAUNCHED(rt);
}

__global__ void momentum_kernel(size_t n, const float* w, const float* __restrict__ g, const float* vel,
                                float* w_next, float* vel_next, float lr, float momentum,
                                const float* __restrict__ lr_dev)
{
    HX_PDL_PROLOGUE();
    if (lr_dev) lr = *lr_dev;
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    const size_t tid = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    auto one = [&](float wi, float gi, float vi, float& wo, float& vo) {
        vo = __fadd_rn(__fmul_rn(vi, momentum), gi);
        wo = __fsub_rn(wi, __fmul_rn(vo, lr));
    };
    const bool vec = ((reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(g) |
                       reinterpret_cast<uintptr_t>(vel) | reinterpret_cast<uintptr_t>(w_next) |
                       reinterpret_cast<uintptr_t>(vel_next)) & 15) == 0;
    size_t done = 0;
    if (vec) {
        const size_t n4 = n / 4;
        for (size_t i = tid; i < n4; i += stride) {
            const float4 a = reinterpret_cast<const float4*>(w)[i];
            const float4 b = reinterpret_cast<const float4*>(g)[i];
            const float4 c = reinterpret_cast<const float4*>(vel)[i];
            float4 wo, vo;
            one(a.x, b.x, c.x, wo.x, vo.x);
            one(a.y, b.y, c.y, wo.y, vo.y);
            one(a.z, b.z, c.z, wo.z, vo.z);
            one(a.w, b.w, c.w, wo.w, vo.w);
            reinterpret_cast<float4*>(vel_next)[i] = vo;
            reinterpret_cast<float4*>(w_next)[i] = wo;
        }
        done = n4 * 4;
    }
    for (size_t i = done + tid; i < n; i += stride) {
        float wo, vo;
        one(w[i], g[i], vel[i], wo, vo);
        vel_next[i] = vo;
        w_next[i] = wo;
    }
}

void launch_momentum(hx_runtime* rt, size_t n, const float* w, const float* g, const float* vel, float* wn,
                     float* veln, float lr, float momentum, const float* lr_dev = nullptr)
{
    if (n == 0) return;
    ProfScope prof(rt, kTagOptimizer, 3.0 * n, 20.0 * n);
    const int threads = 256;
    const int blocks = (int)std::min<size_t>(((n + 3) / 4 + threads - 1) / threads, size_t(rt->sm_count) * 16);
    ::hx::pdl_launch(momentum_kernel, blocks, threads, 0, rt->stream, n, w, g, vel, wn, veln, lr, momentum, lr_dev);
    HX_LAUNCHED(rt);
}

constexpr int kNormThreads = 512;

__global__ void __launch_bounds__(kNormThreads) grad_sumsq_kernel(const float* __restrict__ g,
                                                                  const GradTensor* __restrict__ tensors,
                                                                  double* __restrict__ sumsq)
{
    HX_PDL_PROLOGUE();
    const GradTensor t = tensors[blockIdx.x];
    const float* p = g + t.offset;
    double s = 0.0;
    for (unsigned long long i = threadIdx.x; i < t.count; i += kNormThreads) {
        const double x = p[i];
        s += x * x;
    }
    __shared__ double part[kNormThreads / 32];
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        double total = 0.0;
        for (int w = 0; w < kNormThreads / 32; ++w) total += part[w];
        sumsq[blockIdx.x] = total;
    }
}

__global__ void clip_scale_kernel(const double* __restrict__ sumsq, int tensors, float threshold,
                                  double* __restrict__ norm_out, float* __restrict__ scale_out)
{
    HX_PDL_PROLOGUE();
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    double sum = 0.0;
    for (int i = 0; i < tensors; ++i) {
        const double norm = sqrt(sumsq[i]);
        sum += norm * norm;
    }
    const double norm = sqrt(sum);
    *norm_out = norm;
    *scale_out = (threshold > 0.f && isfinite(norm) && norm > 0.0)
                     ? float(fmin(1.0, double(threshold) / (norm + 1.0e-6)))
                     : 1.0f;
}

void launch_clip_scale(hx_runtime* rt, const float* g, const GradTensor* tensors, int count, double* sumsq,
                       float threshold, double* norm_out, float* scale_out)
{
    ProfScope prof(rt, kTagReduce, 0.0, 0.0);
    ::hx::pdl_launch(grad_sumsq_kernel, count, kNormThreads, 0, rt->stream, g, tensors, sumsq);
    HX_LAUNCHED(rt);
    ::hx::pdl_launch(clip_scale_kernel, 1, 32, 0, rt->stream, sumsq, count, threshold, norm_out, scale_out);
    HX_LAUNCHED(rt);
}

size_t muon_smem_bytes(int rows, int cols) {
    const int R = std::min(rows, cols), C = std::max(rows, cols);
    return sizeof(float) * (size_t(R) * C + 2 * size_t(R) * R);
}

void check_muon_shape(int rows, int cols) {
    const int R = std::min(rows, cols);
    require(rows > 0 && cols > 0, HX_ERR_ARGUMENT, "Muon: empty matrix");
    require(R <= 128 && rows * cols <= 16384, HX_ERR_UNSUPPORTED,
            "Muon: matrix " + std::to_string(rows) + "x" + std::to_string(cols) +
                " exceeds the single-CTA Newton-Schulz limit (shorter side <= 128, <= 16384 elements)");
}

// Whether every Muon matrix of a launch fits the tensor-core kernel (bf16
// operands, shorter side and longer side at most 128).
bool muon_tc_shape(int rows, int cols) {
    return std::max(rows, cols) <= kMuonTcMaxDim;
}

// Muon for `count` matrices: the tcgen05 kernel when the operands are bf16,
// every matrix fits it (`tc_shapes`) and the GEMM engine is not forced to
// the CUDA cores; the CUDA-core kernel otherwise (FP32 operands, larger
// matrices).
void launch_muon(hx_runtime* rt, const MuonMatrix* d_mats, int count, size_t smem, const MuonScalars& s,
                 const float* lr_dev = nullptr, bool tc_shapes = false) {
    if (count == 0) return;
    ProfScope prof(rt, kTagOptimizer, 0.0, 0.0);
    if (s.bf16 && tc_shapes && rt->gemm_backend != HX_GEMM_CUDA_CORES) {
        HX_CUDA(cudaFuncSetAttribute(muon_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)kMuonTcSmemBytes));
        ::hx::pdl_launch(muon_tc_kernel, count, kMuonTcThreads, kMuonTcSmemBytes, rt->stream, d_mats, s, lr_dev,
                                                                               rt->device_error());
        HX_LAUNCHED(rt);
        return;
    }
    HX_CUDA(cudaFuncSetAttribute(muon_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    ::hx::pdl_launch(muon_kernel, count, 1024, smem, rt->stream, d_mats, s, lr_dev);
    HX_LAUNCHED(rt);
}

}  // namespace hx

using namespace hx;

extern "C" {

int hx_adam_prepare(hx_runtime* rt, uint32_t elements) {
    return hx_guard(rt, [&] {
        require(elements > 0, HX_ERR_ARGUMENT, "Adam optimizer invalid runtime or shape");
        auto pl = std::make_unique<AdamPlan>();
        pl->n = elements;
        const size_t b = sizeof(float) * elements;
        pl->w = pl->arena.reserve(b);
        pl->g = pl->arena.reserve(b);
        pl->m = pl->arena.reserve(b);
        pl->v = pl->arena.reserve(b);
        for (auto& o : pl->out) o = pl->arena.reserve(b);
        pl->arena.commit();
        rt->adam = std::move(pl);
        ++rt->metrics.graph_create_count;
    });
}

static void validate_adam_scalars(float lr, float gs, float c1, float c2) {
    require(std::isfinite(lr) && std::isfinite(gs) && gs >= 0.0f && gs <= 1.0f && std::isfinite(c1) &&
                std::isfinite(c2),
            HX_ERR_ARGUMENT, "Adam optimizer buffer size or scalar");
}

int hx_adam_execute(hx_runtime* rt, const float* current, const float* gradient, const float* m, const float* v,
                    float lr, float gs, float c1, float c2, const hx_adam_outputs* out) {
    const auto t0 = Clock::now();
    const int rc = hx_guard(rt, [&] {
        require(rt->adam != nullptr, HX_ERR_STATE, "Adam optimizer graph not prepared");
        AdamPlan& pl = *rt->adam;
        require(current && gradient && m && v && out && out->w_next, HX_ERR_ARGUMENT, "Adam optimizer buffer size or scalar");
        validate_adam_scalars(lr, gs, c1, c2);
        const size_t n = pl.n, b = n * sizeof(float);
        const Arena& a = pl.arena;
        HX_CUDA(cudaMemcpyAsync(a.at<float>(pl.w), current, b, cudaMemcpyHostToDevice, rt->stream));
        HX_CUDA(cudaMemcpyAsync(a.at<float>(pl.g), gradient, b, cudaMemcpyHostToDevice, rt->stream));
        HX_CUDA(cudaMemcpyAsync(a.at<float>(pl.m), m, b, cudaMemcpyHostToDevice, rt->stream));
        HX_CUDA(cudaMemcpyAsync(a.at<float>(pl.v), v, b, cudaMemcpyHostToDevice, rt->stream));
        float* o[10];
        for (int i = 0; i < 10; ++i) o[i] = a.at<float>(pl.out[i]);
        // out order: m_next v_next m_hat v_hat sqrt_v_hat denominator divided normalized scaled_update w_next
        AdamTaps t{o[2], o[3], o[4], o[5], o[6], o[7], o[8]};
        launch_adam(rt, true, n, a.at<float>(pl.w), a.at<float>(pl.g), a.at<float>(pl.m), a.at<float>(pl.v), o[9], o[0],
                    o[1], adam_scalars(lr, gs, c1, c2), t);
        float* dst[10] = {out->m_next, out->v_next, out->m_hat, out->v_hat, out->sqrt_v_hat, out->denominator,
                          out->divided, out->normalized, out->scaled_update, out->w_next};
        for (int i = 0; i < 10; ++i)
            if (dst[i]) HX_CUDA(cudaMemcpyAsync(dst[i], o[i], b, cudaMemcpyDeviceToHost, rt->stream));
        HX_CUDA(cudaStreamSynchronize(rt->stream));
        if (rt->injected_now()) fail(HX_ERR_CUDA, "injected execute failure after device success");
    });
    if (rt) rt->record_execute(rc == HX_OK, us_since(t0));
    return rc;
}

int hx_adam_execute_device(hx_runtime* rt, size_t n, const float* current, const float* gradient, const float* m,
                           const float* v, float lr, float gs, float c1, float c2, const hx_adam_outputs* out) {
    return hx_guard(rt, [&] {
        require(current && gradient && m && v && out && out->w_next && out->m_next && out->v_next, HX_ERR_ARGUMENT,
                "Adam optimizer null buffer");
        validate_adam_scalars(lr, gs, c1, c2);
        const bool taps = out->m_hat || out->v_hat || out->sqrt_v_hat || out->denominator || out->divided ||
                          out->normalized || out->scaled_update;
        AdamTaps t{out->m_hat, out->v_hat, out->sqrt_v_hat, out->denominator, out->divided, out->normalized,
                   out->scaled_update};
        launch_adam(rt, taps, n, current, gradient, m, v, out->w_next, out->m_next, out->v_next,
                    adam_scalars(lr, gs, c1, c2), t);
    });
}

int hx_momentum_prepare(hx_runtime* rt, uint32_t elements) {
    return hx_guard(rt, [&] {
        require(elements > 0, HX_ERR_ARGUMENT, "momentum optimizer invalid runtime or shape");
        auto pl = std::make_unique<MomentumPlan>();
        pl->n = elements;
        const size_t b = sizeof(float) * elements;
        pl->w = pl->arena.reserve(b);
        pl->g = pl->arena.reserve(b);
        pl->vel = pl->arena.reserve(b);
        pl->vel_next = pl->arena.reserve(b);
        pl->w_next = pl->arena.reserve(b);
        pl->arena.commit();
        rt->momentum = std::move(pl);
        ++rt->metrics.graph_create_count;
        ++rt->metrics.graph_finalize_count;
    });
}

int hx_momentum_execute(hx_runtime* rt, const float* current, const float* gradient, const float* velocity,
                        float lr, float momentum, float* velocity_next, float* weight_next) {
    const auto t0 = Clock::now();
    const int rc = hx_guard(rt, [&] {
        require(rt->momentum != nullptr, HX_ERR_STATE, "momentum optimizer graph not prepared");
        const MomentumPlan& pl = *rt->momentum;
        require(current && gradient && velocity && velocity_next && weight_next && std::isfinite(lr) &&
                    std::isfinite(momentum),
                HX_ERR_ARGUMENT, "momentum optimizer buffer size or scalar");
        const size_t n = pl.n, b = n * sizeof(float);
        const Arena& a = pl.arena;
        HX_CUDA(cudaMemcpyAsync(a.at<float>(pl.w), current, b, cudaMemcpyHostToDevice, rt->stream));
        HX_CUDA(cudaMemcpyAsync(a.at<float>(pl.g), gradient, b, cudaMemcpyHostToDevice, rt->stream));
        HX_CUDA(cudaMemcpyAsync(a.at<float>(pl.vel), velocity, b, cudaMemcpyHostToDevice, rt->stream));
        launch_momentum(rt, n, a.at<float>(pl.w), a.at<float>(pl.g), a.at<float>(pl.vel), a.at<float>(pl.w_next),
                        a.at<float>(pl.vel_next), lr, momentum);
        HX_CUDA(cudaMemcpyAsync(velocity_next, a.at<float>(pl.vel_next), b, cudaMemcpyDeviceToHost, rt->stream));
        HX_CUDA(cudaMemcpyAsync(weight_next, a.at<float>(pl.w_next), b, cudaMemcpyDeviceToHost, rt->stream));
        HX_CUDA(cudaStreamSynchronize(rt->stream));
        if (rt->injected_now()) fail(HX_ERR_CUDA, "injected execute failure after device success");
    });
    if (rt) rt->record_execute(rc == HX_OK, us_since(t0));
    return rc;
}

int hx_momentum_execute_device(hx_runtime* rt, size_t n, const float* current, const float* gradient,
                               const float* velocity, float lr, float momentum, float* velocity_next,
                               float* weight_next) {
    return hx_guard(rt, [&] {
        require(current && gradient && velocity && velocity_next && weight_next && std::isfinite(lr) &&
                    std::isfinite(momentum),
                HX_ERR_ARGUMENT, "momentum optimizer buffer size or scalar");
        launch_momentum(rt, n, current, gradient, velocity, weight_next, velocity_next, lr, momentum);
    });
}

int hx_muon_execute(hx_runtime* rt, uint32_t rows, uint32_t cols, const float* weight, const float* gradient,
                    const float* buffer, float lr, float momentum, int nesterov, uint32_t ns_steps, float a, float b,
                    float c, int bf16, float* weight_next, float* buffer_next) {
    return hx_guard(rt, [&] {
        require(weight && gradient && buffer && weight_next && buffer_next, HX_ERR_ARGUMENT, "Muon: null buffer");
        check_muon_shape((int)rows, (int)cols);
        require(std::isfinite(lr) && std::isfinite(momentum), HX_ERR_ARGUMENT, "Muon: non-finite scalar");
        const size_t n = size_t(rows) * cols, bytes = n * sizeof(float);
        Arena arena;
        const size_t ow = arena.reserve(bytes), og = arena.reserve(bytes), ob = arena.reserve(bytes),
                     om = arena.reserve(sizeof(MuonMatrix));
        arena.commit();
        HX_CUDA(cudaMemcpyAsync(arena.at<float>(ow), weight, bytes, cudaMemcpyHostToDevice, rt->stream));
        HX_CUDA(cudaMemcpyAsync(arena.at<float>(og), gradient, bytes, cudaMemcpyHostToDevice, rt->stream));
        HX_CUDA(cudaMemcpyAsync(arena.at<float>(ob), buffer, bytes, cudaMemcpyHostToDevice, rt->stream));
        MuonMatrix mm{arena.at<float>(ow), arena.at<float>(og), arena.at<float>(ob), (int)rows, (int)cols};
        HX_CUDA(cudaMemcpyAsync(arena.at<MuonMatrix>(om), &mm, sizeof(mm), cudaMemcpyHostToDevice, rt->stream));
        MuonScalars s{lr, momentum, a, b, c, nesterov ? 1 : 0, (int)ns_steps, bf16 ? 1 : 0};
        launch_muon(rt, arena.at<MuonMatrix>(om), 1, muon_smem_bytes((int)rows, (int)cols), s, nullptr,
                    muon_tc_shape((int)rows, (int)cols));
        HX_CUDA(cudaMemcpyAsync(weight_next, arena.at<float>(ow), bytes, cudaMemcpyDeviceToHost, rt->stream));
        HX_CUDA(cudaMemcpyAsync(buffer_next, arena.at<float>(ob), bytes, cudaMemcpyDeviceToHost, rt->stream));
        rt->check_device_error();
    });
}

}  // extern "C"
