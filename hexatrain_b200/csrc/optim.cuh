// optim.cuh -- optimizer kernels: elementwise Adam (HBM-bound, 128-bit
// accesses) and Muon's momentum + Newton-Schulz orthogonalisation.
#pragma once

#include "pdl.cuh"

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace hx {

struct AdamScalars {
    float lr, gradient_scale, c1, c2, beta1, beta2, one_minus_beta1, one_minus_beta2, eps;
};

// Optional outputs of the reference's Adam graph
// (qnn/qnn_runtime_transformer.inc:926-1109), any may be null.
struct AdamTaps {
    float *m_hat, *v_hat, *sqrt_v_hat, *denominator, *divided, *normalized, *scaled_update;
};

// kGraphOrder selects the rounding order:
//   false: tiny_lm::adamUpdate (tiny_language_model_cpu.cpp:137):
//          w' = w - (lr*m^)/(sqrt(v^)+eps)
//   true:  the QNN graph: div = m^/den; norm = (v^>0)?div:0; w' = w - lr*norm
// Both share m', v', m^, v^.  In-place operation (w_next == w, m_next == m,
// v_next == v) is allowed: each element is read before it is written.
template <bool kGraphOrder>
__device__ __forceinline__ float adam_element(float w, float g, float& m, float& v, const AdamScalars& s,
                                              const AdamTaps& t, size_t i)
{
    const float gs = __fmul_rn(g, s.gradient_scale);
    const float nm = __fadd_rn(__fmul_rn(s.beta1, m), __fmul_rn(s.one_minus_beta1, gs));
    const float nv = __fadd_rn(__fmul_rn(s.beta2, v), __fmul_rn(__fmul_rn(s.one_minus_beta2, gs), gs));
    const float mh = __fmul_rn(nm, s.c1);
    const float vh = __fmul_rn(nv, s.c2);
    const float root = __fsqrt_rn(vh);
    const float den = __fadd_rn(root, s.eps);
    m = nm;
    v = nv;
    if (kGraphOrder) {
        const float div = __fdiv_rn(mh, den);
        const float norm = vh > 0.f ? div : 0.f;
        const float upd = __fmul_rn(s.lr, norm);
        if (t.m_hat) t.m_hat[i] = mh;
        if (t.v_hat) t.v_hat[i] = vh;
        if (t.sqrt_v_hat) t.sqrt_v_hat[i] = root;
        if (t.denominator) t.denominator[i] = den;
        if (t.divided) t.divided[i] = div;
        if (t.normalized) t.normalized[i] = norm;
        if (t.scaled_update) t.scaled_update[i] = upd;
        return __fsub_rn(w, upd);
    }
    return __fsub_rn(w, __fdiv_rn(__fmul_rn(s.lr, mh), den));
}

template <bool kGraphOrder>
__global__ void adam_kernel(size_t n, const float* w, const float* __restrict__ g, const float* m,
                            const float* v, float* w_next, float* m_next, float* v_next, AdamScalars s,
                            AdamTaps t, const float* __restrict__ scale_dev, const AdamScalars* __restrict__ s_dev)
{
    HX_PDL_PROLOGUE();
    // Scalars in device memory (a captured training step, whose learning
    // rate and bias corrections change every step) replace the by-value
    // ones; a gradient scale computed on the device (the global-norm clip)
    // replaces the host scalar when given.
    if (s_dev) s = *s_dev;
    if (scale_dev) s.gradient_scale = *scale_dev;
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    const size_t tid = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    const bool vec = !kGraphOrder &&
                     ((reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(g) | reinterpret_cast<uintptr_t>(m) |
                       reinterpret_cast<uintptr_t>(v) | reinterpret_cast<uintptr_t>(w_next) |
                       reinterpret_cast<uintptr_t>(m_next) | reinterpret_cast<uintptr_t>(v_next)) & 15) == 0;
    size_t done = 0;
    if (vec) {
        const size_t n4 = n / 4;
        for (size_t i = tid; i < n4; i += stride) {
            float4 wv = reinterpret_cast<const float4*>(w)[i];
            const float4 gv = reinterpret_cast<const float4*>(g)[i];
            float4 mv = reinterpret_cast<const float4*>(m)[i];
            float4 vv = reinterpret_cast<const float4*>(v)[i];
            wv.x = adam_element<false>(wv.x, gv.x, mv.x, vv.x, s, t, 0);
            wv.y = adam_element<false>(wv.y, gv.y, mv.y, vv.y, s, t, 0);
            wv.z = adam_element<false>(wv.z, gv.z, mv.z, vv.z, s, t, 0);
            wv.w = adam_element<false>(wv.w, gv.w, mv.w, vv.w, s, t, 0);
            reinterpret_cast<float4*>(w_next)[i] = wv;
            reinterpret_cast<float4*>(m_next)[i] = mv;
            reinterpret_cast<float4*>(v_next)[i] = vv;
        }
        done = n4 * 4;
    }
    for (size_t i = done + tid; i < n; i += stride) {
        float mm = m[i], vv = v[i];
        const float wn = adam_element<kGraphOrder>(w[i], g[i], mm, vv, s, t, i);
        w_next[i] = wn;
        m_next[i] = mm;
        v_next[i] = vv;
    }
}

// ---- momentum SGD -----------------------------------------------------------
// The reference's momentum graph (qnn/qnn_runtime_transformer.inc:799-881):
//   scaled = velocity * momentum; velocity' = scaled + gradient;
//   update = velocity' * lr;      w' = w - update
// (tiny_lm::momentumUpdate, tiny_language_model_cpu.cpp:123, rounds the
// same products).  In place is allowed.
__global__ void momentum_kernel(size_t n, const float* w, const float* __restrict__ g, const float* vel,
                                float* w_next, float* vel_next, float lr, float momentum,
                                const float* __restrict__ lr_dev);

// Per-step scalars of the LM optimizer step, read from device memory so that
// a captured step graph replays with each step's values: Adam's learning
// rate and bias corrections, and the scheduled momentum and Muon rates.
struct LmStepScalars {
    AdamScalars adam;
    float momentum_lr, muon_lr;
};

// ---- global gradient norm and clip scale ----------------------------------
// gradientNorm (qnn/qnn_transformer_training.cpp:888-938): per tensor the
// double sum of squares, its square root, then sqrt(sum of squared norms)
// in the reference's tensor order; clip scale = min(1, threshold /
// (norm + 1e-6)) when the norm is finite and positive, else 1
// (:2432-2439).  One CTA per tensor, a fixed reduction tree, so results do
// not depend on scheduling.
struct GradTensor {
    unsigned long long offset, count;
};
__global__ void grad_sumsq_kernel(const float* __restrict__ g, const GradTensor* __restrict__ tensors,
                                  double* __restrict__ sumsq);
__global__ void clip_scale_kernel(const double* __restrict__ sumsq, int tensors, float threshold,
                                  double* __restrict__ norm_out, float* __restrict__ scale_out);

// ---- Muon -----------------------------------------------------------------

struct MuonMatrix {
    float* w;          // weight, updated in place
    const float* g;    // gradient
    float* buf;        // momentum buffer, updated in place
    int rows, cols;
};

struct MuonScalars {
    float lr, momentum, a, b, c;
    int nesterov, steps, bf16;
};

__device__ __forceinline__ float muon_operand(float x, int bf16) {
    return bf16 ? __bfloat162float(__float2bfloat16_rn(x)) : x;
}

// Momentum + Newton-Schulz for a batch of matrices, one CTA each (optim.cu).
// lr_dev, when given, replaces s.lr.
__global__ void muon_kernel(const MuonMatrix* __restrict__ mats, MuonScalars s, const float* __restrict__ lr_dev);

}  // namespace hx
