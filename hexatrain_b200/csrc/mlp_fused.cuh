// mlp_fused.cuh -- the whole MLP full step in one kernel for small shapes.
//
// At the reference's small configurations (B8 I128 H128 O64 and
// B32 I256 H256 O128) a step is 0.9-15 MFLOP: five GEMM launches and a
// reduction each cost more in launch and ramp latency than in arithmetic.
// Here one cluster of 16 CTAs (8 where the GPU does not allow the
// non-portable size) runs the step, exchanging the two
// intermediates every CTA needs (H, dP) through L2 with cluster barriers
// (release/acquire at cluster scope) between the phases:
//
//   phase 1  H[:, cols_c] = ReLU(X W1[:, cols_c])            (mask = H > 0)
//   phase 2  P[:, outs_c] = H W2[:, outs_c]; E = P - Y; dP = E * 2/(B*O);
//            this CTA's sum of E^2 in double
//   phase 3  dW2[cols_c, :] = H[:, cols_c]^T dP;  W2_next = W2 - lr*dW2
//            dH[:, cols_c] = dP W2[cols_c, :]^T;  dZ1 = (H > 0) ? dH : 0
//            CTA 0: loss = (sum of the CTA sums, in CTA order) / (B*O)
//   phase 4  dW1[:, cols_c] = X^T dZ1[:, cols_c];  W1_next = W1 - lr*dW1
//
// H, dP and the CTA sums cross CTAs through L2: they are read with
// ld.global.cg (L2 only) after the cluster barrier that orders them.  Each
// phase first stages its operands in shared memory with coalesced loads by
// all threads, then forms its dot products from shared memory.
// CTA c owns hidden columns cols_c (a contiguous H/8 slice) in phases 1, 3
// and 4, so dZ1 never leaves the CTA, and output columns outs_c in phase 2.
// Products accumulate in FP32 in k order; the elementwise nodes round as the
// GEMM epilogues do (E = P - Y, dP = E * s, W - lr*dW with two roundings).
#pragma once

#include "pdl.cuh"

#include "hx_internal.cuh"
#include "tc_ptx.cuh"

namespace hx {

constexpr int kMlpFusedCtas = 8;  // the portable cluster size; 16 where the GPU allows it
constexpr int kMlpFusedThreads = 512;

struct MlpFusedArgs {
    const float *x, *y, *w1, *w2;
    float *loss, *w1n, *w2n;
    float *h, *p, *e, *dp, *dw2, *dh, *dz1, *dw1;  // h, e, dp required (exchange); the rest optional
    uint8_t* mask;
    double* part;  // the cluster's per-CTA sums of E^2 (at most 16)
    float lr;
    int B, I, H, O;
};

// Shared-memory regions (floats): X for the whole step; A for W1's slice,
// then all of H, then all of dP; Bw for W2's output-column slice, then W2's
// rows of this CTA transposed; Hs for H's slice; Z for dZ1's slice.
constexpr int kMlpFusedX = 16384, kMlpFusedA = 16384, kMlpFusedB = 8192, kMlpFusedS = 4096;
constexpr size_t kMlpFusedSmemBytes = sizeof(float) * (kMlpFusedX + kMlpFusedA + kMlpFusedB + 2 * kMlpFusedS);

// Whether the fused step serves a shape: small enough that one cluster's
// CUDA cores beat five launches, and every staged operand fits its region.
inline bool mlp_fused_eligible(uint32_t B, uint32_t I, uint32_t H, uint32_t O) {
    const double flops = 2.0 * B * (2.0 * I * H + 3.0 * H * O);
    const size_t hc = (H + kMlpFusedCtas - 1) / kMlpFusedCtas, oc = (O + kMlpFusedCtas - 1) / kMlpFusedCtas;
    return flops <= 6.4e7 && size_t(B) * I <= kMlpFusedX && size_t(I) * hc <= kMlpFusedA &&
           size_t(B) * H <= kMlpFusedA && size_t(B) * O <= kMlpFusedA && size_t(H) * oc <= kMlpFusedB &&
           hc * O <= kMlpFusedB && size_t(B) * hc <= kMlpFusedS;
}

template <int CL>
__global__ void __cluster_dims__(CL, 1, 1) __launch_bounds__(kMlpFusedThreads, 1)
mlp_fused_step_kernel(MlpFusedArgs a)
{
    HX_PDL_PROLOGUE();
    extern __shared__ float4 smem4[];
    float* Xs = reinterpret_cast<float*>(smem4);
    float* As = Xs + kMlpFusedX;
    float* Bw = As + kMlpFusedA;
    float* Hs = Bw + kMlpFusedB;
    float* Zs = Hs + kMlpFusedS;
    __shared__ double red[kMlpFusedThreads / 32];
    const int c = int(tc::cluster_ctarank());
    const int tid = threadIdx.x, nt = blockDim.x;
    const int B = a.B, I = a.I, H = a.H, O = a.O;
    const int hc = (H + CL - 1) / CL, h0 = c * hc, h1 = min(H, h0 + hc);
    const int oc = (O + CL - 1) / CL, o0 = c * oc, o1 = min(O, o0 + oc);
    const int hn = max(0, h1 - h0), on = max(0, o1 - o0);

    // ---- phase 1: H = ReLU(X W1) on this CTA's hidden columns
    for (int i = tid; i < B * I; i += nt) Xs[i] = __ldg(a.x + i);
    for (int idx = tid; idx < I * hn; idx += nt) As[idx] = __ldg(a.w1 + (long)(idx / hn) * H + h0 + idx % hn);
    __syncthreads();
    for (int idx = tid; idx < B * hn; idx += nt) {
        const int b = idx / hn, jj = idx % hn;
        const float* xr = Xs + b * I;
        float z = 0.f;
        for (int i = 0; i < I; ++i) z = fmaf(xr[i], As[i * hn + jj], z);
        const float r = 0.f < z ? z : 0.f;
        const long g = (long)b * H + h0 + jj;
        a.h[g] = r;
        Hs[b * hn + jj] = r;
        if (a.mask) a.mask[g] = r > 0.f ? 1 : 0;
    }
    tc::cluster_sync();

    // ---- phase 2: P = H W2 on this CTA's output columns; E, dP, sum E^2
    for (int i = tid; i < B * H; i += nt) As[i] = __ldcg(a.h + i);
    for (int idx = tid; idx < H * on; idx += nt) Bw[idx] = __ldg(a.w2 + (long)(idx / on) * O + o0 + idx % on);
    __syncthreads();
    const float s = 2.0f / float(B * O);
    double se = 0.0;
    for (int idx = tid; idx < B * on; idx += nt) {
        const int b = idx / on, jj = idx % on;
        const float* hr = As + b * H;
        float p = 0.f;
        for (int k = 0; k < H; ++k) p = fmaf(hr[k], Bw[k * on + jj], p);
        const long i = (long)b * O + o0 + jj;
        const float err = __fsub_rn(p, __ldg(a.y + i));
        if (a.p) a.p[i] = p;
        a.e[i] = err;
        a.dp[i] = __fmul_rn(err, s);
        se += double(err) * err;
    }
    for (int o = 16; o > 0; o >>= 1) se += __shfl_xor_sync(0xffffffffu, se, o);
    if ((tid & 31) == 0) red[tid >> 5] = se;
    __syncthreads();
    if (tid == 0) {
        double t = 0.0;
        for (int w = 0; w < nt / 32; ++w) t += red[w];
        a.part[c] = t;
    }
    tc::cluster_sync();

    // ---- phase 3: dW2 and W2_next on rows h0..h1; dH and dZ1 on columns h0..h1
    if (c == 0 && tid == 0) {
        double t = 0.0;
        for (int q = 0; q < CL; ++q) t += __ldcg(a.part + q);
        *a.loss = float(t / double(B * O));
    }
    for (int i = tid; i < B * O; i += nt) As[i] = __ldcg(a.dp + i);
    for (int idx = tid; idx < hn * O; idx += nt) {  // W2's rows h0..h1, transposed: [j][jj]
        const int jj = idx / O, j = idx % O;
        Bw[j * hn + jj] = __ldg(a.w2 + (long)(h0 + jj) * O + j);
    }
    __syncthreads();
    for (int idx = tid; idx < hn * O; idx += nt) {
        const int jj = idx / O, j = idx % O;
        float g = 0.f;
        for (int b = 0; b < B; ++b) g = fmaf(Hs[b * hn + jj], As[b * O + j], g);
        const long i = (long)(h0 + jj) * O + j;
        if (a.dw2) a.dw2[i] = g;
        a.w2n[i] = __fsub_rn(Bw[j * hn + jj], __fmul_rn(a.lr, g));
    }
    for (int idx = tid; idx < B * hn; idx += nt) {
        const int b = idx / hn, jj = idx % hn;
        const float* dpr = As + b * O;
        float g = 0.f;
        for (int j = 0; j < O; ++j) g = fmaf(dpr[j], Bw[j * hn + jj], g);
        const float z = Hs[b * hn + jj] > 0.f ? g : 0.f;
        const long i = (long)b * H + h0 + jj;
        if (a.dh) a.dh[i] = g;
        if (a.dz1) a.dz1[i] = z;
        Zs[b * hn + jj] = z;
    }
    __syncthreads();

    // ---- phase 4: dW1 and W1_next on columns h0..h1
    for (int idx = tid; idx < I * hn; idx += nt) {
        const int i = idx / hn, jj = idx % hn;
        float g = 0.f;
        for (int b = 0; b < B; ++b) g = fmaf(Xs[b * I + i], Zs[b * hn + jj], g);
        const long w = (long)i * H + h0 + jj;
        if (a.dw1) a.dw1[w] = g;
        a.w1n[w] = __fsub_rn(__ldg(a.w1 + w), __fmul_rn(a.lr, g));
    }
}

}  // namespace hx
