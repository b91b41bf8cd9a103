// lm_kernels.cuh -- device kernels of the tiny-Transformer LM step.
//
// Rows are r = b*T + t over a batch of B sequences (the reference runs one
// sequence per graph execute; here the batch is folded into the row index of
// every kernel).  Reference lines are cited per kernel
// (tiny_language_model_cpu.cpp unless noted).
#pragma once

#include "pdl.cuh"

#include <cuda_runtime.h>
#include <cstdint>

namespace hx {

__device__ __forceinline__ float warp_max(float v) {
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ double warp_sum(double v) {
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_sumf(float v) {
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// tokens [B, T+1] -> input ids / target ids [B*T].  Any id >= V sets *bad.
__global__ void split_tokens_kernel(int B, int T, int V, const uint32_t* __restrict__ tokens,
                                    int* __restrict__ in_ids, int* __restrict__ tgt_ids, int* bad)
{
    HX_PDL_PROLOGUE();
    const int M = B * T;
    for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < M; r += gridDim.x * blockDim.x) {
        const int b = r / T, t = r % T;
        const uint32_t a = tokens[(size_t)b * (T + 1) + t], y = tokens[(size_t)b * (T + 1) + t + 1];
        if (a >= (uint32_t)V || y >= (uint32_t)V) atomicExch(bad, 1);
        in_ids[r] = a < (uint32_t)V ? (int)a : 0;
        tgt_ids[r] = y < (uint32_t)V ? (int)y : 0;
    }
}

// ids given directly [M] (validated the same way).
__global__ void copy_ids_kernel(int M, int V, const uint32_t* __restrict__ a, const uint32_t* __restrict__ y,
                                int* __restrict__ in_ids, int* __restrict__ tgt_ids, int* bad)
{
    HX_PDL_PROLOGUE();
    for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < M; r += gridDim.x * blockDim.x) {
        if (a[r] >= (uint32_t)V || y[r] >= (uint32_t)V) atomicExch(bad, 1);
        in_ids[r] = a[r] < (uint32_t)V ? (int)a[r] : 0;
        tgt_ids[r] = y[r] < (uint32_t)V ? (int)y[r] : 0;
    }
}

// x0[r,:] = E[id[r],:] + pos[t,:]   (:42 -- one-hot * E selects a row exactly)
__global__ void embed_kernel(int M, int T, int D, const int* __restrict__ ids, const float* __restrict__ E,
                             const float* __restrict__ pos, float* __restrict__ x)
{
    HX_PDL_PROLOGUE();
    const long total = (long)M * D;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
        const int r = (int)(i / D), d = (int)(i % D);
        x[i] = __fadd_rn(E[(long)ids[r] * D + d], pos[(long)(r % T) * D + d]);
    }
}

// The same sum four columns at a time when D % 4 == 0, every base pointer is
// 16-byte aligned and M * D / 4 fits an int: 32-bit index arithmetic and
// 16-byte loads and stores, so the kernel runs at the rate of its 4*M*D
// written bytes instead of its 64-bit divisions.
__global__ void embed_vec_kernel(int M, int T, int D4, const int* __restrict__ ids,
                                 const float4* __restrict__ E, const float4* __restrict__ pos,
                                 float4* __restrict__ x)
{
    HX_PDL_PROLOGUE();
    const int total = M * D4;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
        const int r = i / D4, d = i - r * D4;
        const float4 e = E[(long)ids[r] * D4 + d];
        const float4 q = pos[(r % T) * D4 + d];
        x[i] = make_float4(__fadd_rn(e.x, q.x), __fadd_rn(e.y, q.y), __fadd_rn(e.z, q.z), __fadd_rn(e.w, q.w));
    }
}

// LayerNorm forward, one warp per row (nf, :36): mean and variance in
// double, inv = float(1/sqrt(var+eps)), xhat = (x - float(mean))*inv,
// y = xhat*gamma + beta.  Saves float(mean) and inv for the backward pass.
__global__ void layernorm_fwd_kernel(int M, int D, float eps, const float* __restrict__ x,
                                     const float* __restrict__ g, const float* __restrict__ b,
                                     float* __restrict__ y, float* __restrict__ mean_out, float* __restrict__ inv_out)
{
    HX_PDL_PROLOGUE();
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (row >= M) return;
    const float* xr = x + (long)row * D;
    double s = 0.0;
    for (int d = lane; d < D; d += 32) s += xr[d];
    const double m = warp_sum(s) / D;
    double v = 0.0;
    for (int d = lane; d < D; d += 32) {
        const double z = xr[d] - m;
        v += z * z;
    }
    v = warp_sum(v) / D;
    const float inv = (float)(1.0 / sqrt(v + (double)eps));
    const float mf = (float)m;
    float* yr = y + (long)row * D;
    for (int d = lane; d < D; d += 32) {
        const float xh = __fmul_rn(__fsub_rn(xr[d], mf), inv);
        yr[d] = __fadd_rn(__fmul_rn(xh, g[d]), b[d]);
    }
    if (lane == 0) {
        mean_out[row] = mf;
        inv_out[row] = inv;
    }
}

// The same for D = 128 C with the row in registers: lane l owns columns
// 128k + 4l .. +3 (k < C), so the row is read once, as C float4 loads, and
// written once.  The double sums are of the same terms as above, in another
// order.
template <int C>
__global__ void layernorm_fwd_vec_kernel(int M, float eps, const float* __restrict__ x, const float* __restrict__ g,
                                         const float* __restrict__ b, float* __restrict__ y,
                                         float* __restrict__ mean_out, float* __restrict__ inv_out)
{
    HX_PDL_PROLOGUE();
    constexpr int D = 128 * C;
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (row >= M) return;
    const float* xr = x + (long)row * D;
    float xv[4 * C];
#pragma unroll
    for (int k = 0; k < C; ++k) {
        const float4 a = *reinterpret_cast<const float4*>(xr + 128 * k + 4 * lane);
        xv[4 * k] = a.x; xv[4 * k + 1] = a.y; xv[4 * k + 2] = a.z; xv[4 * k + 3] = a.w;
    }
    double s = 0.0;
#pragma unroll
    for (int i = 0; i < 4 * C; ++i) s += xv[i];
    const double m = warp_sum(s) / D;
    double v = 0.0;
#pragma unroll
    for (int i = 0; i < 4 * C; ++i) {
        const double z = xv[i] - m;
        v += z * z;
    }
    v = warp_sum(v) / D;
    const float inv = (float)(1.0 / sqrt(v + (double)eps));
    const float mf = (float)m;
    float* yr = y + (long)row * D;
#pragma unroll
    for (int k = 0; k < C; ++k) {
        const float4 gg = *reinterpret_cast<const float4*>(g + 128 * k + 4 * lane);
        const float4 bb = *reinterpret_cast<const float4*>(b + 128 * k + 4 * lane);
        const float gv[4] = {gg.x, gg.y, gg.z, gg.w}, bv[4] = {bb.x, bb.y, bb.z, bb.w};
        float o[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float xh = __fmul_rn(__fsub_rn(xv[4 * k + e], mf), inv);
            o[e] = __fadd_rn(__fmul_rn(xh, gv[e]), bv[e]);
        }
        *reinterpret_cast<float4*>(yr + 128 * k + 4 * lane) = make_float4(o[0], o[1], o[2], o[3]);
    }
    if (lane == 0) {
        mean_out[row] = mf;
        inv_out[row] = inv;
    }
}

// LayerNorm backward fused with the residual add (nb, :37, and "dr = dout +
// drn" of :79): dx = res + inv/D*(D*z - sum z - xhat*sum(z*xhat)), z=dy*g.
// Also writes per-CTA partial column sums of dy*xhat (dgamma) and dy
// (dbeta) to part[blockIdx.x][2][D]; column_reduce finishes them.
// Each CTA handles rows [blockIdx.x*rows_per_cta, ...).
__global__ void layernorm_bwd_kernel(int M, int D, int rows_per_cta, const float* __restrict__ dy,
                                     const float* __restrict__ x, const float* __restrict__ mean,
                                     const float* __restrict__ inv, const float* __restrict__ g,
                                     const float* __restrict__ res, float* __restrict__ dx,
                                     float* __restrict__ part)
{
    HX_PDL_PROLOGUE();
    extern __shared__ float acc[];  // [warps][2][D]
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    float* ga = acc + (size_t)warp * 2 * D;
    float* ba = ga + D;
    for (int d = lane; d < D; d += 32) { ga[d] = 0.f; ba[d] = 0.f; }
    const int r0 = blockIdx.x * rows_per_cta;
    const int r1 = min(M, r0 + rows_per_cta);
    for (int row = r0 + warp; row < r1; row += nw) {
        const float* dyr = dy + (long)row * D;
        const float* xr = x + (long)row * D;
        const float mf = mean[row], iv = inv[row];
        double s = 0.0, sx = 0.0;
        for (int d = lane; d < D; d += 32) {
            const float xh = __fmul_rn(__fsub_rn(xr[d], mf), iv);
            const double z = __fmul_rn(dyr[d], g[d]);
            s += z;
            sx += z * xh;
            ga[d] = __fadd_rn(ga[d], __fmul_rn(dyr[d], xh));
            ba[d] = __fadd_rn(ba[d], dyr[d]);
        }
        s = warp_sum(s);
        sx = warp_sum(sx);
        const float ivd = __fdiv_rn(iv, (float)D);
        for (int d = lane; d < D; d += 32) {
            const float xh = __fmul_rn(__fsub_rn(xr[d], mf), iv);
            const double z = __fmul_rn(dyr[d], g[d]);
            const float v = (float)((double)ivd * ((double)D * z - s - (double)xh * sx));
            const long i = (long)row * D + d;
            dx[i] = res ? __fadd_rn(res[i], v) : v;
        }
    }
    __syncthreads();
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
        float sg = 0.f, sb = 0.f;
        for (int w = 0; w < nw; ++w) {
            sg += acc[(size_t)w * 2 * D + d];
            sb += acc[(size_t)w * 2 * D + D + d];
        }
        part[((size_t)blockIdx.x * 2) * D + d] = sg;
        part[((size_t)blockIdx.x * 2 + 1) * D + d] = sb;
    }
}

// The same for D = 128 C: lane l owns columns 128k + 4l .. +3 (k < C), so a
// row moves as C float4 loads per operand, the row stays in registers
// between the two reductions, and each lane keeps its columns' dgamma /
// dbeta partials in registers (rows of the warp in the same order as above,
// so the partials, summed across warps in warp order, are identical).  The
// row sums s and sx are double sums of the same terms in another order.
template <int C>
__global__ void layernorm_bwd_vec_kernel(int M, int rows_per_cta, const float* __restrict__ dy,
                                         const float* __restrict__ x, const float* __restrict__ mean,
                                         const float* __restrict__ inv, const float* __restrict__ g,
                                         const float* __restrict__ res, float* __restrict__ dx,
                                         float* __restrict__ part)
{
    HX_PDL_PROLOGUE();
    constexpr int D = 128 * C;
    extern __shared__ float acc[];  // [warps][2][D]
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    float gl[4 * C], ga[4 * C], ba[4 * C];
#pragma unroll
    for (int k = 0; k < C; ++k) {
        const float4 v = *reinterpret_cast<const float4*>(g + 128 * k + 4 * lane);
        gl[4 * k] = v.x; gl[4 * k + 1] = v.y; gl[4 * k + 2] = v.z; gl[4 * k + 3] = v.w;
    }
#pragma unroll
    for (int i = 0; i < 4 * C; ++i) { ga[i] = 0.f; ba[i] = 0.f; }
    const int r0 = blockIdx.x * rows_per_cta;
    const int r1 = min(M, r0 + rows_per_cta);
    const float ivd_scale = float(D);
    for (int row = r0 + warp; row < r1; row += nw) {
        const long base = (long)row * D;
        // dy, x and the residual of the row are loaded together: one round
        // trip to memory per row
        float dyv[4 * C], xv[4 * C], rv[4 * C];
#pragma unroll
        for (int k = 0; k < C; ++k) {
            const float4 a = *reinterpret_cast<const float4*>(dy + base + 128 * k + 4 * lane);
            const float4 b = *reinterpret_cast<const float4*>(x + base + 128 * k + 4 * lane);
            const float4 r = res ? *reinterpret_cast<const float4*>(res + base + 128 * k + 4 * lane)
                                 : make_float4(0.f, 0.f, 0.f, 0.f);
            dyv[4 * k] = a.x; dyv[4 * k + 1] = a.y; dyv[4 * k + 2] = a.z; dyv[4 * k + 3] = a.w;
            xv[4 * k] = b.x; xv[4 * k + 1] = b.y; xv[4 * k + 2] = b.z; xv[4 * k + 3] = b.w;
            rv[4 * k] = r.x; rv[4 * k + 1] = r.y; rv[4 * k + 2] = r.z; rv[4 * k + 3] = r.w;
        }
        const float mf = mean[row], iv = inv[row];
        double s = 0.0, sx = 0.0;
#pragma unroll
        for (int i = 0; i < 4 * C; ++i) {
            const float xh = __fmul_rn(__fsub_rn(xv[i], mf), iv);
            xv[i] = xh;
            const double z = __fmul_rn(dyv[i], gl[i]);
            s += z;
            sx += z * xh;
            ga[i] = __fadd_rn(ga[i], __fmul_rn(dyv[i], xh));
            ba[i] = __fadd_rn(ba[i], dyv[i]);
        }
        s = warp_sum(s);
        sx = warp_sum(sx);
        const float ivd = __fdiv_rn(iv, ivd_scale);
#pragma unroll
        for (int k = 0; k < C; ++k) {
            float o[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int i = 4 * k + e;
                const double z = __fmul_rn(dyv[i], gl[i]);
                o[e] = (float)((double)ivd * ((double)D * z - s - (double)xv[i] * sx));
            }
            const long off = base + 128 * k + 4 * lane;
            if (res) {
#pragma unroll
                for (int e = 0; e < 4; ++e) o[e] = __fadd_rn(rv[4 * k + e], o[e]);
            }
            *reinterpret_cast<float4*>(dx + off) = make_float4(o[0], o[1], o[2], o[3]);
        }
    }
    float* wa = acc + (size_t)warp * 2 * D;
#pragma unroll
    for (int k = 0; k < C; ++k)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            wa[128 * k + 4 * lane + e] = ga[4 * k + e];
            wa[D + 128 * k + 4 * lane + e] = ba[4 * k + e];
        }
    __syncthreads();
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
        float sg = 0.f, sb = 0.f;
        for (int w = 0; w < nw; ++w) {
            sg += acc[(size_t)w * 2 * D + d];
            sb += acc[(size_t)w * 2 * D + D + d];
        }
        part[((size_t)blockIdx.x * 2) * D + d] = sg;
        part[((size_t)blockIdx.x * 2 + 1) * D + d] = sb;
    }
}

// out[c] = sum over parts p of part[p][which][c].  A CTA takes 32 columns
// (lane = column, so every load is a 128-byte segment); warp w sums parts
// w, w + 32, w + 64, ... and the 32 warp sums are added in warp order, so
// the result does not depend on timing.
constexpr int kColReduceWarps = 32;
__global__ void __launch_bounds__(32 * kColReduceWarps)
column_reduce_kernel(int parts, int D, const float* __restrict__ part, float* __restrict__ dgamma,
                     float* __restrict__ dbeta)
{
    HX_PDL_PROLOGUE();
    __shared__ float red[kColReduceWarps][32];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int c = blockIdx.x * 32 + lane;
    const bool ok = c < 2 * D;
    const int which = ok ? c / D : 0, d = ok ? c % D : 0;
    float s = 0.f;
    if (ok) {
        const float* src = part + (size_t)which * D + d;
#pragma unroll 4
        for (int p = w; p < parts; p += kColReduceWarps) s += src[(size_t)p * 2 * D];
    }
    red[w][lane] = s;
    __syncthreads();
    if (w == 0 && ok) {
        float t = red[0][lane];
#pragma unroll
        for (int i = 1; i < kColReduceWarps; ++i) t += red[i][lane];
        (which ? dbeta : dgamma)[d] = t;
    }
}

// ---- causal attention ------------------------------------------------------
// qkv: [M, 3D] with q at columns [0,D), k at [D,2D), v at [2D,3D); head h
// owns columns h*dh .. h*dh+dh-1 of each.  One CTA per (head, sequence).

template <int DH>
__device__ __forceinline__ float dot_dh(const float* a, const float* b) {
    float s = 0.f;
#pragma unroll
    for (int d = 0; d < DH; ++d) s = fmaf(a[d], b[d], s);
    return s;
}

// Forward (:44-45): p = softmax_j<=r(q_r.k_j * scale); ctx_r = sum p_j v_j.
// Saves the row max and the row sum (as float) so the backward pass can
// recompute p exactly; writes full P rows (zeros above the diagonal) only
// when probs != nullptr.
template <int DH>
__global__ void attention_fwd_kernel(int T, int D, int H, float scale, const float* __restrict__ qkv,
                                     float* __restrict__ ctx, float* __restrict__ row_max, float* __restrict__ row_sum,
                                     float* __restrict__ probs)
{
    HX_PDL_PROLOGUE();
    extern __shared__ float sm[];
    const int h = blockIdx.x, b = blockIdx.y;
    const int nw = blockDim.x >> 5, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    constexpr int LD = DH + 1;
    float* Ks = sm;                      // [T][LD]
    float* Vs = Ks + T * LD;             // [T][LD]
    float* Ps = Vs + T * LD;             // [nw][T]
    float* Qs = Ps + nw * T;             // [nw][DH]
    const long rowbase = (long)b * T;
    const int ld = 3 * D;
    for (int i = threadIdx.x; i < T * DH; i += blockDim.x) {
        const int j = i / DH, d = i % DH;
        const float* src = qkv + (rowbase + j) * ld + h * DH + d;
        Ks[j * LD + d] = src[D];
        Vs[j * LD + d] = src[2 * D];
    }
    __syncthreads();
    float* pw = Ps + warp * T;
    float* qw = Qs + warp * DH;
    for (int r = warp; r < T; r += nw) {
        for (int d = lane; d < DH; d += 32) qw[d] = qkv[(rowbase + r) * ld + h * DH + d];
        __syncwarp();
        float mx = -INFINITY;
        for (int j = lane; j <= r; j += 32) {
            const float s = __fmul_rn(dot_dh<DH>(qw, Ks + j * LD), scale);
            pw[j] = s;
            mx = fmaxf(mx, s);
        }
        mx = warp_max(mx);
        double sum = 0.0;
        for (int j = lane; j <= r; j += 32) {
            const float e = expf(__fsub_rn(pw[j], mx));
            pw[j] = e;
            sum += e;
        }
        const float sumf = (float)warp_sum(sum);
        for (int j = lane; j <= r; j += 32) pw[j] = __fdiv_rn(pw[j], sumf);
        __syncwarp();
        if (probs) {
            float* prow = probs + (((long)b * H + h) * T + r) * T;
            for (int j = lane; j < T; j += 32) prow[j] = j <= r ? pw[j] : 0.f;
        }
        for (int d = lane; d < DH; d += 32) {
            float acc = 0.f;
            for (int j = 0; j <= r; ++j) acc = fmaf(pw[j], Vs[j * LD + d], acc);
            ctx[(rowbase + r) * D + h * DH + d] = acc;
        }
        if (lane == 0) {
            row_max[((long)b * H + h) * T + r] = mx;
            row_sum[((long)b * H + h) * T + r] = sumf;
        }
        __syncwarp();
    }
}

// Backward (:80-81).  With p recomputed from the saved row statistics:
//   dP_rj = dc_r . v_j ; dot_r = sum_j dP_rj p_rj (double) ;
//   dS_rj = p_rj (dP_rj - dot_r) ;
//   dq_r = scale sum_j dS_rj k_j ; dk_j = scale sum_r dS_rj q_r ;
//   dv_j = sum_r p_rj dc_r .
// Phase 1 walks rows (dq, dot_r); phase 2 walks columns (dk, dv), lanes
// spread over r, each lane accumulating DH-wide partials in registers.
template <int DH>
__global__ void attention_bwd_kernel(int T, int D, int H, float scale, const float* __restrict__ qkv,
                                     const float* __restrict__ dctx, const float* __restrict__ row_max,
                                     const float* __restrict__ row_sum, float* __restrict__ dqkv)
{
    HX_PDL_PROLOGUE();
    extern __shared__ float sm[];
    const int h = blockIdx.x, b = blockIdx.y;
    const int nw = blockDim.x >> 5, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    constexpr int LD = DH + 1;
    float* Qs = sm;                 // [T][LD]
    float* Ks = Qs + T * LD;
    float* Vs = Ks + T * LD;
    float* Cs = Vs + T * LD;        // dctx head slice
    float* dot = Cs + T * LD;       // [T]
    float* mxs = dot + T;           // [T]
    float* sms = mxs + T;           // [T]
    float* Sw = sms + T;            // [nw][T]
    const long rowbase = (long)b * T;
    const int ld = 3 * D;
    for (int i = threadIdx.x; i < T * DH; i += blockDim.x) {
        const int j = i / DH, d = i % DH;
        const float* src = qkv + (rowbase + j) * ld + h * DH + d;
        Qs[j * LD + d] = src[0];
        Ks[j * LD + d] = src[D];
        Vs[j * LD + d] = src[2 * D];
        Cs[j * LD + d] = dctx[(rowbase + j) * D + h * DH + d];
    }
    for (int i = threadIdx.x; i < T; i += blockDim.x) {
        mxs[i] = row_max[((long)b * H + h) * T + i];
        sms[i] = row_sum[((long)b * H + h) * T + i];
    }
    __syncthreads();
    float* sw = Sw + warp * T;
    // phase 1: rows
    for (int r = warp; r < T; r += nw) {
        const float* qr = Qs + r * LD;
        const float* cr = Cs + r * LD;
        double dsum = 0.0;
        for (int j = lane; j <= r; j += 32) {
            const float p = __fdiv_rn(expf(__fsub_rn(__fmul_rn(dot_dh<DH>(qr, Ks + j * LD), scale), mxs[r])), sms[r]);
            const float dp = dot_dh<DH>(cr, Vs + j * LD);
            sw[j] = dp;
            dsum += (double)__fmul_rn(dp, p);
        }
        const float dt = (float)warp_sum(dsum);
        for (int j = lane; j <= r; j += 32) {
            const float p = __fdiv_rn(expf(__fsub_rn(__fmul_rn(dot_dh<DH>(qr, Ks + j * LD), scale), mxs[r])), sms[r]);
            sw[j] = __fmul_rn(p, __fsub_rn(sw[j], dt));
        }
        __syncwarp();
        for (int d = lane; d < DH; d += 32) {
            float acc = 0.f;
            for (int j = 0; j <= r; ++j) acc = fmaf(sw[j], Ks[j * LD + d], acc);
            dqkv[(rowbase + r) * ld + h * DH + d] = acc * scale;
        }
        if (lane == 0) dot[r] = dt;
        __syncwarp();
    }
    __syncthreads();
    // phase 2: columns
    for (int j = warp; j < T; j += nw) {
        float dk[DH], dv[DH];
#pragma unroll
        for (int d = 0; d < DH; ++d) { dk[d] = 0.f; dv[d] = 0.f; }
        const float* kj = Ks + j * LD;
        const float* vj = Vs + j * LD;
        for (int r = j + lane; r < T; r += 32) {
            const float* qr = Qs + r * LD;
            const float* cr = Cs + r * LD;
            const float p = __fdiv_rn(expf(__fsub_rn(__fmul_rn(dot_dh<DH>(qr, kj), scale), mxs[r])), sms[r]);
            const float ds = __fmul_rn(p, __fsub_rn(dot_dh<DH>(cr, vj), dot[r]));
#pragma unroll
            for (int d = 0; d < DH; ++d) {
                dk[d] = fmaf(ds, qr[d], dk[d]);
                dv[d] = fmaf(p, cr[d], dv[d]);
            }
        }
#pragma unroll
        for (int d = 0; d < DH; ++d) {
            const float sk = warp_sumf(dk[d]);
            const float sv = warp_sumf(dv[d]);
            if (lane == 0) {
                dqkv[(rowbase + j) * ld + D + h * DH + d] = sk * scale;
                dqkv[(rowbase + j) * ld + 2 * D + h * DH + d] = sv;
            }
        }
    }
}

// ---- cross-entropy ------------------------------------------------------------
// One warp per row (:48 softmax, :77 loss/dLogits): max over the row (first
// index of the max is the prediction), e = exp(l - max), s = sum e in
// double, p = e / float(s), dlogits = (p - onehot)/T * scale (in place over
// logits is allowed), row loss = max + log(s) - l[target] in double.
__global__ void softmax_ce_kernel(int M, int V, int T, float scale, float* logits, const int* __restrict__ tgt,
                                  float* __restrict__ probs, float* dlogits, double* __restrict__ row_loss,
                                  int* __restrict__ row_correct)
{
    HX_PDL_PROLOGUE();
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (row >= M) return;
    float* l = logits + (long)row * V;
    float mx = -INFINITY;
    int arg = 0x7fffffff;
    for (int j = lane; j < V; j += 32) {
        const float v = l[j];
        if (v > mx || (v == mx && j < arg)) { mx = v; arg = j; }
    }
    for (int o = 16; o > 0; o >>= 1) {
        const float om = __shfl_xor_sync(0xffffffffu, mx, o);
        const int oa = __shfl_xor_sync(0xffffffffu, arg, o);
        if (om > mx || (om == mx && oa < arg)) { mx = om; arg = oa; }
    }
    double s = 0.0;
    for (int j = lane; j < V; j += 32) s += (double)expf(l[j] - mx);
    s = warp_sum(s);
    const float sf = (float)s;
    const int y = tgt[row];
    const float ly = l[y];
    __syncwarp();
    float* out = dlogits + (long)row * V;
    float* pr = probs ? probs + (long)row * V : nullptr;
    for (int j = lane; j < V; j += 32) {
        const float p = __fdiv_rn(expf(l[j] - mx), sf);
        if (pr) pr[j] = p;
        float d = __fdiv_rn(__fsub_rn(p, j == y ? 1.0f : 0.0f), (float)T);
        if (scale != 1.0f) d = __fmul_rn(d, scale);
        out[j] = d;
    }
    if (lane == 0) {
        row_loss[row] = (double)mx + log(s) - (double)ly;
        row_correct[row] = arg == y;
    }
}

// The same for V = 32 NR with the row in registers: lane l holds columns
// l, l + 32, ... (the order in which the kernel above visits them), so the
// row is read from memory once and exp is evaluated once per logit; every
// result is bit-identical to the kernel above.
template <int NR>
__global__ void softmax_ce_vec_kernel(int M, int T, float scale, float* logits, const int* __restrict__ tgt,
                                      float* __restrict__ probs, float* dlogits, double* __restrict__ row_loss,
                                      int* __restrict__ row_correct)
{
    HX_PDL_PROLOGUE();
    constexpr int V = 32 * NR;
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (row >= M) return;
    const float* l = logits + (long)row * V;
    float v[NR];
#pragma unroll
    for (int i = 0; i < NR; ++i) v[i] = l[lane + 32 * i];
    const int y = tgt[row];
    const float ly = l[y];
    float mx = -INFINITY;
    int arg = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < NR; ++i) {
        const int j = lane + 32 * i;
        if (v[i] > mx || (v[i] == mx && j < arg)) { mx = v[i]; arg = j; }
    }
    for (int o = 16; o > 0; o >>= 1) {
        const float om = __shfl_xor_sync(0xffffffffu, mx, o);
        const int oa = __shfl_xor_sync(0xffffffffu, arg, o);
        if (om > mx || (om == mx && oa < arg)) { mx = om; arg = oa; }
    }
    double s = 0.0;
#pragma unroll
    for (int i = 0; i < NR; ++i) {
        v[i] = expf(v[i] - mx);
        s += (double)v[i];
    }
    s = warp_sum(s);
    const float sf = (float)s;
    __syncwarp();  // every lane has read its logits before any overwrites them
    float* out = dlogits + (long)row * V;
    float* pr = probs ? probs + (long)row * V : nullptr;
#pragma unroll
    for (int i = 0; i < NR; ++i) {
        const int j = lane + 32 * i;
        const float p = __fdiv_rn(v[i], sf);
        if (pr) pr[j] = p;
        float d = __fdiv_rn(__fsub_rn(p, j == y ? 1.0f : 0.0f), (float)T);
        if (scale != 1.0f) d = __fmul_rn(d, scale);
        out[j] = d;
    }
    if (lane == 0) {
        row_loss[row] = (double)mx + log(s) - (double)ly;
        row_correct[row] = arg == y;
    }
}

// Per-sequence loss float(sum_t loss/T) (:77): one warp per sequence loads
// 32 positions at a time and every lane adds them in position order (a
// double sum in the same order as a sequential loop over t).
__global__ void loss_seq_kernel(int B, int T, const double* __restrict__ row_loss, const int* __restrict__ row_correct,
                                float* __restrict__ seq_loss, int* __restrict__ seq_correct)
{
    HX_PDL_PROLOGUE();
    const int lane = threadIdx.x & 31;
    const int b = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (b >= B) return;
    double s = 0.0;
    int correct = 0;
    for (int t0 = 0; t0 < T; t0 += 32) {
        const bool ok = t0 + lane < T;
        const double v = ok ? row_loss[(long)b * T + t0 + lane] : 0.0;
        correct += ok ? row_correct[(long)b * T + t0 + lane] : 0;
        const int n = min(32, T - t0);
        for (int i = 0; i < n; ++i) s += __shfl_sync(0xffffffffu, v, i);
    }
    for (int o = 16; o > 0; o >>= 1) correct += __shfl_xor_sync(0xffffffffu, correct, o);
    if (lane == 0) {
        seq_loss[b] = (float)(s / T);
        seq_correct[b] = correct;
    }
}

// Batch mean of the per-sequence losses in double, the accuracy, and the
// scaled loss term for the data-parallel gradient buffer.  One block.
__global__ void loss_reduce_kernel(int B, int T, const float* __restrict__ seq_loss, const int* __restrict__ seq_correct,
                                   float grad_scale, float* __restrict__ loss_out, float* __restrict__ acc_out,
                                   float* __restrict__ scaled_loss_out)
{
    HX_PDL_PROLOGUE();
    __shared__ double red[32];
    __shared__ long cred[32];
    double tot = 0.0;
    long correct = 0;
    for (int b = threadIdx.x; b < B; b += blockDim.x) {
        tot += (double)seq_loss[b];
        correct += seq_correct[b];
    }
    tot = warp_sum(tot);
    for (int o = 16; o > 0; o >>= 1) correct += __shfl_xor_sync(0xffffffffu, correct, o);
    if ((threadIdx.x & 31) == 0) { red[threadIdx.x >> 5] = tot; cred[threadIdx.x >> 5] = correct; }
    __syncthreads();
    if (threadIdx.x == 0) {
        double t = 0.0;
        long c = 0;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) { t += red[w]; c += cred[w]; }
        if (loss_out) *loss_out = (float)(t / B);
        if (acc_out) *acc_out = (float)c / (float)((long)B * T);
        if (scaled_loss_out) *scaled_loss_out = (float)(t * (double)grad_scale);
    }
}

// Token-embedding gradient gE[v,:] = sum over rows r with id[r] == v of
// dX0[r,:] (one-hot^T * dX0, :82), deterministic.  CTA (chunk c of
// `chunk_rows` rows, block of `tb` tokens) keeps the block's rows of the
// gradient in shared memory ([tb][D], tb * D <= 16384 floats).  The CTA
// first loads the chunk's ids into shared memory in one pass; warp 0 then
// lists, in row order, the rows whose token falls in the block; then warp w,
// which owns columns 32w + lane (and every 256th beyond), walks that list
// kEmbBatch rows at a time (independent loads, then the adds in row order).
// Each (token, column) therefore sums its rows of the chunk in row order;
// the table goes to part[c][v][d], and embed_bwd_combine sums the chunks in
// order.  With skewed token frequencies most rows fall in one block, so that
// block's CTAs carry the kernel: short chunks and many loads in flight keep
// them short, and the other CTAs never wait on global memory for their ids.
constexpr int kEmbWarps = 8;
constexpr int kEmbBatch = 16;   // listed rows loaded together per warp
constexpr int kEmbTableFloats = 16384;  // 64 KB of shared memory
// dynamic shared memory of embed_bwd_partial_kernel
inline size_t embed_bwd_smem_bytes(int tb, int D, int chunk_rows) {
    return sizeof(float) * size_t(tb) * D + sizeof(int) * 3 * size_t(chunk_rows) + 16;
}
__global__ void __launch_bounds__(32 * kEmbWarps)
embed_bwd_partial_kernel(int M, int V, int D, int chunk_rows, int tb, const int* __restrict__ ids,
                         const float* __restrict__ dx, float* __restrict__ part)
{
    HX_PDL_PROLOGUE();
    extern __shared__ float tab[];  // [tb][D], then ids[chunk_rows], rows[chunk_rows], toks[chunk_rows], count
    int* sid = reinterpret_cast<int*>(tab + (size_t)tb * D);
    int* srow = sid + chunk_rows;
    int* stok = srow + chunk_rows;
    int* scount = stok + chunk_rows;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int c = blockIdx.x, v0 = blockIdx.y * tb;
    const int ntok = min(tb, V - v0);
    const int r0 = c * chunk_rows, r1 = min(M, r0 + chunk_rows), nr = r1 - r0;
    for (int i = threadIdx.x; i < ntok * D; i += blockDim.x) tab[i] = 0.f;
    for (int i = threadIdx.x; i < nr; i += blockDim.x) sid[i] = ids[r0 + i];
    __syncthreads();
    if (warp == 0) {
        int n = 0;
        for (int rb = 0; rb < nr; rb += 32) {
            const int v = (rb + lane < nr) ? sid[rb + lane] - v0 : -1;
            const bool in = v >= 0 && v < ntok;
            const unsigned mask = __ballot_sync(0xffffffffu, in);
            if (in) {
                const int pos = n + __popc(mask & ((1u << lane) - 1u));
                srow[pos] = r0 + rb + lane;
                stok[pos] = v;
            }
            n += __popc(mask);
        }
        if (lane == 0) *scount = n;
    }
    __syncthreads();
    const int nsel = *scount;
    for (int cb = 32 * warp; cb < D; cb += 32 * kEmbWarps) {
        const int d = cb + lane;
        const bool dok = d < D;
        for (int b = 0; b < nsel; b += kEmbBatch) {
            const int n = min(kEmbBatch, nsel - b);
            float val[kEmbBatch];
#pragma unroll
            for (int q = 0; q < kEmbBatch; ++q) val[q] = (q < n && dok) ? dx[(long)srow[b + q] * D + d] : 0.f;
#pragma unroll
            for (int q = 0; q < kEmbBatch; ++q)
                if (q < n && dok) tab[stok[b + q] * D + d] += val[q];
        }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < ntok * D; i += blockDim.x) part[((long)c * V + v0) * D + i] = tab[i];
}

__global__ void embed_bwd_combine_kernel(int chunks, int V, int D, const float* __restrict__ part,
                                         float* __restrict__ gE)
{
    HX_PDL_PROLOGUE();
    const long total = (long)V * D;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
        float s = 0.f;
        for (int c = 0; c < chunks; ++c) s += part[(long)c * total + i];
        gE[i] = s;
    }
}

// Learned position table gradient: gP[t,:] = sum_b dx0[b*T+t,:].  A CTA takes
// 32 consecutive elements of the [T][D] table (lane = element, 128-byte
// loads); warp w sums sequences w, w + 8, ... and the eight warp sums are
// added in warp order, so the result does not depend on timing.
constexpr int kPosWarps = 8;
__global__ void __launch_bounds__(32 * kPosWarps)
position_bwd_kernel(int B, int T, int D, const float* __restrict__ dx, float* __restrict__ gP)
{
    HX_PDL_PROLOGUE();
    __shared__ float red[kPosWarps][32];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const long total = (long)T * D;
    const long i = (long)blockIdx.x * 32 + lane;
    float s = 0.f;
    if (i < total) {
#pragma unroll 4
        for (int b = w; b < B; b += kPosWarps) s += dx[(long)b * total + i];
    }
    red[w][lane] = s;
    __syncthreads();
    if (w == 0 && i < total) {
        float t = red[0][lane];
#pragma unroll
        for (int k = 1; k < kPosWarps; ++k) t += red[k][lane];
        gP[i] = t;
    }
}

// Packs wq, wk, wv [D,D] (consecutive in the registry) into W_qkv [D,3D].
__global__ void pack_qkv_kernel(int D, const float* __restrict__ wq, float* __restrict__ packed)
{
    HX_PDL_PROLOGUE();
    const long total = 3L * D * D;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
        const int k = (int)(i / (3 * D)), n = (int)(i % (3 * D));
        const int which = n / D, c = n % D;
        packed[i] = wq[(long)which * D * D + (long)k * D + c];
    }
}

// Checks that every row of a [rows, V] matrix is exactly one-hot (one 1.0,
// the rest 0.0) and extracts the index.  Sets *bad otherwise.
__global__ void one_hot_decode_kernel(int rows, int V, const float* __restrict__ oh, uint32_t* __restrict__ ids, int* bad)
{
    HX_PDL_PROLOGUE();
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (row >= rows) return;
    int ones = 0, other = 0, idx = -1;
    for (int j = lane; j < V; j += 32) {
        const float v = oh[(long)row * V + j];
        if (v == 1.0f) { ++ones; idx = j; } else if (v != 0.0f) ++other;
    }
    for (int o = 16; o > 0; o >>= 1) {
        ones += __shfl_xor_sync(0xffffffffu, ones, o);
        other += __shfl_xor_sync(0xffffffffu, other, o);
        idx = max(idx, __shfl_xor_sync(0xffffffffu, idx, o));
    }
    if (lane == 0) {
        if (ones != 1 || other != 0) atomicExch(bad, 1);
        ids[row] = idx < 0 ? 0u : (uint32_t)idx;
    }
}

}  // namespace hx
