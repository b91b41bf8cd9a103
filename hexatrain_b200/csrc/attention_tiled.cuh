// attention_tiled.cuh -- causal multi-head attention, forward and backward,
// on the CUDA cores in FP32, with everything a (head, sequence) needs held in
// shared memory.  One CTA (256 threads, 8 warps) per (head, sequence);
// query rows are taken in blocks of 64 and key columns beyond the block's
// last row are skipped.
//
// Three register-tiled block products, each fed by float4 shared-memory
// loads so that the FMA pipe, not the load pipe, bounds them:
//   scores  S[r][j] = sum_d A[r][d] B[j][d]: warp w owns the 8 rows
//           8w..8w+7 of the block (A rows are broadcast loads), lane l owns
//           keys l, l+32, ... (B rows are lane-distinct loads); 8x8
//           accumulators per thread, FMA order d = 0..DH-1.
//   P V     (and dS K) split over keys across the warps: warp w takes a
//           contiguous key range (multiple of 4), lane (g, c) = (l/4, l%4)
//           accumulates rows g, g+8, ..., g+56 x DH/4 columns; the eight
//           warp partials are summed in warp order through shared memory.
//   P^T dO  (and dS^T Q) per key: thread t owns keys 4(t/4)..+3 and DH/4
//           columns, accumulating over every query row of every block.
//
// Forward (tiny_language_model_cpu.cpp:44-45 restated per block):
//   S = Q_blk K^T * scale, row max, row sum of exp in double (lane partials
//   then a butterfly over the warp), P = exp(S - max) / float(sum),
//   O_blk = P V.  Row max and row sum are saved; P is written out only on
//   request.
// Backward (:79-81), with P recomputed from the saved row max by the same
//   score routine and FMA order, its row sum recomputed from these same
//   exponentials in the forward's summation order (bit-identical to the
//   forward's after this forward; after the tensor-core forward it keeps
//   sum_j P[r][j] = 1 to FP32 rounding, which the wq/wk gradients of
//   near-uniform attention are sensitive to), and, as the reference,
//   D_r = sum_j P[r][j] dP[r][j] (float products summed in double):
//   dV += P^T dO_blk, dP = dO_blk V^T, dS = P * (dP - D), dQ_blk = scale dS K,
//   dK += scale dS^T Q_blk.  Taking D from P and dP (rather than dO . O)
//   keeps sum_j dS[r][j] = 0 whatever engine produced the forward output.
// Limits: T <= 256, DH in {8, 16, 32}.
#pragma once

#include "pdl.cuh"

#include <cuda_runtime.h>
#include <cstdint>

namespace hx {

constexpr int kAttnQB = 64;       // query rows per block
constexpr int kAttnMaxT = 256;
constexpr int kAttnTiledThreads = 256;

template <int DH>
struct AttnTiledLayout {
    // Row stride of the Q/K/V/dO tiles and of the warp partials: DH + 4
    // keeps rows 16-byte aligned and puts 8 consecutive rows on distinct
    // 4-bank groups, so float4 accesses of lane-distinct rows are
    // conflict-free.
    static constexpr int LD = DH + 4;
    // Tile rows: T rounded up to a whole query block, zero beyond T, so that
    // every block product reads initialised rows.
    __host__ __device__ static int tpad(int T) { return ((T + kAttnQB - 1) / kAttnQB) * kAttnQB; }
    // Row stride of the P / dS block: keys rounded up to 32, plus 4 (same
    // reason, for rows g, g+8, ... read with float4 by 8 lane groups).
    __host__ __device__ static int ldp(int T) { return ((T + 31) / 32) * 32 + 4; }
    __host__ __device__ static size_t blk_floats(int T) {
        const size_t a = size_t(kAttnQB) * ldp(T), b = size_t(8) * kAttnQB * LD;
        return a > b ? a : b;
    }
    static size_t fwd_bytes(int T) { return sizeof(float) * (size_t(3) * tpad(T) * LD + blk_floats(T)); }
    static size_t bwd_bytes(int T) {
        return sizeof(float) * (size_t(4) * tpad(T) * LD + blk_floats(T) + size_t(T));
    }
};

template <int N>
__device__ __forceinline__ void attn_ld(const float* p, float (&v)[N]) {
    static_assert(N == 2 || N % 4 == 0, "vector width");
    if constexpr (N == 2) {
        const float2 a = *reinterpret_cast<const float2*>(p);
        v[0] = a.x; v[1] = a.y;
    } else {
#pragma unroll
        for (int i = 0; i < N; i += 4) {
            const float4 a = *reinterpret_cast<const float4*>(p + i);
            v[i] = a.x; v[i + 1] = a.y; v[i + 2] = a.z; v[i + 3] = a.w;
        }
    }
}

template <int N>
__device__ __forceinline__ void attn_st(float* p, const float (&v)[N]) {
    static_assert(N == 2 || N % 4 == 0, "vector width");
    if constexpr (N == 2) {
        *reinterpret_cast<float2*>(p) = make_float2(v[0], v[1]);
    } else {
#pragma unroll
        for (int i = 0; i < N; i += 4) *reinterpret_cast<float4*>(p + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
    }
}

// s[i][c] = sum_d A[(8w + i) * LD + d] * B[(lane + 32c) * LD + d] for c < nc,
// FMA order d = 0..DH-1.  A points at the block's first row.
template <int DH>
__device__ __forceinline__ void attn_score_tile(const float* __restrict__ A, const float* __restrict__ B, int warp,
                                                int lane, int nc, float (&s)[8][8])
{
    constexpr int LD = AttnTiledLayout<DH>::LD;
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int c = 0; c < 8; ++c) s[i][c] = 0.f;
    const float* arow = A + 8 * warp * LD;
#pragma unroll 1
    for (int d = 0; d < DH; d += 4) {
        float4 b[8];
#pragma unroll
        for (int c = 0; c < 8; ++c)
            b[c] = c < nc ? *reinterpret_cast<const float4*>(B + (lane + 32 * c) * LD + d) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float4 a = *reinterpret_cast<const float4*>(arow + i * LD + d);
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                if (c < nc) {
                    s[i][c] = fmaf(a.x, b[c].x, s[i][c]);
                    s[i][c] = fmaf(a.y, b[c].y, s[i][c]);
                    s[i][c] = fmaf(a.z, b[c].z, s[i][c]);
                    s[i][c] = fmaf(a.w, b[c].w, s[i][c]);
                }
            }
        }
    }
}

// Partial of O_blk = Pblk V over this warp's key range [j0, j1) (multiples of
// 4): acc[i][x] for block row g + 8i, column cg*CW + x.
template <int DH>
__device__ __forceinline__ void attn_pv_partial(const float* __restrict__ Pb, int ldp, const float* __restrict__ V,
                                                int j0, int j1, int g, int cg, float (&acc)[8][DH / 4])
{
    constexpr int LD = AttnTiledLayout<DH>::LD, CW = DH / 4;
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int x = 0; x < CW; ++x) acc[i][x] = 0.f;
#pragma unroll 1
    for (int j = j0; j < j1; j += 4) {
        float4 p[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) p[i] = *reinterpret_cast<const float4*>(Pb + (g + 8 * i) * ldp + j);
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
            float v[CW];
            attn_ld<CW>(V + (j + jj) * LD + cg * CW, v);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const float pj = jj == 0 ? p[i].x : jj == 1 ? p[i].y : jj == 2 ? p[i].z : p[i].w;
#pragma unroll
                for (int x = 0; x < CW; ++x) acc[i][x] = fmaf(pj, v[x], acc[i][x]);
            }
        }
    }
}

// Stores this warp's partial into the block buffer laid out [warp][64][LD]
// and, after a barrier, reduces the eight partials of output (r, d) in warp
// order.
template <int DH>
__device__ __forceinline__ void attn_store_partial(float* __restrict__ part, int warp, int g, int cg,
                                                   const float (&acc)[8][DH / 4])
{
    constexpr int LD = AttnTiledLayout<DH>::LD, CW = DH / 4;
#pragma unroll
    for (int i = 0; i < 8; ++i) attn_st<CW>(part + (warp * kAttnQB + g + 8 * i) * LD + cg * CW, acc[i]);
}
template <int DH>
__device__ __forceinline__ float attn_reduce_partial(const float* __restrict__ part, int r, int d) {
    constexpr int LD = AttnTiledLayout<DH>::LD;
    float v = part[r * LD + d];
#pragma unroll
    for (int w = 1; w < 8; ++w) v = __fadd_rn(v, part[(w * kAttnQB + r) * LD + d]);
    return v;
}

// Key range of warp w for a block whose visible keys are [0, tlim): equal
// shares rounded up to a multiple of 4, clipped to tlim rounded up to 4.
__device__ __forceinline__ void attn_key_range(int tlim, int warp, int& j0, int& j1) {
    const int t4 = (tlim + 3) & ~3;
    const int per = (((tlim + 7) / 8) + 3) & ~3;
    j0 = min(t4, warp * per);
    j1 = min(t4, j0 + per);
}

__device__ __forceinline__ void attn_cp_async16(float* dst, const float* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src)
                 : "memory");
}
__device__ __forceinline__ void attn_cp_async_wait_all() {
    asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

// Starts the copy of rows [0, T) of one head's DH columns into a [rows][LD]
// tile as 16-byte cp.async transfers (all in flight at once); rows T..rows-1
// are zeroed.  src_ld is the source row stride in floats; src and src_ld
// keep every row 16-byte aligned (DH and the model width are multiples of 8).
// Complete with attn_cp_async_wait_all() and a barrier.
template <int DH>
__device__ __forceinline__ void attn_load_tile(float* __restrict__ dst, const float* __restrict__ src, long src_ld,
                                               int T, int rows)
{
    constexpr int LD = AttnTiledLayout<DH>::LD, V4 = DH / 4;
    for (int i = threadIdx.x; i < rows * V4; i += kAttnTiledThreads) {
        const int j = i / V4, c = (i % V4) * 4;
        float* d = dst + j * LD + c;
        if (j < T)
            attn_cp_async16(d, src + j * src_ld + c);
        else
            *reinterpret_cast<float4*>(d) = make_float4(0.f, 0.f, 0.f, 0.f);
    }
}

template <int DH>
__global__ void __launch_bounds__(kAttnTiledThreads, 1)
attention_fwd_tiled_kernel(int T, int D, int H, float scale, const float* __restrict__ qkv, float* __restrict__ ctx,
                           float* __restrict__ row_max, float* __restrict__ row_sum, float* __restrict__ probs)
{
    HX_PDL_PROLOGUE();
    using Lay = AttnTiledLayout<DH>;
    constexpr int LD = Lay::LD, CW = DH / 4;
    extern __shared__ float4 sm4[];
    float* sm = reinterpret_cast<float*>(sm4);
    const int tpad = Lay::tpad(T), ldp = Lay::ldp(T);
    float* Qs = sm;                    // [tpad][LD]
    float* Ks = Qs + tpad * LD;        // [tpad][LD]
    float* Vs = Ks + tpad * LD;        // [tpad][LD]
    float* Pb = Vs + tpad * LD;        // [64][ldp] P, then [8][64][LD] partials
    const int h = blockIdx.x, b = blockIdx.y;
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const long rowbase = (long)b * T;
    const int ld = 3 * D;
    attn_load_tile<DH>(Qs, qkv + rowbase * ld + h * DH, ld, T, tpad);
    attn_load_tile<DH>(Ks, qkv + rowbase * ld + D + h * DH, ld, T, tpad);
    attn_load_tile<DH>(Vs, qkv + rowbase * ld + 2 * D + h * DH, ld, T, tpad);
    attn_cp_async_wait_all();
    const int g = lane >> 2, cg = lane & 3;
    const int nblk = (T + kAttnQB - 1) / kAttnQB;
    for (int qb = 0; qb < nblk; ++qb) {
        const int q0 = qb * kAttnQB;
        const int tlim = min(T, q0 + kAttnQB);            // keys 0..tlim-1 can be visible
        const int nc = (tlim + 31) >> 5;
        __syncthreads();                                  // tiles landed / previous block done with Pb
        float s[8][8];
        attn_score_tile<DH>(Qs + q0 * LD, Ks, warp, lane, nc, s);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int r = q0 + 8 * warp + i;             // query row (may be >= T in the last block)
            float* prow = Pb + (8 * warp + i) * ldp;
            if (r >= T) {
#pragma unroll
                for (int c = 0; c < 8; ++c)
                    if (c < nc) prow[lane + 32 * c] = 0.f;
                continue;
            }
            float mx = -INFINITY;
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                const int j = lane + 32 * c;
                if (c < nc && j <= r) {
                    s[i][c] = __fmul_rn(s[i][c], scale);
                    mx = fmaxf(mx, s[i][c]);
                }
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            double sum = 0.0;
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                const int j = lane + 32 * c;
                if (c < nc && j <= r) {
                    s[i][c] = expf(__fsub_rn(s[i][c], mx));
                    sum += s[i][c];
                }
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
            const float sumf = (float)sum;
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                const int j = lane + 32 * c;
                if (c < nc) prow[j] = (j <= r) ? __fdiv_rn(s[i][c], sumf) : 0.f;
            }
            if (lane == 0) {
                row_max[((long)b * H + h) * T + r] = mx;
                row_sum[((long)b * H + h) * T + r] = sumf;
            }
        }
        __syncthreads();
        if (probs) {
            for (int i = t; i < kAttnQB * T; i += kAttnTiledThreads) {
                const int r = i / T, j = i % T;
                if (q0 + r < T) probs[(((long)b * H + h) * T + q0 + r) * T + j] = (j < tlim) ? Pb[r * ldp + j] : 0.f;
            }
        }
        int j0, j1;
        attn_key_range(tlim, warp, j0, j1);
        float acc[8][CW];
        attn_pv_partial<DH>(Pb, ldp, Vs, j0, j1, g, cg, acc);
        __syncthreads();                                  // P no longer read: the block becomes the partials
        attn_store_partial<DH>(Pb, warp, g, cg, acc);
        __syncthreads();
        for (int o = t; o < kAttnQB * DH; o += kAttnTiledThreads) {
            const int r = o / DH, d = o % DH;
            const float v = attn_reduce_partial<DH>(Pb, r, d);
            if (q0 + r < T) ctx[(rowbase + q0 + r) * D + h * DH + d] = v;
        }
    }
}

template <int DH>
__global__ void __launch_bounds__(kAttnTiledThreads, 1)
attention_bwd_tiled_kernel(int T, int D, int H, float scale, const float* __restrict__ qkv,
                           const float* __restrict__ dctx,
                           const float* __restrict__ row_max, float* __restrict__ dqkv)
{
    HX_PDL_PROLOGUE();
    using Lay = AttnTiledLayout<DH>;
    constexpr int LD = Lay::LD, CW = DH / 4;
    extern __shared__ float4 sm4[];
    float* sm = reinterpret_cast<float*>(sm4);
    const int tpad = Lay::tpad(T), ldp = Lay::ldp(T);
    float* Qs = sm;                      // [tpad][LD]
    float* Ks = Qs + tpad * LD;
    float* Vs = Ks + tpad * LD;
    float* Os = Vs + tpad * LD;          // dO (the incoming gradient of the context)
    float* Blk = Os + tpad * LD;         // [64][ldp] P, then dS, then [8][64][LD] dQ partials
    float* Mx = Blk + Lay::blk_floats(T);  // [T]
    const int h = blockIdx.x, b = blockIdx.y;
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const long rowbase = (long)b * T;
    const int ld = 3 * D;
    attn_load_tile<DH>(Qs, qkv + rowbase * ld + h * DH, ld, T, tpad);
    attn_load_tile<DH>(Ks, qkv + rowbase * ld + D + h * DH, ld, T, tpad);
    attn_load_tile<DH>(Vs, qkv + rowbase * ld + 2 * D + h * DH, ld, T, tpad);
    attn_load_tile<DH>(Os, dctx + rowbase * D + h * DH, D, T, tpad);
    for (int i = t; i < T; i += kAttnTiledThreads) Mx[i] = row_max[((long)b * H + h) * T + i];
    attn_cp_async_wait_all();
    __syncthreads();
    // dK / dV accumulators: thread -> keys 4*kr .. 4*kr+3, columns [kc, kc+CW)
    const int kr = t >> 2, kc = (t & 3) * CW;
    float dk[4][CW], dv[4][CW];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int x = 0; x < CW; ++x) { dk[i][x] = 0.f; dv[i][x] = 0.f; }
    const int g = lane >> 2, cg = lane & 3;
    const int nblk = (T + kAttnQB - 1) / kAttnQB;
    for (int qb = 0; qb < nblk; ++qb) {
        const int q0 = qb * kAttnQB;
        const int tlim = min(T, q0 + kAttnQB);
        const int nc = (tlim + 31) >> 5;
        const int rows = min(kAttnQB, T - q0);
        // 1. P (recomputed exactly as the forward) into the block
        {
            float s[8][8];
            attn_score_tile<DH>(Qs + q0 * LD, Ks, warp, lane, nc, s);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int r = q0 + 8 * warp + i;
                const bool rv = r < T;
                const float mx = rv ? Mx[r] : 0.f;
                double sum = 0.0;
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    const int j = lane + 32 * c;
                    if (c < nc && rv && j <= r) {
                        s[i][c] = expf(__fsub_rn(__fmul_rn(s[i][c], scale), mx));
                        sum += s[i][c];
                    }
                }
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
                const float sumf = rv ? (float)sum : 1.f;
                float* prow = Blk + (8 * warp + i) * ldp;
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    const int j = lane + 32 * c;
                    if (c < nc) prow[j] = (rv && j <= r) ? __fdiv_rn(s[i][c], sumf) : 0.f;
                }
            }
        }
        // 2. dP = dO_blk V^T (same tiling as S)
        float dp[8][8];
        attn_score_tile<DH>(Os + q0 * LD, Vs, warp, lane, nc, dp);
        __syncthreads();  // P complete
        // 3. dV[j] += sum_r P[r][j] dO[r]
        if (4 * kr < tlim) {
#pragma unroll 2
            for (int r = 0; r < rows; ++r) {
                const float4 p = *reinterpret_cast<const float4*>(Blk + r * ldp + 4 * kr);
                float o[CW];
                attn_ld<CW>(Os + (q0 + r) * LD + kc, o);
#pragma unroll
                for (int x = 0; x < CW; ++x) {
                    dv[0][x] = fmaf(p.x, o[x], dv[0][x]);
                    dv[1][x] = fmaf(p.y, o[x], dv[1][x]);
                    dv[2][x] = fmaf(p.z, o[x], dv[2][x]);
                    dv[3][x] = fmaf(p.w, o[x], dv[3][x]);
                }
            }
        }
        // 4. D_r = sum_j P dP (lane partials, then a butterfly over the
        //    warp, in double), dS = P * (dP - D), from this thread's own P
        //    entries (written by this thread in step 1)
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int r = q0 + 8 * warp + i;
            const float* prow = Blk + (8 * warp + i) * ldp;
            double dot = 0.0;
#pragma unroll
            for (int c = 0; c < 8; ++c)
                if (c < nc) dot += double(__fmul_rn(prow[lane + 32 * c], dp[i][c]));
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
            const float dr = float(dot);
#pragma unroll
            for (int c = 0; c < 8; ++c)
                if (c < nc) dp[i][c] = r < T ? __fmul_rn(prow[lane + 32 * c], __fsub_rn(dp[i][c], dr)) : 0.f;
        }
        __syncthreads();  // every read of P done
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            float* prow = Blk + (8 * warp + i) * ldp;
#pragma unroll
            for (int c = 0; c < 8; ++c)
                if (c < nc) prow[lane + 32 * c] = dp[i][c];
        }
        __syncthreads();  // dS complete
        // 5. dK[j] += sum_r dS[r][j] Q[r]
        if (4 * kr < tlim) {
#pragma unroll 2
            for (int r = 0; r < rows; ++r) {
                const float4 p = *reinterpret_cast<const float4*>(Blk + r * ldp + 4 * kr);
                float q[CW];
                attn_ld<CW>(Qs + (q0 + r) * LD + kc, q);
#pragma unroll
                for (int x = 0; x < CW; ++x) {
                    dk[0][x] = fmaf(p.x, q[x], dk[0][x]);
                    dk[1][x] = fmaf(p.y, q[x], dk[1][x]);
                    dk[2][x] = fmaf(p.z, q[x], dk[2][x]);
                    dk[3][x] = fmaf(p.w, q[x], dk[3][x]);
                }
            }
        }
        // 6. dQ_blk = scale * dS K, split over keys across warps
        int j0, j1;
        attn_key_range(tlim, warp, j0, j1);
        float acc[8][CW];
        attn_pv_partial<DH>(Blk, ldp, Ks, j0, j1, g, cg, acc);
        __syncthreads();  // dS no longer read: the block becomes the partials
        attn_store_partial<DH>(Blk, warp, g, cg, acc);
        __syncthreads();
        for (int o = t; o < kAttnQB * DH; o += kAttnTiledThreads) {
            const int r = o / DH, d = o % DH;
            const float v = attn_reduce_partial<DH>(Blk, r, d);
            if (q0 + r < T) dqkv[(rowbase + q0 + r) * ld + h * DH + d] = v * scale;
        }
        __syncthreads();  // before the next block overwrites the buffer
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int j = 4 * kr + i;
        if (j >= T) continue;
#pragma unroll
        for (int x = 0; x < CW; ++x) {
            dqkv[(rowbase + j) * ld + D + h * DH + kc + x] = dk[i][x] * scale;
            dqkv[(rowbase + j) * ld + 2 * D + h * DH + kc + x] = dv[i][x];
        }
    }
}

}  // namespace hx
