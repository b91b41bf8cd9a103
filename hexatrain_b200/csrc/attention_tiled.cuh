// attention_tiled.cuh -- causal multi-head attention, forward and backward,
// as register-tiled block products with K, V (and Q, dO) resident in shared
// memory.  One CTA (256 threads) per (head, sequence); query rows are taken
// in blocks of 64, and key columns above the block's diagonal are skipped.
//
// Forward (tiny_language_model_cpu.cpp:44-45 restated per block):
//   S = Q_blk K^T * scale  (4 rows x 16 strided columns per thread, FMA order
//   d = 0..DH-1), row max and row sum of exp (sum in double) across the 16
//   lanes that share a row, P = exp(S - max) / float(sum), O_blk = P V.
//   Row max and row sum are saved; P is written out only on request.
// Backward (:80-81), with P recomputed bit-identically from the saved
//   statistics and D_r = dO_r . O_r (= sum_j P_rj dP_rj):
//   dV += P^T dO_blk, dP = dO_blk V^T, dS = P * (dP - D), dQ_blk = scale dS K,
//   dK += scale dS^T Q_blk;  dK and dV stay in registers across blocks.
// Limits: T <= 256, DH in {8, 16, 32}.
#pragma once

#include <cuda_runtime.h>
#include <cstdint>

namespace hx {

constexpr int kAttnQB = 64;       // query rows per block
constexpr int kAttnMaxT = 256;
constexpr int kAttnTiledThreads = 256;

template <int DH>
struct AttnTiledLayout {
    static constexpr int LD = DH + 1;          // row stride of Q/K/V/dO tiles (conflict-free column reads)
    static constexpr int LDP = kAttnMaxT + 4;  // row stride of the P / dS block
    static size_t fwd_bytes(int T) { return sizeof(float) * (size_t(2) * T * LD + size_t(kAttnQB) * LD + size_t(kAttnQB) * LDP); }
    static size_t bwd_bytes(int T) {
        return sizeof(float) * (size_t(4) * T * LD + size_t(kAttnQB) * LDP + size_t(3) * T);
    }
};

// S tile for query rows q0 + 4*tr + i (i < 4) and key columns tc + 16*c
// (c < 16, only c < ncg computed): s[i][c] = sum_d Q[row][d] K[col][d].
template <int DH>
__device__ __forceinline__ void attn_scores(const float* Qs, int q_row_base, const float* Ks, int tr, int tc, int ncg,
                                            float (&s)[4][16])
{
    constexpr int LD = AttnTiledLayout<DH>::LD;
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int c = 0; c < 16; ++c) s[i][c] = 0.f;
#pragma unroll 4
    for (int d = 0; d < DH; ++d) {
        float a[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) a[i] = Qs[(q_row_base + 4 * tr + i) * LD + d];
#pragma unroll
        for (int c = 0; c < 16; ++c) {
            if (c < ncg) {
                const float b = Ks[(tc + 16 * c) * LD + d];
#pragma unroll
                for (int i = 0; i < 4; ++i) s[i][c] = fmaf(a[i], b, s[i][c]);
            }
        }
    }
}

template <int DH>
__global__ void __launch_bounds__(kAttnTiledThreads, 1)
attention_fwd_tiled_kernel(int T, int D, int H, float scale, const float* __restrict__ qkv, float* __restrict__ ctx,
                           float* __restrict__ row_max, float* __restrict__ row_sum, float* __restrict__ probs)
{
    using Lay = AttnTiledLayout<DH>;
    constexpr int LD = Lay::LD, LDP = Lay::LDP;
    extern __shared__ float sm[];
    float* Ks = sm;                       // [T][LD]
    float* Vs = Ks + T * LD;              // [T][LD]
    float* Qb = Vs + T * LD;              // [64][LD]
    float* Pb = Qb + kAttnQB * LD;        // [64][LDP]
    const int h = blockIdx.x, b = blockIdx.y;
    const int t = threadIdx.x;
    const long rowbase = (long)b * T;
    const int ld = 3 * D;
    for (int i = t; i < T * DH; i += kAttnTiledThreads) {
        const int j = i / DH, d = i % DH;
        const float* src = qkv + (rowbase + j) * ld + h * DH + d;
        Ks[j * LD + d] = src[D];
        Vs[j * LD + d] = src[2 * D];
    }
    const int tr = t >> 4, tc = t & 15;
    const int nblk = (T + kAttnQB - 1) / kAttnQB;
    for (int qb = 0; qb < nblk; ++qb) {
        const int q0 = qb * kAttnQB;
        const int tlim = min(T, q0 + kAttnQB);            // keys 0..tlim-1 can be visible
        const int ncg = (tlim + 15) >> 4;
        __syncthreads();                                  // previous block done with Qb / Pb
        for (int i = t; i < kAttnQB * DH; i += kAttnTiledThreads) {
            const int r = i / DH, d = i % DH;
            Qb[r * LD + d] = (q0 + r < T) ? qkv[(rowbase + q0 + r) * ld + h * DH + d] : 0.f;
        }
        __syncthreads();
        float s[4][16];
        attn_scores<DH>(Qb, 0, Ks, tr, tc, ncg, s);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int r = q0 + 4 * tr + i;               // query row (may be >= T in the last block)
            float mx = -INFINITY;
#pragma unroll
            for (int c = 0; c < 16; ++c) {
                const int j = tc + 16 * c;
                if (c < ncg && j <= r && j < T) {
                    s[i][c] = __fmul_rn(s[i][c], scale);
                    mx = fmaxf(mx, s[i][c]);
                }
            }
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            double sum = 0.0;
#pragma unroll
            for (int c = 0; c < 16; ++c) {
                const int j = tc + 16 * c;
                if (c < ncg && j <= r && j < T) {
                    s[i][c] = expf(__fsub_rn(s[i][c], mx));
                    sum += s[i][c];
                }
            }
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
            const float sumf = (float)sum;
            float* prow = Pb + (4 * tr + i) * LDP;
#pragma unroll
            for (int c = 0; c < 16; ++c) {
                const int j = tc + 16 * c;
                if (c < ncg) prow[j] = (j <= r && j < T) ? __fdiv_rn(s[i][c], sumf) : 0.f;
            }
            if (tc == 0 && r < T) {
                row_max[((long)b * H + h) * T + r] = mx;
                row_sum[((long)b * H + h) * T + r] = sumf;
            }
        }
        __syncthreads();
        if (probs) {
            for (int i = t; i < kAttnQB * T; i += kAttnTiledThreads) {
                const int r = i / T, j = i % T;
                if (q0 + r < T) probs[(((long)b * H + h) * T + q0 + r) * T + j] = (j < tlim) ? Pb[r * LDP + j] : 0.f;
            }
        }
        // O_blk = P V : thread -> rows (2*orow, 2*orow+1), columns [opc*ow, opc*ow + ow)
        constexpr int OW = DH / 8;                        // columns per thread (DH = 8..32 -> 1..4)
        const int orow = t >> 3, ocol = (t & 7) * OW;
        float o0[OW], o1[OW];
#pragma unroll
        for (int x = 0; x < OW; ++x) { o0[x] = 0.f; o1[x] = 0.f; }
        const float* p0 = Pb + (2 * orow) * LDP;
        const float* p1 = p0 + LDP;
        for (int j = 0; j < tlim; ++j) {
            const float a0 = p0[j], a1 = p1[j];
#pragma unroll
            for (int x = 0; x < OW; ++x) {
                const float v = Vs[j * LD + ocol + x];
                o0[x] = fmaf(a0, v, o0[x]);
                o1[x] = fmaf(a1, v, o1[x]);
            }
        }
        const int r0 = q0 + 2 * orow;
#pragma unroll
        for (int x = 0; x < OW; ++x) {
            if (r0 < T) ctx[(rowbase + r0) * D + h * DH + ocol + x] = o0[x];
            if (r0 + 1 < T) ctx[(rowbase + r0 + 1) * D + h * DH + ocol + x] = o1[x];
        }
    }
}

template <int DH>
__global__ void __launch_bounds__(kAttnTiledThreads, 1)
attention_bwd_tiled_kernel(int T, int D, int H, float scale, const float* __restrict__ qkv,
                           const float* __restrict__ ctx, const float* __restrict__ dctx,
                           const float* __restrict__ row_max, const float* __restrict__ row_sum,
                           float* __restrict__ dqkv)
{
    using Lay = AttnTiledLayout<DH>;
    constexpr int LD = Lay::LD, LDP = Lay::LDP;
    extern __shared__ float sm[];
    float* Qs = sm;                  // [T][LD]
    float* Ks = Qs + T * LD;
    float* Vs = Ks + T * LD;
    float* Os = Vs + T * LD;         // dO (the incoming gradient of the context)
    float* Pb = Os + T * LD;         // [64][LDP]  P, then dS
    float* Dr = Pb + kAttnQB * LDP;  // [T] D_r = dO_r . O_r
    float* Mx = Dr + T;              // [T]
    float* Sm = Mx + T;              // [T]
    const int h = blockIdx.x, b = blockIdx.y;
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const long rowbase = (long)b * T;
    const int ld = 3 * D;
    for (int i = t; i < T * DH; i += kAttnTiledThreads) {
        const int j = i / DH, d = i % DH;
        const float* src = qkv + (rowbase + j) * ld + h * DH + d;
        Qs[j * LD + d] = src[0];
        Ks[j * LD + d] = src[D];
        Vs[j * LD + d] = src[2 * D];
        Os[j * LD + d] = dctx[(rowbase + j) * D + h * DH + d];
    }
    for (int i = t; i < T; i += kAttnTiledThreads) {
        Mx[i] = row_max[((long)b * H + h) * T + i];
        Sm[i] = row_sum[((long)b * H + h) * T + i];
    }
    // D_r = dO_r . O_r, one warp per row
    for (int r = warp; r < T; r += kAttnTiledThreads / 32) {
        float acc = 0.f;
        for (int d = lane; d < DH; d += 32) acc = fmaf(dctx[(rowbase + r) * D + h * DH + d], ctx[(rowbase + r) * D + h * DH + d], acc);
        for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (lane == 0) Dr[r] = acc;
    }
    __syncthreads();
    // dK / dV accumulators: thread -> key rows 4*kr .. 4*kr+3, columns [kc*CW, kc*CW+CW)
    constexpr int CW = DH / 4;
    const int kr = t >> 2, kc = (t & 3) * CW;
    float dk[4][CW], dv[4][CW];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int x = 0; x < CW; ++x) { dk[i][x] = 0.f; dv[i][x] = 0.f; }
    const int tr = t >> 4, tc = t & 15;
    const int nblk = (T + kAttnQB - 1) / kAttnQB;
    for (int qb = 0; qb < nblk; ++qb) {
        const int q0 = qb * kAttnQB;
        const int tlim = min(T, q0 + kAttnQB);
        const int ncg = (tlim + 15) >> 4;
        const int rows = min(kAttnQB, T - q0);
        // 1. P (recomputed exactly as the forward) into Pb
        float s[4][16];
        attn_scores<DH>(Qs, q0, Ks, tr, tc, ncg, s);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int r = q0 + 4 * tr + i;
            const bool rv = r < T;
            const float mx = rv ? Mx[r] : 0.f, sumf = rv ? Sm[r] : 1.f;
            float* prow = Pb + (4 * tr + i) * LDP;
#pragma unroll
            for (int c = 0; c < 16; ++c) {
                const int j = tc + 16 * c;
                if (c < ncg)
                    prow[j] = (rv && j <= r && j < T) ? __fdiv_rn(expf(__fsub_rn(__fmul_rn(s[i][c], scale), mx)), sumf) : 0.f;
            }
        }
        __syncthreads();
        // 2. dV[j] += sum_r P[r][j] dO[r]   (keys j = 4*kr + i)
        if (4 * kr < tlim) {
            for (int r = 0; r < rows; ++r) {
                const float* prow = Pb + r * LDP + 4 * kr;
                float pv[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) pv[i] = prow[i];
                const float* orow = Os + (q0 + r) * LD + kc;
#pragma unroll
                for (int x = 0; x < CW; ++x) {
                    const float g = orow[x];
#pragma unroll
                    for (int i = 0; i < 4; ++i) dv[i][x] = fmaf(pv[i], g, dv[i][x]);
                }
            }
        }
        // 3. dP = dO_blk V^T (same tiling as S), dS = P * (dP - D)
        float dp[4][16];
        attn_scores<DH>(Os, q0, Vs, tr, tc, ncg, dp);
        __syncthreads();  // everyone finished reading P for dV
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int r = q0 + 4 * tr + i;
            const float dr = r < T ? Dr[r] : 0.f;
            float* prow = Pb + (4 * tr + i) * LDP;
#pragma unroll
            for (int c = 0; c < 16; ++c) {
                const int j = tc + 16 * c;
                if (c < ncg) prow[j] = __fmul_rn(prow[j], __fsub_rn(dp[i][c], dr));
            }
        }
        __syncthreads();
        // 4. dQ_blk = scale * dS K : thread -> rows (2*orow, +1), columns ocol..
        {
            constexpr int OW = DH / 8;
            const int orow = t >> 3, ocol = (t & 7) * OW;
            float q0a[OW], q1a[OW];
#pragma unroll
            for (int x = 0; x < OW; ++x) { q0a[x] = 0.f; q1a[x] = 0.f; }
            const float* d0 = Pb + (2 * orow) * LDP;
            const float* d1 = d0 + LDP;
            for (int j = 0; j < tlim; ++j) {
                const float a0 = d0[j], a1 = d1[j];
#pragma unroll
                for (int x = 0; x < OW; ++x) {
                    const float k = Ks[j * LD + ocol + x];
                    q0a[x] = fmaf(a0, k, q0a[x]);
                    q1a[x] = fmaf(a1, k, q1a[x]);
                }
            }
            const int r0 = q0 + 2 * orow;
#pragma unroll
            for (int x = 0; x < OW; ++x) {
                if (r0 < T) dqkv[(rowbase + r0) * ld + h * DH + ocol + x] = q0a[x] * scale;
                if (r0 + 1 < T) dqkv[(rowbase + r0 + 1) * ld + h * DH + ocol + x] = q1a[x] * scale;
            }
        }
        // 5. dK[j] += sum_r dS[r][j] Q[r]
        if (4 * kr < tlim) {
            for (int r = 0; r < rows; ++r) {
                const float* srow = Pb + r * LDP + 4 * kr;
                float sv[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) sv[i] = srow[i];
                const float* qrow = Qs + (q0 + r) * LD + kc;
#pragma unroll
                for (int x = 0; x < CW; ++x) {
                    const float g = qrow[x];
#pragma unroll
                    for (int i = 0; i < 4; ++i) dk[i][x] = fmaf(sv[i], g, dk[i][x]);
                }
            }
        }
        __syncthreads();  // before the next block overwrites Pb
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
