// muon_tc.cuh -- Muon's Newton-Schulz iterations on the tcgen05 tensor cores.
//
// Muon (no counterpart in the reference; Jordan et al. 2024): per 2-D weight
// W [rows x cols] with gradient G and momentum buffer M,
//   M' = mu M + G;  U = Nesterov ? G + mu M' : M';  X = U / (||U||_F + 1e-7)
// transposed so that X is [R x C] with R <= C, then ns_steps times
//   A = X X^T;  Bm = b A + c A A;  X = a X + Bm X
// and W' = W - lr * sqrt(max(1, rows/cols)) * X (transposed back).
//
// Every product reads bf16 operands (the FP32 values rounded to nearest) and
// accumulates in FP32: tcgen05.mma kind::f16 with BF16 A and B, M = 128 (rows
// of X on TMEM lanes), K-major operands in shared memory with the 128-byte
// swizzle.  One CTA of 128 threads per matrix, thread t owning row t:
//   D0 = X X^T           (A and B: the bf16 rows of X)
//   D1 = A A             (A and B: the bf16 rows of A; A is symmetric)
//   Bm = b D0 + c D1     (FP32, then bf16 into A's tile)
//   D0 = Bm X            (B: the bf16 rows of X^T)
//   X  = a X + D0        (FP32 master copy of X in shared memory)
// Limits: R <= 128 and C <= 128 (two 64-element K chunks per tile row).
// The wait on each product's commit is bounded; on timeout the CTA records
// kMuonTcErr in the runtime's error word, frees its TMEM and returns.
#pragma once

#include "pdl.cuh"

#include <cuda_bf16.h>

#include <cstddef>

#include "optim.cuh"
#include "tc_ptx.cuh"

namespace hx {

constexpr int kMuonTcThreads = 128;
constexpr int kMuonTcMaxDim = 128;
constexpr int kMuonTcErr = 16;
constexpr uint32_t kMuonTcChunkBytes = 128 * 128;  // one 64-element K chunk of a 128-row tile
constexpr int kMuonXfStride = kMuonTcMaxDim + 1;   // FP32 rows of X, padded against bank conflicts

struct MuonTcSmem {
    alignas(1024) uint8_t xs[2 * kMuonTcChunkBytes];  // X, rows r, K = C
    alignas(1024) uint8_t xt[2 * kMuonTcChunkBytes];  // X^T, rows c, K = R
    alignas(1024) uint8_t as[2 * kMuonTcChunkBytes];  // A, then Bm: rows r, K = R
    float xf[kMuonTcMaxDim * kMuonXfStride];         // X in FP32, [R][C]
    double red[kMuonTcThreads / 32];
    uint64_t bar;
    uint32_t tmem;
    int abort;
};
constexpr size_t kMuonTcSmemBytes = sizeof(MuonTcSmem) + 1024;
static_assert(kMuonTcSmemBytes <= 232448, "Muon tensor-core kernel shared memory exceeds 227 KB");

// Byte offset of bf16 element (row, k) in a K-major tile set with the
// 128-byte swizzle: 64-element K chunks of 128 rows, 8-row 1024-byte atoms,
// 16-byte chunk j of row r stored at chunk j ^ (r % 8).
__device__ __forceinline__ uint32_t muon_sw_off(int row, int k) {
    const int chunk = k >> 6, kb = (k & 63) * 2;
    return uint32_t(chunk) * kMuonTcChunkBytes + uint32_t(row >> 3) * 1024 + uint32_t(row & 7) * 128 +
           uint32_t(((kb >> 4) ^ (row & 7)) << 4) + uint32_t(kb & 15);
}
__device__ __forceinline__ void muon_st_bf16(uint8_t* tile, int row, int k, float v) {
    *reinterpret_cast<__nv_bfloat16*>(tile + muon_sw_off(row, k)) = __float2bfloat16_rn(v);
}

// Instruction descriptor for kind::f16 with BF16 A and B, FP32 D, both
// operands K-major: bits 4-5 D format (1 = F32), 7-9 A format (1 = BF16),
// 10-12 B format (1 = BF16), 17-22 N >> 3, 24-28 M >> 4.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N) {
    return (1u << 4) | (1u << 7) | (1u << 10) | (uint32_t(N >> 3) << 17) | (uint32_t(M >> 4) << 24);
}

__device__ __forceinline__ void mma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// D = A B^T over K (a multiple of 16, at most 128) for tiles a, b in the
// layout above; N rows of b.  Issued by one thread, committed to `bar`.
__device__ __forceinline__ void muon_product(uint32_t d, const uint8_t* a, const uint8_t* b, int N, int K,
                                             uint64_t* bar) {
    const uint32_t idesc = idesc_bf16(128, N);
    for (int kk = 0; kk < K / 16; ++kk) {
        const uint32_t off = uint32_t(kk >> 2) * kMuonTcChunkBytes + uint32_t(kk & 3) * 32;
        const uint64_t ad = tc::smem_desc(tc::smem_u32(a) + off, 16, 1024, tc::kLayoutSw128);
        const uint64_t bd = tc::smem_desc(tc::smem_u32(b) + off, 16, 1024, tc::kLayoutSw128);
        mma_bf16(d, ad, bd, idesc, kk > 0 ? 1u : 0u);
    }
    tc::mma_commit(bar);
}

__device__ __forceinline__ int round16(int x) { return (x + 15) & ~15; }

__global__ void __launch_bounds__(kMuonTcThreads, 1)
muon_tc_kernel(const MuonMatrix* __restrict__ mats, MuonScalars s, const float* __restrict__ lr_dev,
               int* __restrict__ err)
{
    HX_PDL_PROLOGUE();
    extern __shared__ uint8_t smem_raw[];
    MuonTcSmem& sm = *reinterpret_cast<MuonTcSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int t = threadIdx.x, warp = t >> 5;
    if (lr_dev) s.lr = *lr_dev;
    const MuonMatrix mt = mats[blockIdx.x];
    const int rows = mt.rows, cols = mt.cols;
    const bool tr = rows > cols;
    const int R = tr ? cols : rows, C = tr ? rows : cols;
    const int n = rows * cols;

    // zero the three operand tiles (contiguous: xs, xt, as), so that their
    // padding rows and K columns stay zero; set up the barrier
    static_assert(offsetof(MuonTcSmem, as) == offsetof(MuonTcSmem, xs) + 4 * kMuonTcChunkBytes, "tile order");
    for (int i = t; i < int(3 * 2 * kMuonTcChunkBytes / 16); i += kMuonTcThreads)
        reinterpret_cast<uint4*>(sm.xs)[i] = make_uint4(0, 0, 0, 0);
    if (t == 0) {
        tc::mbar_init(&sm.bar, 1);
        tc::fence_mbar_init();
        sm.abort = 0;
    }
    if (warp == 0) {
        tc::tmem_alloc(&sm.tmem, 256);
        tc::tmem_relinquish();
    }

    // momentum, Nesterov, Frobenius norm (the same roundings as muon_kernel)
    double ss = 0.0;
    for (int i = t; i < n; i += kMuonTcThreads) {
        const float bn = __fadd_rn(__fmul_rn(s.momentum, mt.buf[i]), mt.g[i]);
        mt.buf[i] = bn;
        const float u = s.nesterov ? __fadd_rn(mt.g[i], __fmul_rn(s.momentum, bn)) : bn;
        const int r = i / cols, c = i % cols;
        if (tr) sm.xf[c * kMuonXfStride + r] = u; else sm.xf[r * kMuonXfStride + c] = u;
        ss += (double)u * u;
    }
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((t & 31) == 0) sm.red[warp] = ss;
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = sm.tmem;
    const uint32_t d0 = tmem, d1 = tmem + 128;
    const uint32_t lane_addr = uint32_t(warp * 32) << 16;
    const float inv = (float)(1.0 / (sqrt(sm.red[0] + sm.red[1] + sm.red[2] + sm.red[3]) + 1e-7));
    // thread t owns row t of X: normalise it and write its bf16 copies
    if (t < R) {
        for (int c = 0; c < C; ++c) {
            const float x = __fmul_rn(sm.xf[t * kMuonXfStride + c], inv);
            sm.xf[t * kMuonXfStride + c] = x;
            muon_st_bf16(sm.xs, t, c, x);
            muon_st_bf16(sm.xt, c, t, x);
        }
    }
    const int Rp = round16(R), Cp = round16(C);
    uint32_t phase = 0;
    bool ok = true;
    auto product_done = [&]() {
        // every thread waits for the commit of the product just issued
        if (!tc::mbar_wait(&sm.bar, phase)) {
            atomicCAS(err, 0, kMuonTcErr);
            sm.abort = 1;
        }
        phase ^= 1;
        tc::tc_fence_after();
        __syncthreads();
        ok = sm.abort == 0;
    };
    auto issue = [&](uint32_t d, const uint8_t* a, const uint8_t* b, int N, int K) {
        tc::fence_proxy_async_smem();  // this thread's tile writes, before the MMA reads them
        tc::tc_fence_before();
        __syncthreads();
        if (t == 0) {
            tc::tc_fence_after();
            muon_product(d, a, b, N, K, &sm.bar);
        }
        product_done();
    };

    for (int it = 0; it < s.steps && ok; ++it) {
        // D0 = X X^T  ->  A (bf16) into the `as` tile
        issue(d0, sm.xs, sm.xs, Rp, round16(C));
        if (!ok) break;
        for (int q0 = 0; q0 < Rp; q0 += 16) {
            uint32_t v[16];
            tc::tmem_ld_32x32b_x16(d0 + lane_addr + q0, v);
            tc::tmem_ld_wait();
            if (t < R)
#pragma unroll
                for (int j = 0; j < 16; ++j)
                    if (q0 + j < R) muon_st_bf16(sm.as, t, q0 + j, __uint_as_float(v[j]));
        }
        // D1 = A A  ->  Bm = b A + c A A (bf16) over A's tile
        issue(d1, sm.as, sm.as, Rp, Rp);
        if (!ok) break;
        __syncthreads();  // every row of A has been read by the MMA before any row is overwritten
        for (int q0 = 0; q0 < Rp; q0 += 16) {
            uint32_t a0[16], a1[16];
            tc::tmem_ld_32x32b_x16(d0 + lane_addr + q0, a0);
            tc::tmem_ld_32x32b_x16(d1 + lane_addr + q0, a1);
            tc::tmem_ld_wait();
            if (t < R)
#pragma unroll
                for (int j = 0; j < 16; ++j)
                    if (q0 + j < R)
                        muon_st_bf16(sm.as, t, q0 + j, s.b * __uint_as_float(a0[j]) + s.c * __uint_as_float(a1[j]));
        }
        // D0 = Bm X  ->  X = a X + Bm X
        issue(d0, sm.as, sm.xt, Cp, Rp);
        if (!ok) break;
        for (int c0 = 0; c0 < Cp; c0 += 16) {
            uint32_t v[16];
            tc::tmem_ld_32x32b_x16(d0 + lane_addr + c0, v);
            tc::tmem_ld_wait();
            if (t < R)
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const int c = c0 + j;
                    if (c >= C) continue;
                    const float x = s.a * sm.xf[t * kMuonXfStride + c] + __uint_as_float(v[j]);
                    sm.xf[t * kMuonXfStride + c] = x;
                    muon_st_bf16(sm.xs, t, c, x);
                    muon_st_bf16(sm.xt, c, t, x);
                }
        }
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, 256);
    }
    if (!ok) return;
    const float sc = sqrtf(fmaxf(1.f, (float)rows / (float)cols));
    for (int i = t; i < n; i += kMuonTcThreads) {
        const int r = i / cols, c = i % cols;
        const float xo = tr ? sm.xf[c * kMuonXfStride + r] : sm.xf[r * kMuonXfStride + c];
        mt.w[i] = __fsub_rn(mt.w[i], __fmul_rn(s.lr, __fmul_rn(sc, xo)));
    }
}

}  // namespace hx
