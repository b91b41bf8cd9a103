// gemm_tc.cuh -- FP32-accurate GEMM on the 5th-generation tensor cores.
//
// C[M,N] = op(A)[M,K] * op(B)[K,N] in "3xTF32": every operand x is split in
// shared memory into hi = x rounded to the nearest TF32 value and
// lo = x - hi (exact in FP32), and the accumulator collects
// hi*hi + hi*lo + lo*hi in FP32 in TMEM.  The dropped lo*lo term and the
// truncation of lo to TF32 leave a relative error near 2^-21 per product,
// against 2^-11 for plain TF32 -- close to a CUDA-core FP32 GEMM.
//
// The MMA's FP32 accumulation truncates, which biases long sums toward
// zero; so each 32-deep k-block is accumulated fresh in TMEM (double
// buffered) and drained into FP32 registers with round-to-nearest adds.
// Measured against fp64 on random matrices this matches a CUDA-core FP32
// GEMM (max error ~4e-7 of max|C| at K = 1024..16384).
//
// One CTA computes one 128x128 output tile (split-K over gridDim.z):
//   warp 0      TMA producer: 128B-swizzled tiles of A and B per 32-deep
//               k-block into a 3-stage ring (full[] barriers, expect_tx);
//   warp 1      TMEM owner and MMA issuer: 4 k-steps x 3 tcgen05.mma
//               (M128 N128 K8, kind::tf32) per k-block into accumulator
//               buffer kb%2; tcgen05.commit frees the smem stage (empty[])
//               and hands the buffer to the drain warps (acc_ready[]);
//   warps 2-5   split each landed stage into hi (in place) and lo, fence the
//               generic->async proxy, arrive on lo_ready[];
//   warps 6-13  drain: one TMEM row per thread, 64 columns per warp, added
//               into FP32 registers; release the buffer (acc_free[]); at the
//               end apply the epilogue functor (or store split-K partials).
// Operands may be K-major or MN-major (instruction-descriptor bits 15/16).
// K-major tiles use the 128-byte swizzle; MN-major tiles arrive as four
// 32-wide TMA boxes (LBO = 4 KB) in the 128-byte/32-byte-atom swizzle, the
// only shared-memory layout the MMA takes for MN-major 32-bit operands.
// Every barrier wait is bounded (tc::kWaitCycles); on timeout the kernel
// records an error code, drains its own MMAs and TMA loads (bounded), frees
// TMEM and returns.
#pragma once

#include "tc_ptx.cuh"

namespace hx {

constexpr int kTcBM = 128, kTcBN = 128, kTcBK = 32, kTcStages = 3;
constexpr int kTcTileFloats = 128 * 32;   // one 128 x 32 fp32 tile = 16 KB
constexpr int kTcThreads = 448;   // 14 warps
constexpr uint32_t kTcTmemCols = 256;  // two 128-column accumulators

struct TcSmem {
    float a_hi[kTcStages][kTcTileFloats];
    float b_hi[kTcStages][kTcTileFloats];
    float a_lo[kTcStages][kTcTileFloats];
    float b_lo[kTcStages][kTcTileFloats];
    uint64_t full[kTcStages], lo_ready[kTcStages], empty[kTcStages];
    uint64_t acc_ready[2], acc_free[2], drain;
    uint32_t tmem_addr;
    int abort;
};
constexpr size_t kTcSmemBytes = sizeof(TcSmem) + 1024;  // + alignment slack

enum TcError { kTcErrProducer = 1, kTcErrConverter = 2, kTcErrMma = 3, kTcErrEpilogue = 4 };

__device__ __forceinline__ void tc_fail(TcSmem& sm, int* err, int code) {
    if (err) atomicCAS(err, 0, code);
    *reinterpret_cast<volatile int*>(&sm.abort) = 1;
}
__device__ __forceinline__ bool tc_aborted(TcSmem& sm) { return *reinterpret_cast<volatile int*>(&sm.abort) != 0; }

// Nearest TF32 value (ties away from zero): add half a TF32 ulp to the
// magnitude bits, clear the 13 low mantissa bits.  Rounding (rather than
// truncating) leaves lo = x - hi with either sign, so the MMA's own
// truncation of lo does not bias the products.  Values within a TF32 ulp of
// the largest float are truncated instead, so hi stays finite.
__device__ __forceinline__ float tf32_round(float x) {
    const uint32_t u = __float_as_uint(x);
    const uint32_t r = ((u & 0x7FFFFFFFu) >= 0x7F7FF000u) ? (u & 0xFFFFE000u) : ((u + 0x1000u) & 0xFFFFE000u);
    return __uint_as_float(r);
}
__device__ __forceinline__ float4 tf32_hi(float4 x) {
    return make_float4(tf32_round(x.x), tf32_round(x.y), tf32_round(x.z), tf32_round(x.w));
}

template <bool A_MN, bool B_MN, class Epi>
__global__ void __launch_bounds__(kTcThreads, 1)
gemm_tc_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b, int M, int N,
               int K, int k_chunk, Epi epi, float* __restrict__ partial, int* __restrict__ err)
{
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // 128B-swizzled TMA tiles and UMMA descriptors need 1024-byte alignment
    // of the shared-memory address itself.
    const uint32_t pad = (1024u - (tc::smem_u32(smem_raw) & 1023u)) & 1023u;
    TcSmem& sm = *reinterpret_cast<TcSmem*>(smem_raw + pad);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.y * kTcBM, n0 = blockIdx.x * kTcBN;
    const int kbeg = blockIdx.z * k_chunk;
    const int kend = min(K, kbeg + k_chunk);
    const int nk = kend > kbeg ? (kend - kbeg + kTcBK - 1) / kTcBK : 0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kTcStages; ++s) {
            tc::mbar_init(&sm.full[s], 1);
            tc::mbar_init(&sm.lo_ready[s], 128);
            tc::mbar_init(&sm.empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            tc::mbar_init(&sm.acc_ready[b], 1);
            tc::mbar_init(&sm.acc_free[b], 256);
        }
        tc::mbar_init(&sm.drain, 1);
        sm.abort = 0;
        tc::fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        tc::prefetch_tensormap(&map_a);
        tc::prefetch_tensormap(&map_b);
    }
    if (warp == 1) {
        tc::tmem_alloc(&sm.tmem_addr, kTcTmemCols);
        tc::tmem_relinquish();
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = sm.tmem_addr;

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            int issued_parity[kTcStages];
            bool issued[kTcStages];
            for (int s = 0; s < kTcStages; ++s) issued[s] = false;
            for (int kb = 0; kb < nk; ++kb) {
                const int s = kb % kTcStages;
                const uint32_t ph = (kb / kTcStages) & 1;
                if (!tc::mbar_wait(&sm.empty[s], ph ^ 1)) { tc_fail(sm, err, kTcErrProducer); break; }
                if (tc_aborted(sm)) break;
                tc::mbar_arrive_expect_tx(&sm.full[s], 2 * kTcTileFloats * 4);
                const int k = kbeg + kb * kTcBK;
                if (!A_MN) {
                    tc::tma_load_2d(sm.a_hi[s], &map_a, &sm.full[s], k, m0);
                } else {
#pragma unroll
                    for (int c = 0; c < 4; ++c) tc::tma_load_2d(sm.a_hi[s] + c * 1024, &map_a, &sm.full[s], m0 + 32 * c, k);
                }
                if (!B_MN) {
                    tc::tma_load_2d(sm.b_hi[s], &map_b, &sm.full[s], k, n0);
                } else {
#pragma unroll
                    for (int c = 0; c < 4; ++c) tc::tma_load_2d(sm.b_hi[s] + c * 1024, &map_b, &sm.full[s], n0 + 32 * c, k);
                }
                issued[s] = true;
                issued_parity[s] = (int)ph;
            }
            if (tc_aborted(sm)) {
                // let our own loads land before the CTA can exit
                for (int s = 0; s < kTcStages; ++s)
                    if (issued[s]) tc::mbar_wait(&sm.full[s], (uint32_t)issued_parity[s]);
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            constexpr uint32_t idesc = tc::idesc_tf32(kTcBM, kTcBN, A_MN, B_MN);
            // K-major: SW128, SBO 1024, k-step = 32 bytes along the row.
            // MN-major: SW128 with 32-byte atoms, SBO 512, LBO 4 KB between
            // 32-wide chunks, k-step = 8 K-rows = 1024 bytes.
            constexpr uint32_t a_lbo = A_MN ? 32 * 128 : 16, b_lbo = B_MN ? 32 * 128 : 16;
            constexpr uint32_t a_sbo = A_MN ? 512 : 1024, b_sbo = B_MN ? 512 : 1024;
            constexpr uint32_t a_lay = A_MN ? tc::kLayoutSw128Base32 : tc::kLayoutSw128;
            constexpr uint32_t b_lay = B_MN ? tc::kLayoutSw128Base32 : tc::kLayoutSw128;
            constexpr uint32_t a_step = A_MN ? 1024 : 32, b_step = B_MN ? 1024 : 32;
            for (int kb = 0; kb < nk; ++kb) {
                const int s = kb % kTcStages;
                const uint32_t ph = (kb / kTcStages) & 1;
                const int b = kb & 1;
                const uint32_t use = (uint32_t)(kb >> 1);
                if (!tc::mbar_wait(&sm.lo_ready[s], ph)) { tc_fail(sm, err, kTcErrMma); break; }
                if (!tc::mbar_wait(&sm.acc_free[b], (use & 1) ^ 1)) { tc_fail(sm, err, kTcErrMma); break; }
                if (tc_aborted(sm)) break;
                tc::tc_fence_after();
                const uint32_t acc = tmem + uint32_t(b * 128);
                const uint32_t ah = tc::smem_u32(sm.a_hi[s]), al = tc::smem_u32(sm.a_lo[s]);
                const uint32_t bh = tc::smem_u32(sm.b_hi[s]), bl = tc::smem_u32(sm.b_lo[s]);
#pragma unroll
                for (int k = 0; k < kTcBK / 8; ++k) {
                    const uint64_t dah = tc::smem_desc(ah + k * a_step, a_lbo, a_sbo, a_lay);
                    const uint64_t dal = tc::smem_desc(al + k * a_step, a_lbo, a_sbo, a_lay);
                    const uint64_t dbh = tc::smem_desc(bh + k * b_step, b_lbo, b_sbo, b_lay);
                    const uint64_t dbl = tc::smem_desc(bl + k * b_step, b_lbo, b_sbo, b_lay);
                    tc::mma_tf32(acc, dah, dbh, idesc, k > 0 ? 1u : 0u);
                    tc::mma_tf32(acc, dah, dbl, idesc, 1u);
                    tc::mma_tf32(acc, dal, dbh, idesc, 1u);
                }
                tc::mma_commit(&sm.empty[s]);
                tc::mma_commit(&sm.acc_ready[b]);
            }
            // drain: every MMA issued above has completed before teardown
            tc::mma_commit(&sm.drain);
            tc::mbar_wait(&sm.drain, 0);
        }
    } else if (warp < 6) {
        // ---------------- converter ----------------
        const int ct = threadIdx.x - 64;  // 0..127
        for (int kb = 0; kb < nk; ++kb) {
            const int s = kb % kTcStages;
            const uint32_t ph = (kb / kTcStages) & 1;
            if (!tc::mbar_wait(&sm.full[s], ph)) { tc_fail(sm, err, kTcErrConverter); break; }
            if (tc_aborted(sm)) break;
            float4* ah = reinterpret_cast<float4*>(sm.a_hi[s]);
            float4* al = reinterpret_cast<float4*>(sm.a_lo[s]);
            float4* bh = reinterpret_cast<float4*>(sm.b_hi[s]);
            float4* bl = reinterpret_cast<float4*>(sm.b_lo[s]);
#pragma unroll 4
            for (int i = ct; i < kTcTileFloats / 4; i += 128) {
                const float4 x = ah[i];
                const float4 h = tf32_hi(x);
                ah[i] = h;
                al[i] = make_float4(x.x - h.x, x.y - h.y, x.z - h.z, x.w - h.w);
                const float4 y = bh[i];
                const float4 g = tf32_hi(y);
                bh[i] = g;
                bl[i] = make_float4(y.x - g.x, y.y - g.y, y.z - g.z, y.w - g.w);
            }
            tc::fence_proxy_async_smem();
            tc::mbar_arrive(&sm.lo_ready[s]);
        }
    } else {
        // ---------------- drain, then epilogue ----------------
        const int q = warp & 3;          // TMEM lane quarter this warp may access
        const int half = (warp - 6) >> 2;  // which 64 of the 128 columns
        const int row = m0 + 32 * q + lane;
        float acc[64];
#pragma unroll
        for (int i = 0; i < 64; ++i) acc[i] = 0.f;
        bool ok = true;
        for (int kb = 0; kb < nk; ++kb) {
            const int b = kb & 1;
            const uint32_t use = (uint32_t)(kb >> 1);
            if (!tc::mbar_wait(&sm.acc_ready[b], use & 1)) { tc_fail(sm, err, kTcErrEpilogue); ok = false; break; }
            if (tc_aborted(sm)) { ok = false; break; }
            tc::tc_fence_after();
            uint32_t r0[32], r1[32];
            const uint32_t base = tmem + (uint32_t(32 * q) << 16) + uint32_t(b * 128 + 64 * half);
            tc::tmem_ld_32x32b_x32(base, r0);
            tc::tmem_ld_32x32b_x32(base + 32, r1);
            tc::tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                acc[i] = __fadd_rn(acc[i], __uint_as_float(r0[i]));
                acc[32 + i] = __fadd_rn(acc[32 + i], __uint_as_float(r1[i]));
            }
            tc::tc_fence_before();
            tc::mbar_arrive(&sm.acc_free[b]);
        }
        if (ok && !tc_aborted(sm) && row < M) {
            const int nb = n0 + 64 * half;
#pragma unroll
            for (int i = 0; i < 64; ++i) {
                const int n = nb + i;
                if (n < N) {
                    if (partial)
                        partial[((long)blockIdx.z * M + row) * N + n] = acc[i];
                    else
                        epi(row, n, acc[i]);
                }
            }
        }
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, kTcTmemCols);
    }
}

}  // namespace hx
