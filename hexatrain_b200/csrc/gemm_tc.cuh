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
// zero; so each 32-deep k-block is accumulated fresh in TMEM and drained
// into FP32 registers with round-to-nearest adds.  Measured against fp64 on
// random matrices this matches a CUDA-core FP32 GEMM (max error ~4e-7 of
// max|C| at K = 1024..16384).
//
// Persistent: the grid is at most one CTA per SM, and each CTA walks work
// units u = blockIdx.x, blockIdx.x + gridDim.x, ...  A unit is one 128x128
// output tile of one K split; units are numbered with the N tile fastest so
// that CTAs running together share A row blocks in L2.  The operand ring and
// the accumulator buffers run on across unit boundaries, so the epilogue of
// one tile overlaps the k-loop of the next.
//
// Roles (16 warps):
//   warp 0      TMA producer: 128B-swizzled tiles of A and B per 32-deep
//               k-block into a 3-stage ring (full[] barriers, expect_tx);
//   warp 1      TMEM owner and MMA issuer: 4 k-steps x 3 tcgen05.mma
//               (M128 N128 K8, kind::tf32) per k-block into accumulator
//               buffer g%4 (g counts this CTA's k-blocks); tcgen05.commit
//               frees the smem stage (empty[]) and hands the buffer to the
//               drain warps (acc_ready[]);
//   warps 2-7   split each landed stage into hi (in place) and lo, fence the
//               generic->async proxy, arrive on lo_ready[];
//   warps 8-15  drain: one TMEM row per thread, 64 columns per warp, added
//               into FP32 registers; release the buffer (acc_free[]); at the
//               end of a unit, stage the 32x64 block through shared memory
//               16 columns at a time so that each store instruction writes
//               two 64-byte row segments (coalesced), applying the epilogue
//               functor (or storing split-K partials); the epilogue's own
//               global inputs for a chunk are loaded before any is used.
// Operands may be K-major or MN-major (instruction-descriptor bits 15/16).
// K-major tiles use the 128-byte swizzle; MN-major tiles arrive as four
// 32-wide TMA boxes (LBO = 4 KB) in the 128-byte/32-byte-atom swizzle, the
// only shared-memory layout the MMA takes for MN-major 32-bit operands.
// Every barrier wait is bounded (tc::kWaitCycles); on timeout the kernel
// records an error code, drains its own MMAs and TMA loads (bounded), frees
// TMEM and returns.
#pragma once

#include <algorithm>

#include "tc_ptx.cuh"

namespace hx {

constexpr int kTcBM = 128, kTcBN = 128, kTcBK = 32, kTcStages = 3;
constexpr int kTcTileFloats = 128 * 32;   // one 128 x 32 fp32 tile = 16 KB
constexpr int kTcConvWarps = 6, kTcDrainWarps = 8;
constexpr int kTcConvThreads = 32 * kTcConvWarps;
constexpr int kTcFirstDrainWarp = 2 + kTcConvWarps;
constexpr int kTcThreads = 32 * (kTcFirstDrainWarp + kTcDrainWarps);  // 512
constexpr int kTcAccBufs = 4;
constexpr uint32_t kTcTmemCols = 128 * kTcAccBufs;  // 512: four 128-column accumulators
constexpr int kTcStageLd = 17;  // epilogue staging row stride (floats): 16 columns + 1 pad

struct TcSmem {
    float a_hi[kTcStages][kTcTileFloats];
    float b_hi[kTcStages][kTcTileFloats];
    float a_lo[kTcStages][kTcTileFloats];
    float b_lo[kTcStages][kTcTileFloats];
    float stage[kTcDrainWarps][32 * kTcStageLd];
    uint64_t full[kTcStages], lo_ready[kTcStages], empty[kTcStages];
    uint64_t acc_ready[kTcAccBufs], acc_free[kTcAccBufs], drain;
    uint32_t tmem_addr;
    int abort;
};
constexpr size_t kTcSmemBytes = sizeof(TcSmem) + 1024;  // + alignment slack
static_assert(kTcSmemBytes <= 232448, "tcgen05 GEMM shared memory exceeds the 227 KB per-CTA limit");

enum TcError { kTcErrProducer = 1, kTcErrConverter = 2, kTcErrMma = 3, kTcErrEpilogue = 4 };

// Work decomposition shared by every role.
struct TcGrid {
    int M, N, K;
    int tiles_m, tiles_n, splits;
    int k_chunk;   // multiple of kTcBK
    int units;     // tiles_m * tiles_n * splits
};

struct TcUnit {
    int m0, n0, z, kbeg, nk;
};

__device__ __forceinline__ TcUnit tc_unit(const TcGrid& g, int u) {
    TcUnit t;
    const int tn = u % g.tiles_n;
    const int rest = u / g.tiles_n;
    const int tm = rest % g.tiles_m;
    t.z = rest / g.tiles_m;
    t.m0 = tm * kTcBM;
    t.n0 = tn * kTcBN;
    t.kbeg = t.z * g.k_chunk;
    const int kend = min(g.K, t.kbeg + g.k_chunk);
    t.nk = kend > t.kbeg ? (kend - t.kbeg + kTcBK - 1) / kTcBK : 0;
    return t;
}

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
gemm_tc_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b, TcGrid g, Epi epi,
               float* __restrict__ partial, int* __restrict__ err)
{
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // 128B-swizzled TMA tiles and UMMA descriptors need 1024-byte alignment
    // of the shared-memory address itself.
    const uint32_t pad = (1024u - (tc::smem_u32(smem_raw) & 1023u)) & 1023u;
    TcSmem& sm = *reinterpret_cast<TcSmem*>(smem_raw + pad);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kTcStages; ++s) {
            tc::mbar_init(&sm.full[s], 1);
            tc::mbar_init(&sm.lo_ready[s], kTcConvThreads);
            tc::mbar_init(&sm.empty[s], 1);
        }
        for (int b = 0; b < kTcAccBufs; ++b) {
            tc::mbar_init(&sm.acc_ready[b], 1);
            tc::mbar_init(&sm.acc_free[b], 32 * kTcDrainWarps);
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
            uint32_t issued_parity[kTcStages];
            bool issued[kTcStages];
            for (int s = 0; s < kTcStages; ++s) issued[s] = false;
            uint32_t it = 0;  // k-blocks issued by this CTA
            bool stop = false;
            for (int u = blockIdx.x; u < g.units && !stop; u += gridDim.x) {
                const TcUnit t = tc_unit(g, u);
                for (int kb = 0; kb < t.nk; ++kb, ++it) {
                    const int s = it % kTcStages;
                    const uint32_t ph = (it / kTcStages) & 1;
                    if (!tc::mbar_wait(&sm.empty[s], ph ^ 1)) { tc_fail(sm, err, kTcErrProducer); stop = true; break; }
                    if (tc_aborted(sm)) { stop = true; break; }
                    tc::mbar_arrive_expect_tx(&sm.full[s], 2 * kTcTileFloats * 4);
                    const int k = t.kbeg + kb * kTcBK;
                    if (!A_MN) {
                        tc::tma_load_2d(sm.a_hi[s], &map_a, &sm.full[s], k, t.m0);
                    } else {
#pragma unroll
                        for (int c = 0; c < 4; ++c)
                            tc::tma_load_2d(sm.a_hi[s] + c * 1024, &map_a, &sm.full[s], t.m0 + 32 * c, k);
                    }
                    if (!B_MN) {
                        tc::tma_load_2d(sm.b_hi[s], &map_b, &sm.full[s], k, t.n0);
                    } else {
#pragma unroll
                        for (int c = 0; c < 4; ++c)
                            tc::tma_load_2d(sm.b_hi[s] + c * 1024, &map_b, &sm.full[s], t.n0 + 32 * c, k);
                    }
                    issued[s] = true;
                    issued_parity[s] = ph;
                }
            }
            if (tc_aborted(sm)) {
                // let our own loads land before the CTA can exit
                for (int s = 0; s < kTcStages; ++s)
                    if (issued[s]) tc::mbar_wait(&sm.full[s], issued_parity[s]);
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
            uint32_t it = 0;
            bool stop = false;
            for (int u = blockIdx.x; u < g.units && !stop; u += gridDim.x) {
                const TcUnit t = tc_unit(g, u);
                for (int kb = 0; kb < t.nk; ++kb, ++it) {
                    const int s = it % kTcStages;
                    const uint32_t ph = (it / kTcStages) & 1;
                    const int b = it % kTcAccBufs;
                    const uint32_t use = it / kTcAccBufs;
                    if (!tc::mbar_wait(&sm.lo_ready[s], ph)) { tc_fail(sm, err, kTcErrMma); stop = true; break; }
                    if (!tc::mbar_wait(&sm.acc_free[b], (use & 1) ^ 1)) { tc_fail(sm, err, kTcErrMma); stop = true; break; }
                    if (tc_aborted(sm)) { stop = true; break; }
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
            }
            // drain: every MMA issued above has completed before teardown
            tc::mma_commit(&sm.drain);
            tc::mbar_wait(&sm.drain, 0);
        }
    } else if (warp < kTcFirstDrainWarp) {
        // ---------------- converter ----------------
        const int ct = threadIdx.x - 64;  // 0..kTcConvThreads-1
        uint32_t it = 0;
        bool stop = false;
        for (int u = blockIdx.x; u < g.units && !stop; u += gridDim.x) {
            const TcUnit t = tc_unit(g, u);
            for (int kb = 0; kb < t.nk; ++kb, ++it) {
                const int s = it % kTcStages;
                const uint32_t ph = (it / kTcStages) & 1;
                if (!tc::mbar_wait(&sm.full[s], ph)) { tc_fail(sm, err, kTcErrConverter); stop = true; break; }
                if (tc_aborted(sm)) { stop = true; break; }
                float4* ah = reinterpret_cast<float4*>(sm.a_hi[s]);
                float4* al = reinterpret_cast<float4*>(sm.a_lo[s]);
                float4* bh = reinterpret_cast<float4*>(sm.b_hi[s]);
                float4* bl = reinterpret_cast<float4*>(sm.b_lo[s]);
#pragma unroll 2
                for (int i = ct; i < kTcTileFloats / 4; i += kTcConvThreads) {
                    const float4 x = ah[i];
                    const float4 y = bh[i];
                    const float4 h = tf32_hi(x);
                    const float4 gg = tf32_hi(y);
                    ah[i] = h;
                    al[i] = make_float4(x.x - h.x, x.y - h.y, x.z - h.z, x.w - h.w);
                    bh[i] = gg;
                    bl[i] = make_float4(y.x - gg.x, y.y - gg.y, y.z - gg.z, y.w - gg.w);
                }
                tc::fence_proxy_async_smem();
                tc::mbar_arrive(&sm.lo_ready[s]);
            }
        }
    } else {
        // ---------------- drain, then epilogue ----------------
        const int dw = warp - kTcFirstDrainWarp;  // 0..7
        const int q = warp & 3;                   // TMEM lane quarter this warp may access
        const int half = dw >> 2;                 // which 64 of the 128 columns
        float* stg = sm.stage[dw];
        uint32_t it = 0;
        bool stop = false;
        for (int u = blockIdx.x; u < g.units && !stop; u += gridDim.x) {
            const TcUnit t = tc_unit(g, u);
            float acc[64];
#pragma unroll
            for (int i = 0; i < 64; ++i) acc[i] = 0.f;
            for (int kb = 0; kb < t.nk; ++kb, ++it) {
                const int b = it % kTcAccBufs;
                const uint32_t use = it / kTcAccBufs;
                if (!tc::mbar_wait(&sm.acc_ready[b], use & 1)) { tc_fail(sm, err, kTcErrEpilogue); stop = true; break; }
                if (tc_aborted(sm)) { stop = true; break; }
                tc::tc_fence_after();
                const uint32_t base = tmem + (uint32_t(32 * q) << 16) + uint32_t(b * 128 + 64 * half);
#pragma unroll
                for (int h2 = 0; h2 < 2; ++h2) {  // two 32-column loads keep 32 temporaries live
                    uint32_t r[32];
                    tc::tmem_ld_32x32b_x32(base + 32 * h2, r);
                    tc::tmem_ld_wait();
#pragma unroll
                    for (int i = 0; i < 32; ++i) acc[32 * h2 + i] = __fadd_rn(acc[32 * h2 + i], __uint_as_float(r[i]));
                }
                tc::tc_fence_before();
                tc::mbar_arrive(&sm.acc_free[b]);
            }
            if (stop || tc_aborted(sm)) break;
            // Coalesced epilogue: this warp owns rows m0+32q .. +31 and
            // columns n0+64*half .. +63.  Per 16-column chunk, lane = row
            // writes its 16 values into the staging block (row stride 17:
            // conflict-free), then lanes 0-15 / 16-31 read rows 2i / 2i+1
            // column-wise and store 16 consecutive columns each.
            const int rbase = t.m0 + 32 * q;
            const int cbase = t.n0 + 64 * half;
            const int rsub = lane >> 4, csub = lane & 15;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                __syncwarp();
#pragma unroll
                for (int j = 0; j < 16; ++j) stg[lane * kTcStageLd + j] = acc[c * 16 + j];
                __syncwarp();
                const int n = cbase + c * 16 + csub;
                if (partial) {
#pragma unroll 4
                    for (int i = 0; i < 16; ++i) {
                        const int row = rbase + 2 * i + rsub;
                        if (row < g.M && n < g.N)
                            partial[((long)t.z * g.M + row) * g.N + n] = stg[(2 * i + rsub) * kTcStageLd + csub];
                    }
                } else if constexpr (Epi::kReads) {
                    // the chunk's global epilogue inputs, all loads in flight together
                    float pre[16];
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const int row = rbase + 2 * i + rsub;
                        pre[i] = (row < g.M && n < g.N) ? epi.prefetch(row, n) : 0.f;
                    }
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const int r = 2 * i + rsub;
                        const int row = rbase + r;
                        if (row < g.M && n < g.N) epi.finish(row, n, stg[r * kTcStageLd + csub], pre[i]);
                    }
                } else {
#pragma unroll 4
                    for (int i = 0; i < 16; ++i) {
                        const int r = 2 * i + rsub;
                        const int row = rbase + r;
                        if (row < g.M && n < g.N) epi.finish(row, n, stg[r * kTcStageLd + csub], 0.f);
                    }
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

// Work split for an M x N x K problem: with fewer output tiles than SMs and
// a long K, split K so that tiles x splits fills the SMs in a single wave
// (each split at least 256 deep).  `max_splits` = 1 forbids splitting.
inline TcGrid tc_grid(int M, int N, int K, int sm_count, int max_splits) {
    TcGrid g{};
    g.M = M; g.N = N; g.K = K;
    g.tiles_m = (M + kTcBM - 1) / kTcBM;
    g.tiles_n = (N + kTcBN - 1) / kTcBN;
    const long tiles = (long)g.tiles_m * g.tiles_n;
    int splits = 1;
    if (max_splits > 1 && tiles < sm_count && K >= 2 * 256) {
        splits = (int)(sm_count / tiles);
        splits = std::max(1, std::min({splits, K / 256, max_splits}));
    }
    int chunk = (K + splits - 1) / splits;
    chunk = std::max(kTcBK, ((chunk + kTcBK - 1) / kTcBK) * kTcBK);
    splits = std::max(1, (K + chunk - 1) / chunk);
    g.splits = splits;
    g.k_chunk = chunk;
    g.units = (int)(tiles * splits);
    return g;
}

// Launches the persistent kernel: min(units, SMs) CTAs.
template <bool A_MN, bool B_MN, class Epi>
inline cudaError_t launch_tc_kernel(cudaStream_t stream, int sm_count, const CUtensorMap& ma, const CUtensorMap& mb,
                                    const TcGrid& g, Epi epi, float* partial, int* err)
{
    const cudaError_t a = cudaFuncSetAttribute(gemm_tc_kernel<A_MN, B_MN, Epi>,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kTcSmemBytes);
    if (a != cudaSuccess) return a;
    const int grid = std::max(1, std::min(g.units, sm_count));
    gemm_tc_kernel<A_MN, B_MN, Epi><<<grid, kTcThreads, kTcSmemBytes, stream>>>(ma, mb, g, epi, partial, err);
    return cudaGetLastError();
}

}  // namespace hx
