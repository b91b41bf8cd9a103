// gemm_tc.cuh -- FP32-accurate GEMM on the 5th-generation tensor cores.
//
// C[M,N] = op(A)[M,K] * op(B)[K,N] in "3xTF32": every operand x is split
// into hi = x rounded to the nearest TF32 value and lo = x - hi (exact in
// FP32), and the accumulator collects hi*hi + hi*lo + lo*hi in FP32 in TMEM.
// The dropped lo*lo term and the truncation of lo to TF32 leave a relative
// error near 2^-21 per product, against 2^-11 for plain TF32 -- close to a
// CUDA-core FP32 GEMM.
//
// The MMA's FP32 accumulation truncates, which biases long sums toward
// zero; so each 32-deep k-block is accumulated fresh in TMEM, with the small
// hi*lo and lo*hi terms issued before hi*hi (four full-magnitude truncations
// per k-block), and drained into FP32 registers with round-to-nearest adds.
//
// Tile shape.  A kind::tf32 MMA with M = 128, K = 8 costs about 120 cycles
// whether N is 64 or 128, and about 140 at N = 256 with A read from TMEM
// (measured on B200: 592 vs 1020 TFLOP/s of TF32 per GPU), so tiles are
// 128 x 256.  A lives in TMEM: the A tile of each k-block is split by four
// warps, one tile row per thread, straight from the landed raw tile into a
// TMEM slot (hi 32 columns, lo 32 columns); the MMA reads only B (hi and lo)
// from shared memory.  TMEM: the 256-column accumulator and three A slots.
// The accumulator is single-buffered; the drain warps release it as soon as
// their TMEM loads have landed, before adding.
//
// Persistent: the grid is at most one CTA per SM, and each CTA walks work
// units u = blockIdx.x, blockIdx.x + gridDim.x, ...  A unit is one 128x256
// output tile of one K split; units are numbered with the N tile fastest so
// that CTAs running together share A row blocks in L2.  The operand ring and
// the A slots run on across unit boundaries, so the epilogue of one tile
// overlaps the next tile's first k-block.
//
// Roles (22 warps):
//   warp 0      TMA producers: lane 0 loads the raw A tile (16 KB) of each
//               32-deep k-block into a 4-slot ring (full_a[]), freed as soon
//               as the converters hold the values; lane 1 the B tile (hi, or
//               hi and lo when B comes pre-split; 32/64 KB) into a 2-slot
//               ring (full_b[]), freed by the MMA's commit;
//   warp 1      TMEM owner and MMA issuer: 12 tcgen05.mma (M128 N256 K8,
//               kind::tf32, A from TMEM) per k-block; tcgen05.commit frees
//               the B slot (empty_b[]) and the A slot (a_free[]) and hands the
//               accumulator to the drain warps (acc_ready);
//   warps 2-5   converters.  A: thread = tile row (TMEM lane 32(w%4) +
//               lane) reads its 32 values of the raw tile, frees the raw A
//               stage, writes hi/lo into A slot g%3 with tcgen05.st, arrives
//               on a_ready[].  B: split the stage's B tile into hi (in place)
//               and lo, fence the generic->async proxy, arrive on b_ready[];
//   warps 6-21  drain: one TMEM row per thread, 64 columns per warp, added
//               into FP32 registers; at the end of a unit, apply the epilogue
//               functor 8 columns at a time and hand each 32x8 chunk to a TMA
//               bulk store (single-output epilogues), or stage it so that each
//               store instruction writes four 32-byte row segments; the
//               epilogue's own global inputs for a chunk are loaded before
//               any is used.
// Layouts: a K-major A tile arrives 128B-swizzled (row m's 16-byte chunk c
// at ((c ^ (m & 7)) << 4)), an MN-major A tile unswizzled (K-row k at
// 512 k bytes, so that lanes read consecutive words).  B is K-major with the
// 128-byte swizzle, or MN-major as eight 32-wide boxes (LBO = 4 KB) in the
// 128-byte/32-byte-atom swizzle, the only shared-memory layout the MMA takes
// for MN-major 32-bit operands.
// Every barrier wait is bounded (tc::kWaitCycles); on timeout the kernel
// records an error code, drains its own MMAs and TMA loads (bounded), frees
// TMEM and returns.
#pragma once

#include <algorithm>

#include "tc_ptx.cuh"

namespace hx {

// A (16 KB per k-block, from HBM) and B (hi + lo, 64 KB per k-block) have
// separate rings: a raw A slot is free as soon as the converters have read
// it, so A loads run up to kTcAStages k-blocks ahead of the MMA.
constexpr int kTcBM = 128, kTcBN = 256, kTcBK = 32, kTcAStages = 4, kTcBStages = 2;
constexpr int kTcATileFloats = kTcBM * kTcBK;  // 16 KB
constexpr int kTcBTileFloats = kTcBN * kTcBK;  // 32 KB
constexpr int kTcConvWarps = 4, kTcDrainWarps = 16;
constexpr int kTcConvThreads = 32 * kTcConvWarps;
constexpr int kTcFirstDrainWarp = 2 + kTcConvWarps;
constexpr int kTcThreads = 32 * (kTcFirstDrainWarp + kTcDrainWarps);  // 704
constexpr int kTcASlots = 3;
constexpr uint32_t kTcTmemCols = 512;
constexpr uint32_t kTcColA = kTcBN;  // A slots after the accumulator: 64 columns each (hi 32, lo 32)
static_assert(kTcColA + 64 * kTcASlots <= kTcTmemCols, "TMEM budget");
constexpr int kTcStageLd = 9;  // epilogue staging row stride (floats): 8 columns + 1 pad
// TMA-store epilogue: per drain warp two 32x8 fp32 chunks (1 KB each),
// 32-byte swizzled as the output tensor map's box expects
constexpr int kTcTmaStageFloats = 2 * 32 * 8;

struct TcSmem {
    float a_raw[kTcAStages][kTcATileFloats];
    float b_hi[kTcBStages][kTcBTileFloats];
    float b_lo[kTcBStages][kTcBTileFloats];
    union {
        float stage[kTcDrainWarps][32 * kTcStageLd];
        float stage_tma[kTcDrainWarps][kTcTmaStageFloats];
    };
    uint64_t full_a[kTcAStages], empty_a[kTcAStages];
    uint64_t full_b[kTcBStages], b_ready[kTcBStages], empty_b[kTcBStages];
    uint64_t a_ready[kTcASlots], a_free[kTcASlots];
    uint64_t acc_ready, acc_free, drain;
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
// magnitude bits, clear the 13 low mantissa bits -- two integer operations,
// which matters: the split of a 128x32 A tile and a 128x32 B tile per
// k-block would otherwise fill the SM's integer pipe for as long as the
// k-block's MMAs take.  Rounding (rather than truncating) leaves lo = x - hi
// with either sign, so the MMA's own truncation of lo does not bias the
// products.  NaN and infinity pass through; finite |x| >= 0x1.fffffp+127
// (within half a TF32 ulp of FLT_MAX) rounds to infinity, outside the range
// the tensor-core paths accept.
__device__ __forceinline__ float tf32_round(float x) {
    return __uint_as_float((__float_as_uint(x) + 0x1000u) & 0xFFFFE000u);
}
__device__ __forceinline__ float4 tf32_hi(float4 x) {
    return make_float4(tf32_round(x.x), tf32_round(x.y), tf32_round(x.z), tf32_round(x.w));
}

// acc[8 c + j] for a runtime chunk c, by selection (keeps acc in registers)
__device__ __forceinline__ float chunk8(const float (&acc)[64], int c, int j) {
    float v = acc[j];
#pragma unroll
    for (int k = 1; k < 8; ++k) v = (c == k) ? acc[8 * k + j] : v;
    return v;
}

template <bool A_MN, bool B_MN, bool B_SPLIT, bool C_TMA, class Epi>
__global__ void __launch_bounds__(kTcThreads, 1)
gemm_tc_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
               const __grid_constant__ CUtensorMap map_blo, const __grid_constant__ CUtensorMap map_c, TcGrid g,
               Epi epi, float* __restrict__ partial, int* __restrict__ err)
{
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // 128B-swizzled TMA tiles and UMMA descriptors need 1024-byte alignment
    // of the shared-memory address itself.
    const uint32_t pad = (1024u - (tc::smem_u32(smem_raw) & 1023u)) & 1023u;
    TcSmem& sm = *reinterpret_cast<TcSmem*>(smem_raw + pad);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kTcAStages; ++s) {
            tc::mbar_init(&sm.full_a[s], 1);
            tc::mbar_init(&sm.empty_a[s], kTcConvWarps);  // the A warps, once they hold the values
        }
        for (int s = 0; s < kTcBStages; ++s) {
            tc::mbar_init(&sm.full_b[s], 1);
            tc::mbar_init(&sm.b_ready[s], kTcConvThreads);
            tc::mbar_init(&sm.empty_b[s], 1);             // the MMA's commit
        }
        for (int j = 0; j < kTcASlots; ++j) {
            tc::mbar_init(&sm.a_ready[j], kTcConvWarps);
            tc::mbar_init(&sm.a_free[j], 1);
        }
        tc::mbar_init(&sm.acc_ready, 1);
        tc::mbar_init(&sm.acc_free, kTcDrainWarps);
        tc::mbar_init(&sm.drain, 1);
        sm.abort = 0;
        tc::fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        tc::prefetch_tensormap(&map_a);
        tc::prefetch_tensormap(&map_b);
        if (B_SPLIT) tc::prefetch_tensormap(&map_blo);
        if (C_TMA) tc::prefetch_tensormap(&map_c);
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
        // ---------------- TMA producers: lane 0 the A ring, lane 1 the B ring
        if (lane < 2) {
            const bool ring_a = lane == 0;
            const int ns = ring_a ? kTcAStages : kTcBStages;
            uint32_t issued_parity[kTcAStages];
            bool issued[kTcAStages];
            for (int s = 0; s < kTcAStages; ++s) issued[s] = false;
            uint32_t it = 0;  // k-blocks issued by this CTA
            bool stop = false;
            for (int u = blockIdx.x; u < g.units && !stop; u += gridDim.x) {
                const TcUnit t = tc_unit(g, u);
                for (int kb = 0; kb < t.nk; ++kb, ++it) {
                    const int s = it % ns;
                    const uint32_t ph = (it / ns) & 1;
                    uint64_t* full = ring_a ? &sm.full_a[s] : &sm.full_b[s];
                    if (!tc::mbar_wait(ring_a ? &sm.empty_a[s] : &sm.empty_b[s], ph ^ 1)) {
                        tc_fail(sm, err, kTcErrProducer); stop = true; break;
                    }
                    if (tc_aborted(sm)) { stop = true; break; }
                    const int k = t.kbeg + kb * kTcBK;
                    if (ring_a) {
                        tc::mbar_arrive_expect_tx(full, kTcATileFloats * 4);
                        if (!A_MN)
                            tc::tma_load_2d(sm.a_raw[s], &map_a, full, k, t.m0);   // box 32 (K) x 128 rows
                        else
                            tc::tma_load_2d(sm.a_raw[s], &map_a, full, t.m0, k);   // box 128 (M) x 32 K-rows
                    } else {
                        tc::mbar_arrive_expect_tx(full, (B_SPLIT ? 2 : 1) * kTcBTileFloats * 4);
#pragma unroll
                        for (int part = 0; part < (B_SPLIT ? 2 : 1); ++part) {
                            float* dst = part ? sm.b_lo[s] : sm.b_hi[s];
                            const CUtensorMap* mp = part ? &map_blo : &map_b;
                            if (!B_MN) {
                                tc::tma_load_2d(dst, mp, full, k, t.n0);    // box 32 (K) x 256 rows
                            } else {
#pragma unroll
                                for (int c = 0; c < kTcBN / 32; ++c)
                                    tc::tma_load_2d(dst + c * 1024, mp, full, t.n0 + 32 * c, k);
                            }
                        }
                    }
                    issued[s] = true;
                    issued_parity[s] = ph;
                }
            }
            if (tc_aborted(sm)) {
                // let our own loads land before the CTA can exit
                for (int s = 0; s < ns; ++s)
                    if (issued[s]) tc::mbar_wait(ring_a ? &sm.full_a[s] : &sm.full_b[s], issued_parity[s]);
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            constexpr uint32_t idesc = tc::idesc_tf32(kTcBM, kTcBN, false, B_MN);
            // B K-major: SW128, SBO 1024, k-step = 32 bytes along the row.
            // B MN-major: SW128 with 32-byte atoms, SBO 512, LBO 4 KB between
            // 32-wide chunks, k-step = 8 K-rows = 1024 bytes.
            constexpr uint32_t b_lbo = B_MN ? 32 * 128 : 16, b_sbo = B_MN ? 512 : 1024;
            constexpr uint32_t b_lay = B_MN ? tc::kLayoutSw128Base32 : tc::kLayoutSw128;
            constexpr uint32_t b_step = B_MN ? 1024 : 32;
            uint32_t it = 0;
            bool stop = false;
            for (int u = blockIdx.x; u < g.units && !stop; u += gridDim.x) {
                const TcUnit t = tc_unit(g, u);
                for (int kb = 0; kb < t.nk; ++kb, ++it) {
                    const int s = it % kTcBStages;
                    const uint32_t ph = (it / kTcBStages) & 1;
                    const int j = it % kTcASlots;
                    if (!tc::mbar_wait(&sm.a_ready[j], (it / kTcASlots) & 1)) { tc_fail(sm, err, kTcErrMma); stop = true; break; }
                    if (!tc::mbar_wait(B_SPLIT ? &sm.full_b[s] : &sm.b_ready[s], ph)) { tc_fail(sm, err, kTcErrMma); stop = true; break; }
                    if (!tc::mbar_wait(&sm.acc_free, (it & 1) ^ 1)) { tc_fail(sm, err, kTcErrMma); stop = true; break; }
                    if (tc_aborted(sm)) { stop = true; break; }
                    tc::tc_fence_after();
                    const uint32_t ah = tmem + kTcColA + 64 * j, al = ah + 32;
                    const uint32_t bh = tc::smem_u32(sm.b_hi[s]), bl = tc::smem_u32(sm.b_lo[s]);
                    // hi*lo and lo*hi first, then hi*hi
#pragma unroll
                    for (int k = 0; k < kTcBK / 8; ++k) {
                        const uint64_t dbh = tc::smem_desc(bh + k * b_step, b_lbo, b_sbo, b_lay);
                        const uint64_t dbl = tc::smem_desc(bl + k * b_step, b_lbo, b_sbo, b_lay);
                        tc::mma_tf32_ts(tmem, ah + 8 * k, dbl, idesc, k > 0 ? 1u : 0u);
                        tc::mma_tf32_ts(tmem, al + 8 * k, dbh, idesc, 1u);
                    }
#pragma unroll
                    for (int k = 0; k < kTcBK / 8; ++k) {
                        const uint64_t dbh = tc::smem_desc(bh + k * b_step, b_lbo, b_sbo, b_lay);
                        tc::mma_tf32_ts(tmem, ah + 8 * k, dbh, idesc, 1u);
                    }
                    tc::mma_commit(&sm.empty_b[s]);
                    tc::mma_commit(&sm.a_free[j]);
                    tc::mma_commit(&sm.acc_ready);
                }
            }
            // drain: every MMA issued above has completed before teardown
            tc::mma_commit(&sm.drain);
            tc::mbar_wait(&sm.drain, 0);
        }
    } else if (warp < kTcFirstDrainWarp) {
        // ---------------- converters ----------------
        const int ct = threadIdx.x - 64;  // 0..kTcConvThreads-1
        const int q = warp & 3;            // TMEM lane quarter
        const int m = 32 * q + lane;       // the A tile row this thread splits
        const uint32_t a_lane = tmem + (uint32_t(32 * q) << 16) + kTcColA;
        uint32_t it = 0;
        bool stop = false;
        for (int u = blockIdx.x; u < g.units && !stop; u += gridDim.x) {
            const TcUnit t = tc_unit(g, u);
            for (int kb = 0; kb < t.nk; ++kb, ++it) {
                const int sa = it % kTcAStages, s = it % kTcBStages;
                if (!tc::mbar_wait(&sm.full_a[sa], (it / kTcAStages) & 1)) { tc_fail(sm, err, kTcErrConverter); stop = true; break; }
                if (tc_aborted(sm)) { stop = true; break; }
                {
                    // row m's 32 K-values -> hi/lo in A slot it % 3, 16 at a time
                    const int j = it % kTcASlots;
                    if (!tc::mbar_wait(&sm.a_free[j], ((it / kTcASlots) & 1) ^ 1)) {
                        tc_fail(sm, err, kTcErrConverter); stop = true; break;
                    }
                    tc::tc_fence_after();
                    const float* raw = sm.a_raw[sa];
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        float x[16];
                        if (!A_MN) {
#pragma unroll
                            for (int c = 0; c < 4; ++c) {
                                const int cc = 4 * h + c;
                                const float4 v = *reinterpret_cast<const float4*>(raw + m * 32 + ((cc ^ (m & 7)) << 2));
                                x[4 * c] = v.x; x[4 * c + 1] = v.y; x[4 * c + 2] = v.z; x[4 * c + 3] = v.w;
                            }
                        } else {
#pragma unroll
                            for (int k = 0; k < 16; ++k) x[k] = raw[(16 * h + k) * 128 + m];
                        }
                        uint32_t hi[16], lo[16];
#pragma unroll
                        for (int i = 0; i < 16; ++i) {
                            const float hv = tf32_round(x[i]);
                            hi[i] = __float_as_uint(hv);
                            lo[i] = __float_as_uint(x[i] - hv);
                        }
                        tc::tmem_st_32x32b_x16(a_lane + 64 * j + 16 * h, hi);
                        tc::tmem_st_32x32b_x16(a_lane + 64 * j + 32 + 16 * h, lo);
                    }
                    __syncwarp();
                    if (lane == 0) tc::mbar_arrive(&sm.empty_a[sa]);  // raw A read
                    tc::tmem_st_wait();
                    tc::tc_fence_before();
                    __syncwarp();
                    if (lane == 0) tc::mbar_arrive(&sm.a_ready[j]);
                }
                if (!B_SPLIT) {  // pre-split B goes from its TMA barrier straight to the MMA
                    if (!tc::mbar_wait(&sm.full_b[s], (it / kTcBStages) & 1)) {
                        tc_fail(sm, err, kTcErrConverter); stop = true; break;
                    }
                    float4* bh = reinterpret_cast<float4*>(sm.b_hi[s]);
                    float4* bl = reinterpret_cast<float4*>(sm.b_lo[s]);
#pragma unroll 4
                    for (int i = ct; i < kTcBTileFloats / 4; i += kTcConvThreads) {
                        const float4 y = bh[i];
                        const float4 gg = tf32_hi(y);
                        bh[i] = gg;
                        bl[i] = make_float4(y.x - gg.x, y.y - gg.y, y.z - gg.z, y.w - gg.w);
                    }
                    tc::fence_proxy_async_smem();
                    tc::mbar_arrive(&sm.b_ready[s]);
                }
            }
        }
    } else {
        // ---------------- drain, then epilogue ----------------
        const int dw = warp - kTcFirstDrainWarp;  // 0..15
        const int q = warp & 3;                   // TMEM lane quarter this warp may access
        const int slice = dw >> 2;                // which 64 of the 256 columns
        float* stg = sm.stage[dw];
        const uint32_t base = tmem + (uint32_t(32 * q) << 16) + uint32_t(64 * slice);
        uint32_t it = 0;
        bool stop = false;
        for (int u = blockIdx.x; u < g.units && !stop; u += gridDim.x) {
            const TcUnit t = tc_unit(g, u);
            float acc[64];
#pragma unroll
            for (int i = 0; i < 64; ++i) acc[i] = 0.f;
            for (int kb = 0; kb < t.nk; ++kb, ++it) {
                if (!tc::mbar_wait(&sm.acc_ready, it & 1)) { tc_fail(sm, err, kTcErrEpilogue); stop = true; break; }
                if (tc_aborted(sm)) { stop = true; break; }
                tc::tc_fence_after();
                // 16 columns at a time (registers: 64 sums + 16 loaded); the
                // accumulator is released once the last piece is in registers
#pragma unroll
                for (int p = 0; p < 4; ++p) {
                    uint32_t r[16];
                    tc::tmem_ld_32x32b_x16(base + 16 * p, r);
                    tc::tmem_ld_wait();
                    if (p == 3) {
                        tc::tc_fence_before();
                        __syncwarp();
                        if (lane == 0) tc::mbar_arrive(&sm.acc_free);
                    }
#pragma unroll
                    for (int i = 0; i < 16; ++i) acc[16 * p + i] = __fadd_rn(acc[16 * p + i], __uint_as_float(r[i]));
                }
            }
            if (stop || tc_aborted(sm)) break;
            const int rbase = t.m0 + 32 * q;
            const int cbase = t.n0 + 64 * slice;
            if constexpr (C_TMA) {
                // TMA-store epilogue: per 8-column chunk, lane = row applies
                // the functor, writes the chunk into one of two 32B-swizzled
                // staging buffers (row r's 16-byte half h at (h ^ ((r >> 2) & 1))),
                // and lane 0 issues one bulk store (the split-K partials go to
                // [split][M][N] through a 3-D map); rows and columns outside
                // the output are clipped by TMA
                const int row = rbase + lane;
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    const int n = cbase + c * 8;
                    float pre[8];
#pragma unroll
                    for (int i = 0; i < 8; ++i) pre[i] = 0.f;
                    if constexpr (Epi::kReads) {
                        if (!partial && row < g.M) {
                            const float* pp = epi.pre_ptr() + (long)row * epi.tma_ld() + n;
                            if (n + 8 <= g.N) {
#pragma unroll
                                for (int v4 = 0; v4 < 2; ++v4) {
                                    const float4 x4 = *reinterpret_cast<const float4*>(pp + 4 * v4);
                                    pre[4 * v4] = x4.x; pre[4 * v4 + 1] = x4.y; pre[4 * v4 + 2] = x4.z; pre[4 * v4 + 3] = x4.w;
                                }
                            } else {
                                for (int i = 0; i < 8 && n + i < g.N; ++i) pre[i] = pp[i];
                            }
                        }
                    }
                    float* buf = sm.stage_tma[dw] + (c & 1) * 256;
                    if (lane == 0) tc::bulk_wait_read<1>();  // the store that last read this buffer is done
                    __syncwarp();
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        float o[4];
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const float v = acc[8 * c + 4 * h + e];
                            o[e] = partial ? v : epi.value(v, pre[4 * h + e]);
                        }
                        *reinterpret_cast<float4*>(buf + lane * 8 + ((h ^ ((lane >> 2) & 1)) << 2)) =
                            make_float4(o[0], o[1], o[2], o[3]);
                    }
                    tc::fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) {
                        if (partial) tc::tma_store_3d(&map_c, buf, n, rbase, t.z);
                        else tc::tma_store_2d(&map_c, buf, n, rbase);
                        tc::bulk_commit();
                    }
                }
            } else {
                // Coalesced epilogue: this warp owns rows m0+32q .. +31 and
                // columns n0+64*slice .. +63.  Per 8-column chunk, lane = row
                // writes its 8 values into the staging block (row stride 9:
                // conflict-free), then lane (r, c) = (lane / 8, lane % 8) reads
                // rows 4i + r column-wise, so that each store instruction
                // writes four 32-byte row segments.
                const int rsub = lane >> 3, csub = lane & 7;
#pragma unroll 1
                for (int c = 0; c < 8; ++c) {
                    __syncwarp();
#pragma unroll
                    for (int jj = 0; jj < 8; ++jj) stg[lane * kTcStageLd + jj] = chunk8(acc, c, jj);
                    __syncwarp();
                    const int n = cbase + c * 8 + csub;
                    if (partial) {
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            const int row = rbase + 4 * i + rsub;
                            if (row < g.M && n < g.N)
                                partial[((long)t.z * g.M + row) * g.N + n] = stg[(4 * i + rsub) * kTcStageLd + csub];
                        }
                    } else if constexpr (Epi::kReads) {
                        // the chunk's global epilogue inputs, all loads in flight together
                        float pre[8];
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            const int row = rbase + 4 * i + rsub;
                            pre[i] = (row < g.M && n < g.N) ? epi.prefetch(row, n) : 0.f;
                        }
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            const int r = 4 * i + rsub;
                            const int row = rbase + r;
                            if (row < g.M && n < g.N) epi.finish(row, n, stg[r * kTcStageLd + csub], pre[i]);
                        }
                    } else {
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            const int r = 4 * i + rsub;
                            const int row = rbase + r;
                            if (row < g.M && n < g.N) epi.finish(row, n, stg[r * kTcStageLd + csub], 0.f);
                        }
                    }
                }
            }
        }
        if (C_TMA && lane == 0) tc::bulk_wait_all();  // stores complete before the CTA exits
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

// Launches the persistent kernel: min(units, SMs) CTAs.  With B_SPLIT, B
// arrives as two tensors, hi (already rounded to TF32) through mb and
// lo = B - hi through mb_lo, and is not split on the device.  With C_TMA the
// epilogue writes through mc (box 16 x 32, 64-byte swizzle; for split-K
// partials a 3-D map over [split][M][N]).
template <bool A_MN, bool B_MN, bool B_SPLIT = false, bool C_TMA = false, class Epi>
inline cudaError_t launch_tc_kernel(cudaStream_t stream, int sm_count, const CUtensorMap& ma, const CUtensorMap& mb,
                                    const CUtensorMap& mb_lo, const CUtensorMap& mc, const TcGrid& g, Epi epi,
                                    float* partial, int* err)
{
    const cudaError_t a = cudaFuncSetAttribute(gemm_tc_kernel<A_MN, B_MN, B_SPLIT, C_TMA, Epi>,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kTcSmemBytes);
    if (a != cudaSuccess) return a;
    const int grid = std::max(1, std::min(g.units, sm_count));
    gemm_tc_kernel<A_MN, B_MN, B_SPLIT, C_TMA, Epi>
        <<<grid, kTcThreads, kTcSmemBytes, stream>>>(ma, mb, mb_lo, mc, g, epi, partial, err);
    return cudaGetLastError();
}

}  // namespace hx
