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
// CTA pairs.  The kernel runs as clusters of two CTAs on two SMs, and the
// even CTA issues tcgen05.mma with cta_group::2 (kind::tf32, M = 256,
// N = 256, K = 8): CTA r holds rows [128 r, 128 r + 128) of either operand in
// its shared memory and receives rows [128 r, ...) of the product in its own
// TMEM.  Measured on B200 one such instruction costs what an M = 128, N = 256
// one costs on a single SM (about 175 cycles), so per SM the rate is the same
// while each SM stages and the MMA reads only half of the N-side operand.
//
// Orientation.  A pair tile is 256 output rows x 256 output columns,
// computed transposed: the MMA's A operand is op(B)^T (the 256 output
// columns; CTA r holds columns n0 + 128 r ...) and its B operand is op(A)
// (the 256 output rows; CTA r holds rows m0 + 128 r ...).  TMEM lane l of
// CTA r then holds output column n0 + 128 r + l, and TMEM column c output
// row m0 + c: a warp that drains 32 lanes holds 32 consecutive columns of
// each row, so the epilogue's global loads and stores are whole 128-byte row
// segments straight from registers, with no staging.
//
// The accumulator is double-buffered (two 256-column buffers fill the 512
// TMEM columns): the MMAs of one k-block run while the drain warps read the
// previous k-block's sums out of the other buffer.
//
// Persistent: the grid is at most the number of pairs that fit at once, and
// pair p walks work units u = p, p + pairs, ...  A unit is one 256x256
// output tile of one K split; units are numbered with the column tile
// fastest so that pairs running together share op(A) row blocks in L2.  The
// rings run on across unit boundaries.
//
// Shared memory per CTA (224 KB): three stages of this CTA's op(B) tile ("W",
// 128 x 32, hi and lo) and op(A) tile ("X", 128 x 32, hi and lo), and two
// landing buffers for raw X tiles.  W tiles arrive already split when B is
// pre-split (weights), else raw into the hi half and are split in place; X
// tiles land raw and are split from there into a free X stage, so the next
// tile's load overlaps the current tile's split.
//
// Roles (22 warps per CTA):
//   warp 0      TMA producers: lane 0 this CTA's W tiles, lane 1 its raw X
//               tiles;
//   warp 1      TMEM allocation for the pair; in the even CTA, lane 0 issues
//               the 12 pair MMAs of each k-block into accumulator buffer
//               (k-block & 1) and commits to both CTAs' barriers: the W and
//               X stages are free, the buffer is ready;
//   warps 2-5   converters: split the W stage (unless pre-split) and the
//               landed X tile, then arrive on the even CTA's ready barriers;
//   warps 6-21  drain: warp (quarter q, slice s) adds TMEM lanes 32q..32q+31
//               and columns 64s..64s+63 of each k-block's buffer into FP32
//               registers and arrives on the even CTA's buffer-free barrier
//               once its loads have landed; at the end of a unit it applies
//               the epilogue functor row by row (output columns on lanes).
// Layouts: K-major tiles arrive 128B-swizzled (row r's 16-byte chunk c at
// ((c ^ (r & 7)) << 4)); MN-major tiles as 32-wide boxes (4 KB apart) in the
// 128-byte/32-byte-atom swizzle, the only shared-memory layout the MMA takes
// for MN-major 32-bit operands.  The hi/lo split is elementwise, so split
// tiles keep the layout TMA wrote.
// Every barrier wait is bounded (tc::kWaitCycles); on timeout the kernel
// records an error code, drains its own MMAs and TMA loads (bounded), meets
// the other CTA at the cluster barrier, frees TMEM and returns.
#pragma once

#include "pdl.cuh"

#include <algorithm>

#include "tc_ptx.cuh"

namespace hx {

constexpr int kTcBM = 256, kTcBN = 256, kTcBK = 32;  // pair tile: output rows, output columns; K per k-block
constexpr int kTcHalf = 128;                         // rows of either operand one CTA of the pair holds
constexpr int kTcStages = 3;                         // W and X stages (hi and lo)
constexpr int kTcTileFloats = kTcHalf * kTcBK;       // 16 KB
constexpr int kTcConvWarps = 6, kTcDrainWarps = 16;
constexpr int kTcStoreRows = 16;                     // rows per TMA-store chunk of a drain warp (32 x 16, 2 KB)
constexpr int kTcConvThreads = 32 * kTcConvWarps;
constexpr int kTcFirstDrainWarp = 2 + kTcConvWarps;
constexpr int kTcThreads = 32 * (kTcFirstDrainWarp + kTcDrainWarps);  // 768
// Registers: the kernel is built for 80 per thread (768 threads on one SM);
// the producer/MMA/converter warpgroups give theirs down to 48 and the four
// drain warpgroups, which hold 64 running sums per thread, take 96:
// 256 x 48 + 512 x 96 = 768 x 80.
constexpr int kTcRegsLaunch = 80, kTcRegsLow = 48, kTcRegsDrain = 96;
static_assert(kTcFirstDrainWarp % 4 == 0, "warpgroups must not mix drain and other warps");
static_assert(32 * kTcFirstDrainWarp * kTcRegsLow + 32 * kTcDrainWarps * kTcRegsDrain <= kTcThreads * kTcRegsLaunch,
              "register split exceeds the registers the CTA is launched with");
constexpr uint32_t kTcTmemCols = 512;                // two 256-column accumulators
constexpr uint32_t kTcAccCols = kTcBM;

struct TcSmem {
    float w_hi[kTcStages][kTcTileFloats];
    float w_lo[kTcStages][kTcTileFloats];
    float x_hi[kTcStages][kTcTileFloats];
    float x_lo[kTcStages][kTcTileFloats];
    float stage[kTcDrainWarps][kTcStoreRows * 32];   // TMA-store staging, one chunk per drain warp
    // this CTA's own TMA loads
    uint64_t w_full[kTcStages], x_full[kTcStages];
    // arrived on by the pair MMA's commit, in both CTAs
    uint64_t w_empty[kTcStages], x_empty[kTcStages], acc_ready[2];
    // used in the even CTA only, arrived on by both CTAs
    uint64_t w_ready[kTcStages], x_ready[kTcStages], acc_free[2];
    uint64_t drain;
    uint32_t tmem_addr;
    int abort;
};
constexpr size_t kTcSmemBytes = sizeof(TcSmem) + 1024;  // + alignment slack
static_assert(kTcSmemBytes <= 232448, "tcgen05 GEMM shared memory exceeds the 227 KB per-CTA limit");
static_assert((232448 >> 4) < (1 << 14), "shared addresses fit a descriptor's 14-bit start-address field");

enum TcError { kTcErrProducer = 1, kTcErrConverter = 2, kTcErrMma = 3, kTcErrEpilogue = 4 };

// Work decomposition shared by every role of both CTAs of a pair.
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
// which matters: the split of the operand tiles of every k-block would
// otherwise keep the SM's integer pipe busy for much of the time the
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

// Splits one 16 KB tile `src` into hi (to `hi`, which may be `src`) and lo;
// thread t of the converter warps takes every kTcConvThreads-th float4.
__device__ __forceinline__ void tc_split_tile(const float* src, float* hi, float* lo, int t) {
    const float4* s4 = reinterpret_cast<const float4*>(src);
    float4* h4 = reinterpret_cast<float4*>(hi);
    float4* l4 = reinterpret_cast<float4*>(lo);
#pragma unroll
    for (int i = t; i < kTcTileFloats / 4; i += kTcConvThreads) {
        const float4 y = s4[i];
        const float4 h = tf32_hi(y);
        h4[i] = h;
        l4[i] = make_float4(y.x - h.x, y.y - h.y, y.z - h.z, y.w - h.w);
    }
}

// TMA loads of one k-block's 128-row tile of a [rows][K] operand (K-major:
// one box of 32 K x 128 rows) or a [K][rows] operand (MN-major: four boxes of
// 32 x 32 K-rows, 4 KB apart).
template <bool MN>
__device__ __forceinline__ void tc_load_tile(float* dst, const CUtensorMap* map, uint64_t* bar, int k, int r0) {
    if (!MN) {
        tc::tma_load_2d(dst, map, bar, k, r0);
    } else {
#pragma unroll
        for (int c = 0; c < kTcHalf / 32; ++c) tc::tma_load_2d(dst + c * 1024, map, bar, r0 + 32 * c, k);
    }
}

// Shared-memory descriptor of k-step kk (8 K) of a split tile: K-major
// 128B-swizzled rows of 128 bytes (SBO 1024, k-step 32 bytes), or MN-major
// 32-wide boxes 4 KB apart (LBO), 4-K-row atoms 512 bytes apart (SBO),
// k-step 8 K-rows = 1024 bytes.
template <bool MN>
__device__ __forceinline__ uint64_t tc_desc(const float* tile, int kk) {
    return MN ? tc::smem_desc(tc::smem_u32(tile) + kk * 1024, 32 * 128, 512, tc::kLayoutSw128Base32)
              : tc::smem_desc(tc::smem_u32(tile) + kk * 32, 16, 1024, tc::kLayoutSw128);
}

template <bool A_MN, bool B_MN, bool B_SPLIT, bool C_TMA, class Epi>
__global__ void __launch_bounds__(kTcThreads, 1)
gemm_tc_kernel(const __grid_constant__ CUtensorMap map_x, const __grid_constant__ CUtensorMap map_w,
               const __grid_constant__ CUtensorMap map_wlo, const __grid_constant__ CUtensorMap map_c, TcGrid g,
               Epi epi, float* __restrict__ partial, int* __restrict__ err)
{
    HX_PDL_PROLOGUE();
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // 128B-swizzled TMA tiles and UMMA descriptors need 1024-byte alignment
    // of the shared-memory address itself (the same offset in both CTAs).
    const uint32_t pad = (1024u - (tc::smem_u32(smem_raw) & 1023u)) & 1023u;
    TcSmem& sm = *reinterpret_cast<TcSmem*>(smem_raw + pad);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = tc::cluster_ctarank();           // 0: issues the pair's MMAs
    const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kTcStages; ++s) {
            tc::mbar_init(&sm.w_full[s], 1);
            tc::mbar_init(&sm.x_full[s], 1);
            tc::mbar_init(&sm.w_empty[s], 1);
            tc::mbar_init(&sm.x_empty[s], 1);
            tc::mbar_init(&sm.w_ready[s], 2 * kTcConvWarps);
            tc::mbar_init(&sm.x_ready[s], 2 * kTcConvWarps);
        }
        for (int b = 0; b < 2; ++b) {
            tc::mbar_init(&sm.acc_ready[b], 1);
            tc::mbar_init(&sm.acc_free[b], 2 * kTcDrainWarps);
        }
        tc::mbar_init(&sm.drain, 1);
        sm.abort = 0;
        tc::fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        tc::prefetch_tensormap(&map_x);
        tc::prefetch_tensormap(&map_w);
        if (B_SPLIT) tc::prefetch_tensormap(&map_wlo);
        if (C_TMA) tc::prefetch_tensormap(&map_c);
    }
    if (warp == 1) {
        tc::tmem_alloc_pair(&sm.tmem_addr, kTcTmemCols);
        tc::tmem_relinquish_pair();
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::cluster_sync();  // both CTAs' barriers exist before either arrives on the other's
    tc::tc_fence_after();
    const uint32_t tmem = sm.tmem_addr;

    if (warp < kTcFirstDrainWarp) tc::setmaxnreg_dec<kTcRegsLow>();
    if (warp == 0) {
        // ---------------- TMA producers: lane 0 the W tiles, lane 1 the X tiles
        if (lane < 2) {
            const bool ring_w = lane == 0;
            const int ns = kTcStages;
            uint32_t issued = 0, issued_parity = 0;  // per stage: a load was issued, and its phase parity
            uint32_t it = 0;  // k-blocks issued by this CTA
            bool stop = false;
            for (int u = pair; u < g.units && !stop; u += npairs) {
                const TcUnit t = tc_unit(g, u);
                for (int kb = 0; kb < t.nk; ++kb, ++it) {
                    const int s = it % ns;
                    const uint32_t ph = (it / ns) & 1;
                    if (!tc::mbar_wait(ring_w ? &sm.w_empty[s] : &sm.x_empty[s], ph ^ 1)) {
                        tc_fail(sm, err, kTcErrProducer); stop = true; break;
                    }
                    if (tc_aborted(sm)) { stop = true; break; }
                    const int k = t.kbeg + kb * kTcBK;
                    if (ring_w) {
                        tc::mbar_arrive_expect_tx(&sm.w_full[s], (B_SPLIT ? 2 : 1) * kTcTileFloats * 4);
                        tc_load_tile<B_MN>(sm.w_hi[s], &map_w, &sm.w_full[s], k, t.n0 + kTcHalf * rank);
                        if (B_SPLIT) tc_load_tile<B_MN>(sm.w_lo[s], &map_wlo, &sm.w_full[s], k, t.n0 + kTcHalf * rank);
                    } else {
                        tc::mbar_arrive_expect_tx(&sm.x_full[s], kTcTileFloats * 4);
                        tc_load_tile<A_MN>(sm.x_hi[s], &map_x, &sm.x_full[s], k, t.m0 + kTcHalf * rank);
                    }
                    issued |= 1u << s;
                    issued_parity = (issued_parity & ~(1u << s)) | (ph << s);
                }
            }
            if (tc_aborted(sm)) {
                // let our own loads land before the CTA can exit
                for (int s = 0; s < ns; ++s)
                    if ((issued >> s) & 1u) tc::mbar_wait(ring_w ? &sm.w_full[s] : &sm.x_full[s], (issued_parity >> s) & 1u);
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer (even CTA of the pair) ----------------
        if (lane == 0 && rank == 0) {
            // MMA A = op(B)^T (256 output columns, 128 per CTA),
            // MMA B = op(A) (256 output rows, 128 per CTA)
            constexpr uint32_t idesc = tc::idesc_tf32(2 * kTcHalf, kTcBM, B_MN, A_MN);
            uint32_t it = 0;
            bool stop = false;
            for (int u = pair; u < g.units && !stop; u += npairs) {
                const TcUnit t = tc_unit(g, u);
                for (int kb = 0; kb < t.nk; ++kb, ++it) {
                    const int s = it % kTcStages;
                    const uint32_t ph = (it / kTcStages) & 1;
                    const int b = it & 1;
                    if (!tc::mbar_wait(&sm.w_ready[s], ph)) { tc_fail(sm, err, kTcErrMma); stop = true; break; }
                    if (!tc::mbar_wait(&sm.x_ready[s], ph)) { tc_fail(sm, err, kTcErrMma); stop = true; break; }
                    if (!tc::mbar_wait(&sm.acc_free[b], ((it >> 1) & 1) ^ 1)) { tc_fail(sm, err, kTcErrMma); stop = true; break; }
                    if (tc_aborted(sm)) { stop = true; break; }
                    tc::tc_fence_after();
                    const uint32_t d = tmem + kTcAccCols * b;
                    // k-step kk of a tile is its descriptor plus kk * step in
                    // the start-address field (bits 0-13, address >> 4; shared
                    // addresses stay below 2^18, so the field never carries)
                    const uint64_t wh = tc_desc<B_MN>(sm.w_hi[s], 0), wl = tc_desc<B_MN>(sm.w_lo[s], 0);
                    const uint64_t xh = tc_desc<A_MN>(sm.x_hi[s], 0), xl = tc_desc<A_MN>(sm.x_lo[s], 0);
                    constexpr uint64_t ws = (B_MN ? 1024 : 32) >> 4, xs = (A_MN ? 1024 : 32) >> 4;
                    // hi*lo and lo*hi first, then hi*hi
#pragma unroll
                    for (int k = 0; k < kTcBK / 8; ++k) {
                        tc::mma_tf32_pair(d, wh + k * ws, xl + k * xs, idesc, k > 0 ? 1u : 0u);
                        tc::mma_tf32_pair(d, wl + k * ws, xh + k * xs, idesc, 1u);
                    }
#pragma unroll
                    for (int k = 0; k < kTcBK / 8; ++k) tc::mma_tf32_pair(d, wh + k * ws, xh + k * xs, idesc, 1u);
                    tc::mma_commit_pair(&sm.w_empty[s], 0x3);
                    tc::mma_commit_pair(&sm.x_empty[s], 0x3);
                    tc::mma_commit_pair(&sm.acc_ready[b], 0x3);
                }
            }
            // drain: every MMA issued above has completed before teardown
            tc::mma_commit_pair(&sm.drain, 0x1);
            tc::mbar_wait(&sm.drain, 0);
        }
    } else if (warp < kTcFirstDrainWarp) {
        // ---------------- converters ----------------
        const int ct = threadIdx.x - 64;  // 0..kTcConvThreads-1
        uint32_t it = 0;
        bool stop = false;
        for (int u = pair; u < g.units && !stop; u += npairs) {
            const TcUnit t = tc_unit(g, u);
            for (int kb = 0; kb < t.nk; ++kb, ++it) {
                const int s = it % kTcStages;
                const uint32_t ph = (it / kTcStages) & 1;
                // W stage: split in place unless B came pre-split; then
                // report it to the pair's MMA
                if (!tc::mbar_wait(&sm.w_full[s], ph)) { tc_fail(sm, err, kTcErrConverter); stop = true; break; }
                if (tc_aborted(sm)) { stop = true; break; }
                if (!B_SPLIT) {
                    tc_split_tile(sm.w_hi[s], sm.w_hi[s], sm.w_lo[s], ct);
                    tc::fence_proxy_async_smem();
                }
                __syncwarp();
                if (lane == 0) tc::mbar_arrive_cluster(tc::cluster_addr(&sm.w_ready[s], 0));
                // X stage: split in place, then report it
                if (!tc::mbar_wait(&sm.x_full[s], ph)) { tc_fail(sm, err, kTcErrConverter); stop = true; break; }
                if (tc_aborted(sm)) { stop = true; break; }
                tc_split_tile(sm.x_hi[s], sm.x_hi[s], sm.x_lo[s], ct);
                tc::fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) tc::mbar_arrive_cluster(tc::cluster_addr(&sm.x_ready[s], 0));
            }
        }
    } else {
        // ---------------- drain, then epilogue ----------------
        tc::setmaxnreg_inc<kTcRegsDrain>();
        const int dw = warp - kTcFirstDrainWarp;  // 0..15
        const int q = warp & 3;                   // TMEM lane quarter this warp may access
        const int slice = dw >> 2;                // which 64 of the 256 accumulator columns
        const uint32_t base = tmem + (uint32_t(32 * q) << 16) + uint32_t(64 * slice);
        uint32_t it = 0;
        bool stop = false;
        for (int u = pair; u < g.units && !stop; u += npairs) {
            const TcUnit t = tc_unit(g, u);
            if constexpr (C_TMA && Epi::kReads) {
                // the tile's epilogue inputs into L2 now, read after the k-loop:
                // lane l fetches the 128-byte lines of rows l and l + 32
                const int pc = t.n0 + kTcHalf * (int)rank + 32 * q;
                if (!partial && pc < g.N) {
#pragma unroll
                    for (int i = 0; i < 2; ++i) {
                        const int row = t.m0 + 64 * slice + 32 * i + lane;
                        if (row < g.M) tc::prefetch_l2(epi.pre_addr(row, pc));
                    }
                }
            }
            float acc[64];
#pragma unroll
            for (int i = 0; i < 64; ++i) acc[i] = 0.f;
            for (int kb = 0; kb < t.nk; ++kb, ++it) {
                const int b = it & 1;
                if (!tc::mbar_wait(&sm.acc_ready[b], (it >> 1) & 1)) { tc_fail(sm, err, kTcErrEpilogue); stop = true; break; }
                if (tc_aborted(sm)) { stop = true; break; }
                tc::tc_fence_after();
                // 16 columns at a time (registers: 64 sums + 16 loaded); the
                // buffer is released once the last piece is in registers
#pragma unroll
                for (int p = 0; p < 4; ++p) {
                    uint32_t v[16];
                    tc::tmem_ld_32x32b_x16(base + kTcAccCols * b + 16 * p, v);
                    tc::tmem_ld_wait();
                    if (p == 3) {
                        tc::tc_fence_before();
                        __syncwarp();
                        if (lane == 0) tc::mbar_arrive_cluster(tc::cluster_addr(&sm.acc_free[b], 0));
                    }
#pragma unroll
                    for (int i = 0; i < 16; ++i) acc[16 * p + i] = __fadd_rn(acc[16 * p + i], __uint_as_float(v[i]));
                }
            }
            if (stop || tc_aborted(sm)) break;
            const int n = t.n0 + kTcHalf * (int)rank + 32 * q + lane;
            const int row0 = t.m0 + 64 * slice;
            if constexpr (C_TMA) {
                // TMA-store epilogue: per 16-row chunk, lane = column writes
                // its 16 values into the warp's staging block (row-major
                // 16 x 32, conflict-free) and lane 0 hands the block to one
                // bulk tensor store (split-K partials go to [split][M][N]
                // through a 3-D map); rows and columns outside the output
                // are clipped by TMA.
                float* buf = sm.stage[dw];
                const int col0 = t.n0 + kTcHalf * (int)rank + 32 * q;
                // the epilogue's global inputs, eight rows at a time, one
                // group ahead of the rows being staged, so that their load
                // latency overlaps the staging and the store-buffer wait
                constexpr int kGroups = 64 / 8;
                float pre_cur[8], pre_nxt[8] = {};
                auto load_group = [&](int grp8, float (&p)[8]) {
#pragma unroll
                    for (int j = 0; j < 8; ++j) p[j] = 0.f;
                    if constexpr (Epi::kReads) {
                        if (!partial && n < g.N) {
#pragma unroll
                            for (int j = 0; j < 8; ++j)
                                if (row0 + 8 * grp8 + j < g.M) p[j] = epi.prefetch(row0 + 8 * grp8 + j, n);
                        }
                    }
                };
                load_group(0, pre_cur);
#pragma unroll
                for (int c = 0; c < 64 / kTcStoreRows; ++c) {
                    const int r0 = row0 + kTcStoreRows * c;
#pragma unroll
                    for (int hh = 0; hh < kTcStoreRows / 8; ++hh) {
                        const int grp8 = (kTcStoreRows / 8) * c + hh;
                        if (grp8 + 1 < kGroups) load_group(grp8 + 1, pre_nxt);
                        if (hh == 0) {
                            if (lane == 0) tc::bulk_wait_read<0>();  // the last store has read the block
                            __syncwarp();
                        }
#pragma unroll
                        for (int j = 0; j < 8; ++j) {
                            const float v = acc[kTcStoreRows * c + 8 * hh + j];
                            buf[(8 * hh + j) * 32 + lane] = partial ? v : epi.value(v, pre_cur[j]);
                        }
#pragma unroll
                        for (int j = 0; j < 8; ++j) pre_cur[j] = pre_nxt[j];
                    }
                    tc::fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0 && col0 < g.N && r0 < g.M) {
                        if (partial) tc::tma_store_3d(&map_c, buf, col0, r0, t.z);
                        else tc::tma_store_2d(&map_c, buf, col0, r0);
                        tc::bulk_commit();
                    }
                }
            } else if (n < g.N) {
                // direct epilogue: each access is a 128-byte row segment
                // across the warp
                if (partial) {
                    float* pz = partial + ((long)t.z * g.M) * g.N + n;
#pragma unroll
                    for (int i = 0; i < 64; ++i)
                        if (row0 + i < g.M) pz[(long)(row0 + i) * g.N] = acc[i];
                } else {
#pragma unroll
                    for (int c = 0; c < 8; ++c) {
                        // the chunk's global epilogue inputs, all loads in flight together
                        float pre[8];
#pragma unroll
                        for (int j = 0; j < 8; ++j) {
                            const int row = row0 + 8 * c + j;
                            pre[j] = (Epi::kReads && row < g.M) ? epi.prefetch(row, n) : 0.f;
                        }
#pragma unroll
                        for (int j = 0; j < 8; ++j) {
                            const int row = row0 + 8 * c + j;
                            if (row < g.M) epi.finish(row, n, acc[8 * c + j], pre[j]);
                        }
                    }
                }
            }
        }
        if (C_TMA && lane == 0) tc::bulk_wait_all();  // stores complete before the CTA exits
    }
    // Neither CTA leaves while the pair's MMAs may still touch its shared
    // memory or TMEM, or the other CTA may still arrive on its barriers.
    tc::tc_fence_before();
    __syncthreads();
    tc::cluster_sync();
    if (warp == 1) {
        tc::tc_fence_after();
        tc::tmem_dealloc_pair(tmem, kTcTmemCols);
    }
    tc::cluster_sync();
}

// Work split for an M x N x K problem over `pairs` CTA pairs.  With fewer
// output tiles than pairs and a long K (each split at least 256 deep), K is
// split so as to minimise the busiest pair's work: rounds of units per pair
// times k-blocks per unit, plus the split-K reduction's extra reads of
// splits x M x N floats (about 1.8 M floats per k-block time of a pair).  A
// larger split count is taken only when it saves more than 1%.
// `max_splits` = 1 forbids splitting.
inline TcGrid tc_grid(int M, int N, int K, int pairs, int max_splits) {
    TcGrid g{};
    g.M = M; g.N = N; g.K = K;
    g.tiles_m = (M + kTcBM - 1) / kTcBM;
    g.tiles_n = (N + kTcBN - 1) / kTcBN;
    const long tiles = (long)g.tiles_m * g.tiles_n;
    auto chunk_for = [&](int splits) {
        const int chunk = (K + splits - 1) / splits;
        return std::max(kTcBK, ((chunk + kTcBK - 1) / kTcBK) * kTcBK);
    };
    int splits = 1;
    if (max_splits > 1 && tiles < pairs && K >= 2 * 256) {
        double best = 0.0;
        const int smax = std::max(1, std::min(max_splits, K / 256));
        for (int s = 1; s <= smax; ++s) {
            const int chunk = chunk_for(s);
            const long units = tiles * ((K + chunk - 1) / chunk);
            const double rounds = double((units + pairs - 1) / pairs);
            const double cost = rounds * (chunk / kTcBK) + (s > 1 ? double(s) * M * N / 1.8e6 : 0.0);
            if (s == 1 || cost < 0.99 * best) {
                best = cost;
                splits = s;
            }
        }
    }
    const int chunk = chunk_for(splits);
    g.splits = std::max(1, (K + chunk - 1) / chunk);
    g.k_chunk = chunk;
    g.units = (int)(tiles * g.splits);
    return g;
}

inline cudaLaunchConfig_t tc_launch_config(int pairs, cudaStream_t stream, cudaLaunchAttribute* attr) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * std::max(1, pairs));
    cfg.blockDim = dim3(kTcThreads);
    cfg.dynamicSmemBytes = kTcSmemBytes;
    cfg.stream = stream;
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cfg;
}

// CTA pairs of this kernel that can be resident at once: one CTA per SM (its
// shared memory), two SMs per pair; queried once per instantiation.
template <bool A_MN, bool B_MN, bool B_SPLIT, bool C_TMA, class Epi>
inline int tc_pairs(int sm_count) {
    static int pairs = 0;
    if (pairs == 0) {
        auto kern = gemm_tc_kernel<A_MN, B_MN, B_SPLIT, C_TMA, Epi>;
        cudaLaunchAttribute attr[2];
        const cudaLaunchConfig_t cfg = tc_launch_config(sm_count / 2, nullptr, attr);
        int n = 0;
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kTcSmemBytes) == cudaSuccess &&
            cudaOccupancyMaxActiveClusters(&n, kern, &cfg) == cudaSuccess && n > 0)
            pairs = n;
        else
            pairs = std::max(1, sm_count / 2);
        (void)cudaGetLastError();
    }
    return pairs;
}

// Launches the persistent kernel as min(units, pairs) clusters of two CTAs.
// mx maps op(A) (K-major [M][K]: box 32 x kTcHalf, 128B swizzle; MN-major
// [K][M]: box 32 x 32, 128B swizzle with 32-byte atoms), mw op(B) likewise.
// With B_SPLIT, B arrives as two tensors, hi (already rounded to TF32)
// through mw and lo = B - hi through mw_lo, and is not split on the device.
// With `partial`, unit z of the K split writes its sums to partial[z][M][N]
// instead of applying the epilogue.  With C_TMA the epilogue writes through
// mc: the output [M][N] (or, with `partial`, [split][M][N] as a 3-D map),
// box 32 columns x kTcStoreRows rows, no swizzle.
template <bool A_MN, bool B_MN, bool B_SPLIT = false, bool C_TMA = false, class Epi>
inline cudaError_t launch_tc_kernel(cudaStream_t stream, int pairs, const CUtensorMap& mx, const CUtensorMap& mw,
                                    const CUtensorMap& mw_lo, const CUtensorMap& mc, const TcGrid& g, Epi epi,
                                    float* partial, int* err)
{
    auto kern = gemm_tc_kernel<A_MN, B_MN, B_SPLIT, C_TMA, Epi>;
    const cudaError_t a = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kTcSmemBytes);
    if (a != cudaSuccess) return a;
    // the warpgroups' register split must fit what the CTA is launched with
    static int regs = 0;
    if (regs == 0) {
        cudaFuncAttributes fa{};
        const cudaError_t r = cudaFuncGetAttributes(&fa, kern);
        if (r != cudaSuccess) return r;
        regs = fa.numRegs;
    }
    if (regs != kTcRegsLaunch) return cudaErrorInvalidConfiguration;
    cudaLaunchAttribute attr[2];
    const cudaLaunchConfig_t cfg = tc_launch_config(std::min(g.units, pairs), stream, attr);
    return cudaLaunchKernelEx(&cfg, kern, mx, mw, mw_lo, mc, g, epi, partial, err);
}

}  // namespace hx
