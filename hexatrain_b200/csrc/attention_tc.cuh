// attention_tc.cuh -- causal multi-head attention on the 5th-generation
// tensor cores for head dimension 32 and sequences of at most 256 tokens.
//
// Products run in "3xTF32" (hi*hi + hi*lo + lo*hi with hi = the nearest TF32
// value, lo = x - hi; see gemm_tc.cuh), so they carry FP32 accuracy; the
// softmax runs on the CUDA cores in FP32 with the row sum in double.
//
// Forward (tiny_language_model_cpu.cpp:44-45: scores, causal softmax,
// context), one CTA per (head, sequence), query rows in tiles of 128:
//   warps 16-19    lane 0 of each issues MMAs, one issuing warp per warp
//                  scheduler: warp 16 + r issues the E V products of the
//                  chunks c = r mod 4, warps 16 and 17 the two S column
//                  halves, and warp 16 first the TMA loads: Q, K, V rows
//                  [128t, 128t+128) of this head for each tile t, Q/K in the
//                  128-byte swizzle (K-major operands), V in the
//                  128-byte/32-byte-atom swizzle (MN-major B).
//   warps 0-15     split each landed tile into hi (in place) and lo (tile
//                  1 after tile 0's pass 2); the softmax of tile t, one
//                  TMEM lane (query row) per
//                  four threads: warp w reads lanes 32(w%4).. and the
//                  32-key chunks c = w/4, w/4 + 4, ...
// Per tile t (N = 128(t+1) keys):
//   S  = Q_t K[0:N]^T          into TMEM columns [0, N), as two column halves
//        of 12 MMAs M128 N(N/2) K8 each, issued interleaved
//   m  = max_j<=r S[r][j] * scale        (pass 1 over the chunks)
//   e  = exp(S * scale - m) (0 where j > r), sum = sum_j e   (pass 2),
//        as 2^(S * scale * log2 e - m * log2 e) with the hardware ex2
//        e is split into hi (written back over S) and lo (a 4-slot ring of
//        32-column TMEM chunks); each finished chunk is handed to the MMA
//        issuer, which computes E_c V_c into a fresh 32-column accumulator
//        with A read from TMEM (3 MMAs M128 N32 K8 per 8 keys), two chunks
//        at a time with their MMAs interleaved, and frees the slots.
//        Chunks 0-3 accumulate in four dedicated slots, chunk c >= 4 over
//        the S columns of chunk c - 4 once that chunk's MMAs are done, so no
//        MMA waits for the softmax threads to drain and the issuer never
//        waits for the pair just issued.  When
//        the tile's MMAs have completed, every softmax thread adds the
//        chunks' accumulators, in chunk order, into FP32 registers with
//        round-to-nearest adds.
//   ctx[r] = (E V)[r] / sum;  row max m and float(sum) are saved for the
//        backward.
// Accuracy: the MMA's FP32 accumulation truncates, so no accumulator runs
// longer than one 32-deep chunk, and within a chunk the small hi*lo and
// lo*hi terms are issued before hi*hi: only four full-magnitude truncations
// per chunk.  ctx matches an FP64 evaluation to a few 1e-7 of the row max.
// TMEM: S [0,256) (later chunk accumulators), chunk 0-3 accumulators
// [256,384), ring [384,512).
// Every mbarrier wait is bounded; after the first timeout the CTA records an
// error code, stops waiting (later waits return at once), keeps the same
// control flow through its named barriers, drains its MMAs and loads and
// frees TMEM.
#pragma once

#include "pdl.cuh"

#include "gemm_tc.cuh"

namespace hx {

constexpr int kAtcDH = 32, kAtcMaxT = 256, kAtcTile = 128;
constexpr int kAtcSoftWarps = 16, kAtcGroups = 4;  // warps w, w+4, w+8, w+12 share lane quadrant w%4
constexpr int kAtcSoftThreads = 32 * kAtcSoftWarps;
constexpr int kAtcThreads = kAtcSoftThreads + 32;
constexpr int kAtcRing = 4;
constexpr uint32_t kAtcCols = 512, kAtcColS = 0, kAtcColO = 256, kAtcColRing = 384;
// The forward runs four MMA-issuing warps beside the softmax warps, one per
// warp scheduler: issuer r issues the E V products of the chunks c = r mod 4;
// issuers 0 and 1 also issue the two S column halves, and issuer 0 the loads.
constexpr int kAtcFwdIssuers = 4;
constexpr int kAtcFwdThreads = kAtcSoftThreads + 32 * kAtcFwdIssuers;
constexpr int kAtcTileFloats = kAtcTile * kAtcDH;  // 128 rows x 32 fp32 = 16 KB
constexpr float kAtcLog2e = 1.4426950408889634f;

struct AtcFwdSmem {
    float qh[2 * kAtcTileFloats], ql[2 * kAtcTileFloats];
    float kh[2 * kAtcTileFloats], kl[2 * kAtcTileFloats];
    float vh[2 * kAtcTileFloats], vl[2 * kAtcTileFloats];
    float red_max[kAtcGroups][kAtcTile];
    double red_sum[kAtcGroups][kAtcTile];
    uint64_t ld[2], conv[2], pv_done[2], s_ready, ring_full[kAtcRing], ring_empty[kAtcRing];
    uint64_t pv_chunk[4], drained, drain;
    uint32_t tmem_addr;
    int abort;
};
constexpr size_t kAtcFwdSmemBytes = sizeof(AtcFwdSmem) + 1024;  // + alignment slack
static_assert(kAtcFwdSmemBytes <= 232448, "attention forward shared memory exceeds the 227 KB per-CTA limit");

enum AtcError { kAtcErrLoad = 11, kAtcErrMma = 12, kAtcErrSoftmax = 13, kAtcErrEpilogue = 14 };

// L2 prefetch of the 128-byte lines at column `col` of rows [r0, r1) of a
// row-major tensor with leading dimension ld (one head's 32 floats per row),
// spread over threads tid = 0 .. nthreads-1.
__device__ __forceinline__ void atc_prefetch_rows(const float* base, long ld, int col, int r0, int r1, int tid,
                                                  int nthreads) {
    for (int r = r0 + tid; r < r1; r += nthreads) tc::prefetch_l2(base + (long)r * ld + col);
}
// The CTA that starts on an SM one wave after this one (linear block id +
// the number of SMs; one CTA per SM), or -1 past the grid.
__device__ __forceinline__ int atc_next_wave_block() {
    uint32_t nsm;
    asm("mov.u32 %0, %%nsmid;" : "=r"(nsm));
    const long id = blockIdx.x + (long)gridDim.x * (blockIdx.y + (long)gridDim.y * blockIdx.z) + nsm;
    return id < (long)gridDim.x * gridDim.y * gridDim.z ? int(id) : -1;
}

// TMEM address of the E_c V_c accumulator of a tile's chunk c: chunks 0-3
// in the four dedicated 32-column slots, chunk c >= 4 over the S columns of
// chunk c - 4, whose MMAs have completed by then.
__device__ __forceinline__ uint32_t atc_fwd_acc(uint32_t base, int c) {
    return base + (c < 4 ? kAtcColO + 32u * c : kAtcColS + 32u * (c - 4));
}

// NC independent products D_j (M128 x N32) = A_j B_j over K = 32: A_j in TMEM
// (hi at a_hi[j], lo at a_lo[j]), B_j the 32 K-rows of an MN-major tile
// (hi/lo at b_hi[j]/b_lo[j], 128-byte rows, 8 K-rows = 1024 bytes).  Each
// accumulator gets the 3xTF32 terms in the same order (hi*lo and lo*hi per
// k-step, then hi*hi); the chains are interleaved MMA by MMA.
template <int NC>
__device__ __forceinline__ void atc_mma_chunks_mn(const uint32_t (&d)[NC], const uint32_t (&a_hi)[NC],
                                                  const uint32_t (&a_lo)[NC], const uint32_t (&b_hi)[NC],
                                                  const uint32_t (&b_lo)[NC]) {
    constexpr uint32_t idesc = tc::idesc_tf32(kAtcTile, kAtcDH, false, true);
    // descriptors built once; k-step k adds k * 1024 bytes to the start
    // address field (address >> 4; shared addresses stay below 2^18, so the
    // 14-bit field never carries), which keeps the issuing thread's work per
    // MMA to a few instructions
    uint64_t bh[NC], bl[NC];
#pragma unroll
    for (int j = 0; j < NC; ++j) {
        bh[j] = tc::smem_desc(b_hi[j], 4096, 512, tc::kLayoutSw128Base32);
        bl[j] = tc::smem_desc(b_lo[j], 4096, 512, tc::kLayoutSw128Base32);
    }
#pragma unroll
    for (int k = 0; k < 4; ++k)
#pragma unroll
        for (int j = 0; j < NC; ++j) {
            tc::mma_tf32_ts(d[j], a_hi[j] + 8 * k, bl[j] + 64 * k, idesc, k > 0 ? 1u : 0u);
            tc::mma_tf32_ts(d[j], a_lo[j] + 8 * k, bh[j] + 64 * k, idesc, 1u);
        }
#pragma unroll
    for (int k = 0; k < 4; ++k)
#pragma unroll
        for (int j = 0; j < NC; ++j) tc::mma_tf32_ts(d[j], a_hi[j] + 8 * k, bh[j] + 64 * k, idesc, 1u);
}

// Bounded wait; after the first failure anywhere in the CTA it returns
// false at once, so a broken CTA finishes in bounded time.
__device__ __forceinline__ bool atc_wait(int& abort, int* err, int code, uint64_t* bar, uint32_t parity) {
    volatile int* ab = &abort;
    if (*ab) return false;
    if (tc::mbar_wait(bar, parity)) return true;
    if (err) atomicCAS(err, 0, code);
    *ab = 1;
    return false;
}

// Barrier among the softmax threads only (the issuer warp never joins).
__device__ __forceinline__ void atc_soft_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kAtcSoftThreads) : "memory"); }

// hi = nearest TF32 (in place), lo = x - hi, for n4 float4s.
__device__ __forceinline__ void atc_split(float* hi, float* lo, int n4, int t, int nt) {
    float4* h4 = reinterpret_cast<float4*>(hi);
    float4* l4 = reinterpret_cast<float4*>(lo);
    for (int i = t; i < n4; i += nt) {
        const float4 x = h4[i];
        const float4 h = tf32_hi(x);
        h4[i] = h;
        l4[i] = make_float4(x.x - h.x, x.y - h.y, x.z - h.z, x.w - h.w);
    }
}

__global__ void __launch_bounds__(kAtcFwdThreads, 1)
attention_fwd_tc_kernel(const __grid_constant__ CUtensorMap map_qk, const __grid_constant__ CUtensorMap map_v, int T,
                        int D, int H, float scale, const float* __restrict__ qkv, float* __restrict__ ctx,
                        float* __restrict__ row_max, float* __restrict__ row_sum, int* __restrict__ err)
{
    HX_PDL_PROLOGUE();
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    const uint32_t pad = (1024u - (tc::smem_u32(smem_raw) & 1023u)) & 1023u;
    AtcFwdSmem& sm = *reinterpret_cast<AtcFwdSmem*>(smem_raw + pad);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int h = blockIdx.x, b = blockIdx.y;
    const int ntile = T > kAtcTile ? 2 : 1;
    const int y0 = b * T;

    if (threadIdx.x == 0) {
        for (int i = 0; i < 2; ++i) {
            tc::mbar_init(&sm.ld[i], 1);
            tc::mbar_init(&sm.conv[i], kAtcSoftThreads);
            tc::mbar_init(&sm.pv_done[i], kAtcFwdIssuers);  // every issuer commits
        }
        tc::mbar_init(&sm.s_ready, 2);  // the two issuers of the S halves
        for (int i = 0; i < 4; ++i) tc::mbar_init(&sm.pv_chunk[i], 1);
        for (int i = 0; i < kAtcRing; ++i) {
            tc::mbar_init(&sm.ring_full[i], 4);  // the four warps that own a chunk's 128 lanes
            tc::mbar_init(&sm.ring_empty[i], 1);
        }
        tc::mbar_init(&sm.drained, kAtcSoftWarps);
        tc::mbar_init(&sm.drain, kAtcFwdIssuers);
        sm.abort = 0;
        tc::fence_mbar_init();
    }
    if (warp == kAtcSoftWarps) {
        tc::tmem_alloc(&sm.tmem_addr, kAtcCols);
        tc::tmem_relinquish();
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = sm.tmem_addr;
    if (warp < kAtcSoftWarps) {
        // the next wave's CTA finds its Q, K and V rows in L2
        const int nb = atc_next_wave_block();
        if (nb >= 0) {
            const int nh = nb % H, ny = (nb / H) * T;
            for (int part = 0; part < 3; ++part)
                atc_prefetch_rows(qkv, 3L * D, part * D + nh * kAtcDH, ny, ny + T, threadIdx.x, kAtcSoftThreads);
        }
    }

    if (warp >= kAtcSoftWarps) {
        // role r < 2: S column half r (role 0 also the loads); every role:
        // the chunks c = r mod 4.  Chunk g's ring slot (g % 4) and
        // accumulator barrier (g & 3) equal its role, so each belongs to one
        // issuer; pv_done and drain count every issuer's commit, s_ready the
        // two S issuers'.  Every accumulator gets its MMAs in the
        // single-issuer order.
        const int role = warp - kAtcSoftWarps;
        if (lane == 0) {
            if (role == 0) {
                // ---------------- loads ----------------
                tc::prefetch_tensormap(&map_qk);
                tc::prefetch_tensormap(&map_v);
                for (int t = 0; t < ntile; ++t) {
                    tc::mbar_arrive_expect_tx(&sm.ld[t], 3 * kAtcTileFloats * 4);
                    const int y = y0 + kAtcTile * t;
                    tc::tma_load_2d(sm.qh + t * kAtcTileFloats, &map_qk, &sm.ld[t], h * kAtcDH, y);
                    tc::tma_load_2d(sm.kh + t * kAtcTileFloats, &map_qk, &sm.ld[t], D + h * kAtcDH, y);
                    tc::tma_load_2d(sm.vh + t * kAtcTileFloats, &map_v, &sm.ld[t], 2 * D + h * kAtcDH, y);
                }
            }
            // ---------------- MMA issuer ----------------
            const uint32_t qh = tc::smem_u32(sm.qh), ql = tc::smem_u32(sm.ql);
            const uint32_t kh = tc::smem_u32(sm.kh), kl = tc::smem_u32(sm.kl);
            const uint32_t vh = tc::smem_u32(sm.vh), vl = tc::smem_u32(sm.vl);
            uint32_t gch = 0;  // chunks handed over so far (ring position)
            for (int t = 0; t < ntile; ++t) {
                atc_wait(sm.abort, err, kAtcErrMma, &sm.conv[t], 0);
                if (t > 0) {
                    // S columns free again: no MMA reads them and every
                    // accumulator of the previous tile has been drained
                    atc_wait(sm.abort, err, kAtcErrMma, &sm.pv_done[t - 1], 0);
                    atc_wait(sm.abort, err, kAtcErrMma, &sm.drained, 0);
                }
                tc::tc_fence_after();
                // this role's half of the key columns (nh keys; B rows are
                // 128 bytes); corrections (hi*lo, lo*hi) first, then hi*hi;
                // descriptors built once, k-step k at + 32 k bytes (+ 2 k in
                // the start address field)
                const uint32_t nh = kAtcTile * (t + 1) / 2;
                const uint32_t idesc_s = tc::idesc_tf32(kAtcTile, nh, false, false);
                const uint32_t qo = uint32_t(t) * kAtcTileFloats * 4;
                if (role < 2) {
                    const uint64_t ah = tc::smem_desc(qh + qo, 16, 1024, tc::kLayoutSw128);
                    const uint64_t al = tc::smem_desc(ql + qo, 16, 1024, tc::kLayoutSw128);
                    const uint64_t bh = tc::smem_desc(kh + uint32_t(role) * nh * 128, 16, 1024, tc::kLayoutSw128);
                    const uint64_t bl = tc::smem_desc(kl + uint32_t(role) * nh * 128, 16, 1024, tc::kLayoutSw128);
                    const uint32_t d = tmem + kAtcColS + uint32_t(role) * nh;
#pragma unroll
                    for (int k = 0; k < kAtcDH / 8; ++k) {
                        tc::mma_tf32(d, ah + 2 * k, bl + 2 * k, idesc_s, k > 0 ? 1u : 0u);
                        tc::mma_tf32(d, al + 2 * k, bh + 2 * k, idesc_s, 1u);
                    }
#pragma unroll
                    for (int k = 0; k < kAtcDH / 8; ++k) tc::mma_tf32(d, ah + 2 * k, bh + 2 * k, idesc_s, 1u);
                }
                if (role < 2) tc::mma_commit(&sm.s_ready);
                const int nch = 4 * (t + 1);
                // this role's chunks c = role, role + 4
                for (int c = role; c < nch; c += kAtcFwdIssuers) {
                    const uint32_t g = gch + c;
                    const uint32_t slot = g % kAtcRing;
                    atc_wait(sm.abort, err, kAtcErrMma, &sm.ring_full[slot], (g / kAtcRing) & 1);
                    // chunk g - 4's MMAs (this issuer's previous chunk) have
                    // completed, so the S columns that chunk c - 4 read are
                    // free for this result
                    if (g >= 4) atc_wait(sm.abort, err, kAtcErrMma, &sm.pv_chunk[g & 3], ((g >> 2) & 1) ^ 1);
                    const uint32_t d[1] = {atc_fwd_acc(tmem, c)};
                    const uint32_t ahi[1] = {tmem + kAtcColS + 32 * c};
                    const uint32_t alo[1] = {tmem + kAtcColRing + 32 * slot};
                    const uint32_t bhi[1] = {vh + 32 * c * 128};  // V rows are 128-byte K-rows
                    const uint32_t blo[1] = {vl + 32 * c * 128};
                    tc::tc_fence_after();
                    atc_mma_chunks_mn<1>(d, ahi, alo, bhi, blo);
                    tc::mma_commit(&sm.ring_empty[slot]);
                    tc::mma_commit(&sm.pv_chunk[g & 3]);
                }
                gch += nch;
                tc::mma_commit(&sm.pv_done[t]);
            }
            // every MMA above has completed, and every load has landed,
            // before TMEM is freed and the CTA exits
            tc::mma_commit(&sm.drain);
            tc::mbar_wait(&sm.drain, 0);
            if (role == 0)
                for (int t = 0; t < ntile; ++t) tc::mbar_wait(&sm.ld[t], 0);
        }
    } else {
        const int st = threadIdx.x;
        const int q = warp & 3, grp = warp >> 2;
        // ---------------- hi/lo split of a landed tile ----------------
        // tile 0 here; tile 1 after tile 0's pass 2, while the MMA issuers
        // runs tile 0's E V, so that it does not compete with the S MMAs of
        // tile 0 for shared memory
        auto split_tile = [&](int t) {
            atc_wait(sm.abort, err, kAtcErrLoad, &sm.ld[t], 0);
            const int o = t * kAtcTileFloats;
            atc_split(sm.qh + o, sm.ql + o, kAtcTileFloats / 4, st, kAtcSoftThreads);
            atc_split(sm.kh + o, sm.kl + o, kAtcTileFloats / 4, st, kAtcSoftThreads);
            atc_split(sm.vh + o, sm.vl + o, kAtcTileFloats / 4, st, kAtcSoftThreads);
            tc::fence_proxy_async_smem();
            tc::mbar_arrive(&sm.conv[t]);
        };
        split_tile(0);
        // ---------------- softmax and epilogue ----------------
        // e = 2^(s * scale * log2(e) - m * log2(e)): one FFMA and one ex2
        // per score; the per-row constant's rounding cancels in e / sum.
        const float c1 = scale * kAtcLog2e;
        const uint32_t lane_base = tmem + (uint32_t(32 * q) << 16);
        const int rl = 32 * q + lane;
        uint32_t gch = 0;
        for (int t = 0; t < ntile; ++t) {
            const int nch = 4 * (t + 1);
            const int r = kAtcTile * t + rl;
            const int lim = r < T ? r : -1;                   // last key visible to this row
            const int diag = 4 * t + q;                       // chunk on this warp's diagonal
            const bool rows_valid = kAtcTile * t + 32 * q + 31 < T;  // every row of the warp is < T
            atc_wait(sm.abort, err, kAtcErrSoftmax, &sm.s_ready, t & 1);
            tc::tc_fence_after();
            // pass 1: max of the raw scores (scale > 0 commutes with max)
            float mraw = -INFINITY;
            for (int c = grp; c <= diag; c += kAtcGroups) {
                uint32_t v[32];
                tc::tmem_ld_32x32b_x32(lane_base + kAtcColS + 32 * c, v);
                tc::tmem_ld_wait();
                if (c < diag && rows_valid) {
#pragma unroll
                    for (int i = 0; i < 32; ++i) mraw = fmaxf(mraw, __uint_as_float(v[i]));
                } else {
#pragma unroll
                    for (int i = 0; i < 32; ++i)
                        if (32 * c + i <= lim) mraw = fmaxf(mraw, __uint_as_float(v[i]));
                }
            }
            sm.red_max[grp][rl] = mraw;
            atc_soft_sync();
            mraw = fmaxf(fmaxf(sm.red_max[0][rl], sm.red_max[1][rl]), fmaxf(sm.red_max[2][rl], sm.red_max[3][rl]));
            const float m = __fmul_rn(mraw, scale);
            const float negml = __fmul_rn(m, -kAtcLog2e);
            double sum = 0.0;
            float oacc[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) oacc[i] = 0.f;
            // pass 2: e, its hi/lo split, the hand-over to the MMA issuers
            for (int c = grp; c < nch; c += kAtcGroups) {
                const uint32_t g = gch + c;
                const int slot = g % kAtcRing;
                atc_wait(sm.abort, err, kAtcErrSoftmax, &sm.ring_empty[slot], ((g / kAtcRing) & 1) ^ 1);
                tc::tc_fence_after();
                const bool full = c < diag && rows_valid;
#pragma unroll
                for (int half = 0; half < 2; ++half) {  // 16 columns at a time keeps 32 values live
                    const uint32_t col = 32 * c + 16 * half;
                    uint32_t eh[16], el[16];
                    if (c <= diag) {
                        tc::tmem_ld_32x32b_x16(lane_base + kAtcColS + col, eh);
                        tc::tmem_ld_wait();
                        // two scores per paired FP32 instruction; pp holds the
                        // even- and odd-column partial sums
                        float2 pp = make_float2(0.f, 0.f);
#pragma unroll
                        for (int i = 0; i < 16; i += 2) {
                            const float2 t = tc::fma2_rn(make_float2(__uint_as_float(eh[i]), __uint_as_float(eh[i + 1])),
                                                         make_float2(c1, c1), make_float2(negml, negml));
                            float e0 = tc::exp2_approx(t.x), e1 = tc::exp2_approx(t.y);
                            if (!full) {
                                if (int(col) + i > lim) e0 = 0.f;
                                if (int(col) + i + 1 > lim) e1 = 0.f;
                            }
                            pp = tc::add2_rn(pp, make_float2(e0, e1));
                            eh[i] = tc::tf32_rna_bits(e0);
                            eh[i + 1] = tc::tf32_rna_bits(e1);
                            const float2 l = tc::sub2_rn(make_float2(e0, e1),
                                                         make_float2(__uint_as_float(eh[i]), __uint_as_float(eh[i + 1])));
                            el[i] = __float_as_uint(l.x);
                            el[i + 1] = __float_as_uint(l.y);
                        }
                        sum += double(pp.x) + double(pp.y);
                    } else {
#pragma unroll
                        for (int i = 0; i < 16; ++i) { eh[i] = 0u; el[i] = 0u; }
                    }
                    tc::tmem_st_32x32b_x16(lane_base + kAtcColS + col, eh);
                    tc::tmem_st_32x32b_x16(lane_base + kAtcColRing + 32 * slot + 16 * half, el);
                }
                tc::tmem_st_wait();
                tc::tc_fence_before();
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(&sm.ring_full[slot]);
            }
            if (t + 1 < ntile) split_tile(t + 1);
            // every chunk's E_c V_c is in TMEM once the tile's MMAs have
            // completed: add them, in chunk order, into FP32 registers
            // (this thread's row, 8 columns) with round-to-nearest adds;
            // chunks past this warp's diagonal are zero in its rows
            atc_wait(sm.abort, err, kAtcErrEpilogue, &sm.pv_done[t], 0);
            tc::tc_fence_after();
            for (int c = 0; c <= diag && c < nch; ++c) {
                uint32_t o[8];
                tc::tmem_ld_32x32b_x8(atc_fwd_acc(lane_base, c) + 8 * grp, o);
                tc::tmem_ld_wait();
#pragma unroll
                for (int i = 0; i < 8; ++i) oacc[i] = __fadd_rn(oacc[i], __uint_as_float(o[i]));
            }
            tc::tc_fence_before();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&sm.drained);
            gch += nch;
            sm.red_sum[grp][rl] = sum;
            atc_soft_sync();
            const float sumf =
                float(((sm.red_sum[0][rl] + sm.red_sum[1][rl]) + sm.red_sum[2][rl]) + sm.red_sum[3][rl]);
            if (r < T) {
                float* dst = ctx + (long)(y0 + r) * D + h * kAtcDH + 8 * grp;
#pragma unroll
                for (int i = 0; i < 8; i += 4)
                    *reinterpret_cast<float4*>(dst + i) =
                        make_float4(__fdiv_rn(oacc[i], sumf), __fdiv_rn(oacc[i + 1], sumf),
                                    __fdiv_rn(oacc[i + 2], sumf), __fdiv_rn(oacc[i + 3], sumf));
                if (grp == 0) {
                    row_max[((long)b * H + h) * T + r] = m;
                    row_sum[((long)b * H + h) * T + r] = sumf;
                }
            }
        }
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == kAtcSoftWarps) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, kAtcCols);
    }
}

}  // namespace hx
