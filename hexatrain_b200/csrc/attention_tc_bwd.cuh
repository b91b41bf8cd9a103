// attention_tc_bwd.cuh -- causal attention backward on the tcgen05 tensor
// cores, head dimension 32, T <= 256 (tiny_language_model_cpu.cpp:79-81:
// dV = P^T dO, dP = dO V^T, D_r = sum_j P dP, dS = P (dP - D),
// dQ = scale dS K, dK = scale dS^T Q).
//
// Two kernels, both recomputing S and dP with the forward's 3xTF32 MMA
// sequence (hi*lo and lo*hi terms first, then hi*hi) and
// e = 2^(S * scale * log2 e - m * log2 e) from the saved row max m:
//
// attention_bwd_dq_tc_kernel   queries on TMEM lanes, one CTA per (head,
//   sequence).  K, V (K-major) and K (MN-major) for all 256 keys are split
//   into hi/lo in shared memory once; Q and dO of the 128-row query tile go
//   straight into TMEM as A operands.  Per query tile, two passes over its
//   128-key blocks:
//     A: S and dP into TMEM; sum_r = sum_j e, dot_r = sum_j e dP (double);
//        D_r = dot_r / sum_r.
//     B: the key blocks in reverse order, S and dP again except for the
//        first, which is pass A's last block still in TMEM;
//        P = e * (1 / sum_r), dS = P (dP - D_r); dS hi is
//        written over S and dS lo over dP, then each 32-key chunk gives
//        dQ_c = dS_c K_c (A from TMEM) into a fresh accumulator that every
//        thread drains into FP32 registers with round-to-nearest adds.
//   It stores dQ and the row statistics (sum_r, D_r) of its own P, so that
//   sum_j P = 1 and sum_j dS = 0 hold to rounding whatever the forward's
//   engine.
// attention_bwd_dkdv_tc_kernel keys on TMEM lanes, one CTA per (head,
//   sequence, 128-key block).  K and V of the block sit in shared memory
//   (K-major A operands); each 128-query block brings Q and dO in both
//   K-major (for S^T = K Q^T, dP^T = V dO^T) and MN-major (for the B
//   operands of dK and dV) layouts.  P^T and dS^T are formed from the
//   statistics the dQ kernel stored, hi written over S^T / dP^T, lo into a
//   2-slot ring; per 32-query chunk, dV_c = P^T_c dO_c and dK_c = dS^T_c Q_c
//   go into fresh accumulators (chunks 0 and 1 in two dedicated slots,
//   chunk c >= 2 over chunk c - 2's S^T / dP^T columns), which every
//   thread adds into FP32 registers once the block's MMAs have completed.
// Thread layout in both: 16 warps of four groups (warp w: TMEM lane quadrant
// w % 4, group w / 4 owns 32-column chunk w / 4 of each 128-column block;
// each thread drains 8 of the 32 output columns) plus four warps, one per
// warp scheduler, whose lane 0 issues MMAs (the split is given at each
// kernel); the first of them also issues the TMA loads.  Waits are bounded
// as in the forward.
#pragma once

#include "pdl.cuh"

#include "attention_tc.cuh"

namespace hx {

// ---- dQ kernel ---------------------------------------------------------------

constexpr uint32_t kDqColQ = 0, kDqColDo = 64, kDqColS = 128, kDqColDp = 256, kDqColAcc = 384;
// 16 softmax warps and four MMA-issuing warps, one per warp scheduler:
// issuer r issues the dQ products of chunk r; issuer 0 also the loads and S,
// issuer 1 dP
constexpr int kAtcDqIssuers = 4;
constexpr int kAtcDqThreads = kAtcSoftThreads + 32 * kAtcDqIssuers;

struct AtcDqSmem {
    float kh[2 * kAtcTileFloats], kl[2 * kAtcTileFloats];    // K, K-major
    float vh[2 * kAtcTileFloats], vl[2 * kAtcTileFloats];    // V, K-major
    float kmh[2 * kAtcTileFloats], kml[2 * kAtcTileFloats];  // K, MN-major
    double red[kAtcGroups][kAtcTile][2];                     // per-group (sum, dot)
    uint64_t ld, conv, a_ready, sd_ready, sd_free, dq_done, drain;
    uint64_t ds_full[4], acc_full[4], acc_empty[4];
    uint32_t tmem_addr;
    int abort;
};
constexpr size_t kAtcDqSmemBytes = sizeof(AtcDqSmem) + 1024;
static_assert(kAtcDqSmemBytes <= 232448, "attention dQ kernel shared memory exceeds the 227 KB per-CTA limit");

// Loads 8 consecutive floats (two float4) of a row, or zeros.
__device__ __forceinline__ void atc_row8(const float* p, bool ok, float (&v)[8]) {
    if (ok) {
        const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = 0.f;
    }
}
// Writes hi (nearest TF32) and lo = x - hi of 8 values into TMEM.
__device__ __forceinline__ void atc_st_split8(uint32_t hi_addr, uint32_t lo_addr, const float (&x)[8]) {
    uint32_t h[8], l[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float hv = tf32_round(x[i]);
        h[i] = __float_as_uint(hv);
        l[i] = __float_as_uint(x[i] - hv);
    }
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};"
                 ::"r"(hi_addr), "r"(h[0]), "r"(h[1]), "r"(h[2]), "r"(h[3]), "r"(h[4]), "r"(h[5]), "r"(h[6]), "r"(h[7])
                 : "memory");
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};"
                 ::"r"(lo_addr), "r"(l[0]), "r"(l[1]), "r"(l[2]), "r"(l[3]), "r"(l[4]), "r"(l[5]), "r"(l[6]), "r"(l[7])
                 : "memory");
}

// Issues D_j = A_j B_j^T over K = 32 for two independent products j = 0, 1
// in the forward's term order, their MMAs interleaved: A_j hi/lo in TMEM
// (columns a_col[j] .. +31 hi, a_col[j] + 32 .. lo), B_j hi/lo K-major in
// shared memory (b_hi/b_lo: the block's first row).
__device__ __forceinline__ void atc_mma_ts_kmajor2(const uint32_t (&d)[2], const uint32_t (&a_col)[2],
                                                   const uint32_t (&b_hi)[2], const uint32_t (&b_lo)[2],
                                                   uint32_t idesc) {
    // descriptors built once, k-step k at + 32 k bytes (+ 2 k in the start
    // address field)
    uint64_t bh[2], bl[2];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
        bh[j] = tc::smem_desc(b_hi[j], 16, 1024, tc::kLayoutSw128);
        bl[j] = tc::smem_desc(b_lo[j], 16, 1024, tc::kLayoutSw128);
    }
#pragma unroll
    for (int k = 0; k < kAtcDH / 8; ++k)
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            tc::mma_tf32_ts(d[j], a_col[j] + 8 * k, bl[j] + 2 * k, idesc, k > 0 ? 1u : 0u);
            tc::mma_tf32_ts(d[j], a_col[j] + 32 + 8 * k, bh[j] + 2 * k, idesc, 1u);
        }
#pragma unroll
    for (int k = 0; k < kAtcDH / 8; ++k)
#pragma unroll
        for (int j = 0; j < 2; ++j) tc::mma_tf32_ts(d[j], a_col[j] + 8 * k, bh[j] + 2 * k, idesc, 1u);
}

// The same for one product D = A B^T over K = 32 (A hi/lo in TMEM at a_col,
// B hi/lo K-major in shared memory), in the same term order.
__device__ __forceinline__ void atc_mma_ts_kmajor1(uint32_t d, uint32_t a_col, uint32_t b_hi, uint32_t b_lo,
                                                   uint32_t idesc) {
    const uint64_t bh = tc::smem_desc(b_hi, 16, 1024, tc::kLayoutSw128);
    const uint64_t bl = tc::smem_desc(b_lo, 16, 1024, tc::kLayoutSw128);
#pragma unroll
    for (int k = 0; k < kAtcDH / 8; ++k) {
        tc::mma_tf32_ts(d, a_col + 8 * k, bl + 2 * k, idesc, k > 0 ? 1u : 0u);
        tc::mma_tf32_ts(d, a_col + 32 + 8 * k, bh + 2 * k, idesc, 1u);
    }
#pragma unroll
    for (int k = 0; k < kAtcDH / 8; ++k) tc::mma_tf32_ts(d, a_col + 8 * k, bh + 2 * k, idesc, 1u);
}

// Visibility of a 32-key chunk (keys 128 kb + 32 c ..) to the 32 query rows
// 128 t + 32 q .. of a warp: 2 all visible, 1 diagonal, 0 none.
__device__ __forceinline__ int atc_chunk_vis(int t, int q, int kb, int c, bool rows_valid) {
    if (kb < t) return rows_valid ? 2 : 1;
    if (c < q) return rows_valid ? 2 : 1;
    return c == q ? 1 : 0;
}

__global__ void __launch_bounds__(kAtcDqThreads, 1)
attention_bwd_dq_tc_kernel(const __grid_constant__ CUtensorMap map_qk, const __grid_constant__ CUtensorMap map_mn, int T,
                           int D, int H, float scale, const float* __restrict__ qkv, const float* __restrict__ dctx,
                           const float* __restrict__ row_max, float* __restrict__ bstat, float* __restrict__ dqkv,
                           int* __restrict__ err)
{
    HX_PDL_PROLOGUE();
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    const uint32_t pad = (1024u - (tc::smem_u32(smem_raw) & 1023u)) & 1023u;
    AtcDqSmem& sm = *reinterpret_cast<AtcDqSmem*>(smem_raw + pad);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int h = blockIdx.x, b = blockIdx.y;
    const int ntile = T > kAtcTile ? 2 : 1;
    const int y0 = b * T;

    if (threadIdx.x == 0) {
        tc::mbar_init(&sm.ld, 1);
        tc::mbar_init(&sm.conv, kAtcSoftThreads);
        tc::mbar_init(&sm.a_ready, kAtcSoftWarps);
        // S and dP by issuers 0 and 1; dq_done and drain by every issuer
        tc::mbar_init(&sm.sd_ready, 2);
        tc::mbar_init(&sm.sd_free, kAtcSoftWarps);
        tc::mbar_init(&sm.dq_done, kAtcDqIssuers);
        tc::mbar_init(&sm.drain, kAtcDqIssuers);
        for (int i = 0; i < 4; ++i) {
            tc::mbar_init(&sm.ds_full[i], 4);
            tc::mbar_init(&sm.acc_full[i], 1);
            tc::mbar_init(&sm.acc_empty[i], kAtcSoftWarps);
        }
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
        // this CTA's Q and dO rows (read by the softmax threads after the
        // K/V split) and the next wave's K and V rows, into L2
        atc_prefetch_rows(qkv, 3L * D, h * kAtcDH, y0, y0 + T, threadIdx.x, kAtcSoftThreads);
        atc_prefetch_rows(dctx, D, h * kAtcDH, y0, y0 + T, threadIdx.x, kAtcSoftThreads);
        const int nb = atc_next_wave_block();
        if (nb >= 0) {
            const int nh = nb % H, ny = (nb / H) * T;
            for (int part = 1; part < 3; ++part)
                atc_prefetch_rows(qkv, 3L * D, part * D + nh * kAtcDH, ny, ny + T, threadIdx.x, kAtcSoftThreads);
        }
    }
    if (warp >= kAtcSoftWarps) {
        // Four issuers on the four warp schedulers: issuer r issues the dQ
        // products of chunk r, issuer 0 also the TMA loads and S, issuer 1
        // dP.  Each accumulator gets its MMAs in the single-issuer order, so
        // the results are the same bit for bit; sd_ready counts the S and dP
        // issuers' commits, dq_done and drain every issuer's.
        const int role = warp - kAtcSoftWarps;
        if (lane == 0) {
            if (role == 0) {
                // ---------------- loads: K, V (K-major) and K (MN-major), all rows
                tc::prefetch_tensormap(&map_qk);
                tc::prefetch_tensormap(&map_mn);
                tc::mbar_arrive_expect_tx(&sm.ld, 3 * ntile * kAtcTileFloats * 4);
                for (int t = 0; t < ntile; ++t) {
                    const int y = y0 + kAtcTile * t;
                    tc::tma_load_2d(sm.kh + t * kAtcTileFloats, &map_qk, &sm.ld, D + h * kAtcDH, y);
                    tc::tma_load_2d(sm.vh + t * kAtcTileFloats, &map_qk, &sm.ld, 2 * D + h * kAtcDH, y);
                    tc::tma_load_2d(sm.kmh + t * kAtcTileFloats, &map_mn, &sm.ld, D + h * kAtcDH, y);
                }
            }
            // ---------------- MMA issuer ----------------
            // this role's product: S = Q K^T (role 0) or dP = dO V^T (role 1)
            const uint32_t bh0 = tc::smem_u32(role == 1 ? sm.vh : sm.kh), bl0 = tc::smem_u32(role == 1 ? sm.vl : sm.kl);
            const uint32_t d_sd = tmem + (role == 1 ? kDqColDp : kDqColS);
            const uint32_t a_sd = tmem + (role == 1 ? kDqColDo : kDqColQ);
            const uint32_t kmh = tc::smem_u32(sm.kmh), kml = tc::smem_u32(sm.kml);
            const int c = role;  // this issuer's dQ chunk
            constexpr uint32_t idesc_s = tc::idesc_tf32(kAtcTile, kAtcTile, false, false);
            atc_wait(sm.abort, err, kAtcErrMma, &sm.conv, 0);
            uint32_t v = 0, u = 0;  // S/dP blocks issued, pass-B blocks issued
            bool dq_pending = false;
            for (int t = 0; t < ntile; ++t) {
                atc_wait(sm.abort, err, kAtcErrMma, &sm.a_ready, t & 1);
                for (int pass = 0; pass < 2; ++pass) {
                    for (int i = 0; i <= t; ++i) {
                        // pass B walks the key blocks backwards: its first
                        // block is pass A's last, whose S and dP are still in
                        // TMEM (pass A only reads them), so it is not recomputed
                        const int kb = pass ? t - i : i;
                        if (v > 0) atc_wait(sm.abort, err, kAtcErrMma, &sm.sd_free, (v - 1) & 1);
                        if (dq_pending) atc_wait(sm.abort, err, kAtcErrMma, &sm.dq_done, (u - 1) & 1);
                        dq_pending = false;
                        tc::tc_fence_after();
                        if (role < 2 && (pass == 0 || i > 0)) {
                            const uint32_t ko = uint32_t(kb) * kAtcTileFloats * 4;
                            atc_mma_ts_kmajor1(d_sd, a_sd, bh0 + ko, bl0 + ko, idesc_s);
                        }
                        if (role < 2) tc::mma_commit(&sm.sd_ready);
                        ++v;
                        if (pass == 0) continue;
                        // this issuer's chunk's dQ product
                        atc_wait(sm.abort, err, kAtcErrMma, &sm.ds_full[c], u & 1);
                        atc_wait(sm.abort, err, kAtcErrMma, &sm.acc_empty[c], (u & 1) ^ 1);
                        {
                            const uint32_t row = uint32_t(kAtcTile * kb + 32 * c) * 128;
                            const uint32_t d[1] = {tmem + kDqColAcc + 32 * c};
                            const uint32_t ahi[1] = {tmem + kDqColS + 32 * c};
                            const uint32_t alo[1] = {tmem + kDqColDp + 32 * c};
                            const uint32_t bhi[1] = {kmh + row}, blo[1] = {kml + row};
                            tc::tc_fence_after();
                            atc_mma_chunks_mn<1>(d, ahi, alo, bhi, blo);
                        }
                        tc::mma_commit(&sm.acc_full[c]);
                        tc::mma_commit(&sm.dq_done);
                        ++u;
                        dq_pending = true;
                    }
                }
            }
            tc::mma_commit(&sm.drain);
            tc::mbar_wait(&sm.drain, 0);
            if (role == 0) tc::mbar_wait(&sm.ld, 0);
        }
    } else {
        const int st = threadIdx.x;
        const int q = warp & 3, grp = warp >> 2;
        const uint32_t lane_base = tmem + (uint32_t(32 * q) << 16);
        const int rl = 32 * q + lane;
        const float c1 = scale * kAtcLog2e;
        const int ld3 = 3 * D;
        // this thread's Q and dO values of tile 0 (columns 8 grp .. +7),
        // loaded before the split so that their latency overlaps it
        float xq[8], xo[8];
        atc_row8(qkv + ((long)y0 + rl) * ld3 + h * kAtcDH + 8 * grp, rl < T, xq);
        atc_row8(dctx + ((long)y0 + rl) * D + h * kAtcDH + 8 * grp, rl < T, xo);
        // ---------------- hi/lo split of K, V, K_mn ----------------
        atc_wait(sm.abort, err, kAtcErrLoad, &sm.ld, 0);
        const int n4 = ntile * kAtcTileFloats / 4;
        atc_split(sm.kh, sm.kl, n4, st, kAtcSoftThreads);
        atc_split(sm.vh, sm.vl, n4, st, kAtcSoftThreads);
        atc_split(sm.kmh, sm.kml, n4, st, kAtcSoftThreads);
        tc::fence_proxy_async_smem();
        tc::mbar_arrive(&sm.conv);
        atc_st_split8(lane_base + kDqColQ + 8 * grp, lane_base + kDqColQ + 32 + 8 * grp, xq);
        atc_st_split8(lane_base + kDqColDo + 8 * grp, lane_base + kDqColDo + 32 + 8 * grp, xo);
        uint32_t v = 0, u = 0;
        for (int t = 0; t < ntile; ++t) {
            const int r = kAtcTile * t + rl;
            const bool valid = r < T;
            const bool rows_valid = kAtcTile * t + 32 * q + 31 < T;
            const long grow = (long)y0 + r;
            // ---- Q and dO of this row, columns 8 grp .. +7, into TMEM (tile
            // 0's went in after the split; both loads before the stores)
            {
                if (t > 0) {
                    float x[8], y[8];
                    atc_row8(qkv + grow * ld3 + h * kAtcDH + 8 * grp, valid, x);
                    atc_row8(dctx + grow * D + h * kAtcDH + 8 * grp, valid, y);
                    atc_st_split8(lane_base + kDqColQ + 8 * grp, lane_base + kDqColQ + 32 + 8 * grp, x);
                    atc_st_split8(lane_base + kDqColDo + 8 * grp, lane_base + kDqColDo + 32 + 8 * grp, y);
                }
                tc::tmem_st_wait();
                tc::tc_fence_before();
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(&sm.a_ready);
            }
            const float negml = valid ? __fmul_rn(row_max[((long)b * H + h) * T + r], -kAtcLog2e) : 0.f;
            const int lim = valid ? r : -1;
            // ---- pass A: sum_j e and sum_j e dP over this thread's chunks
            double sum = 0.0, dot = 0.0;
            for (int kb = 0; kb <= t; ++kb, ++v) {
                atc_wait(sm.abort, err, kAtcErrSoftmax, &sm.sd_ready, v & 1);
                tc::tc_fence_after();
                const int vis = atc_chunk_vis(t, q, kb, grp, rows_valid);
                if (vis) {
#pragma unroll
                    for (int half = 0; half < 2; ++half) {
                        const uint32_t col = 32 * grp + 16 * half;
                        const int key0 = kAtcTile * kb + col;
                        uint32_t sv[16], dv[16];
                        tc::tmem_ld_32x32b_x16(lane_base + kDqColS + col, sv);
                        tc::tmem_ld_32x32b_x16(lane_base + kDqColDp + col, dv);
                        tc::tmem_ld_wait();
                        float ps = 0.f, pd = 0.f;
#pragma unroll
                        for (int i = 0; i < 16; ++i) {
                            float e = tc::exp2_approx(fmaf(__uint_as_float(sv[i]), c1, negml));
                            if (vis == 1 && key0 + i > lim) e = 0.f;
                            ps += e;
                            pd = fmaf(e, __uint_as_float(dv[i]), pd);
                        }
                        sum += double(ps);
                        dot += double(pd);
                    }
                }
                tc::tc_fence_before();
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(&sm.sd_free);
            }
            sm.red[grp][rl][0] = sum;
            sm.red[grp][rl][1] = dot;
            atc_soft_sync();
            const double tsum = ((sm.red[0][rl][0] + sm.red[1][rl][0]) + sm.red[2][rl][0]) + sm.red[3][rl][0];
            const double tdot = ((sm.red[0][rl][1] + sm.red[1][rl][1]) + sm.red[2][rl][1]) + sm.red[3][rl][1];
            const float sumf = valid ? float(tsum) : 1.f;
            const float dr = valid ? float(tdot / tsum) : 0.f;
            const float inv = __frcp_rn(sumf);
            atc_soft_sync();  // every thread has read red before the next tile writes it
            // ---- pass B: dS, its hand-over, and the dQ drains
            float dq[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) dq[i] = 0.f;
            for (int i = 0; i <= t; ++i, ++v, ++u) {
                const int kb = t - i;  // the MMA issuers' pass-B order
                atc_wait(sm.abort, err, kAtcErrSoftmax, &sm.sd_ready, v & 1);
                tc::tc_fence_after();
                const int vis = atc_chunk_vis(t, q, kb, grp, rows_valid);
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    const uint32_t col = 32 * grp + 16 * half;
                    const int key0 = kAtcTile * kb + col;
                    uint32_t sv[16], dv[16];
                    if (vis) {
                        tc::tmem_ld_32x32b_x16(lane_base + kDqColS + col, sv);
                        tc::tmem_ld_32x32b_x16(lane_base + kDqColDp + col, dv);
                        tc::tmem_ld_wait();
#pragma unroll
                        for (int i = 0; i < 16; ++i) {
                            float e = tc::exp2_approx(fmaf(__uint_as_float(sv[i]), c1, negml));
                            if (vis == 1 && key0 + i > lim) e = 0.f;
                            const float ds = __fmul_rn(__fmul_rn(e, inv), __fsub_rn(__uint_as_float(dv[i]), dr));
                            sv[i] = tc::tf32_rna_bits(ds);
                            dv[i] = __float_as_uint(ds - __uint_as_float(sv[i]));
                        }
                    } else {
#pragma unroll
                        for (int i = 0; i < 16; ++i) { sv[i] = 0u; dv[i] = 0u; }
                    }
                    tc::tmem_st_32x32b_x16(lane_base + kDqColS + col, sv);
                    tc::tmem_st_32x32b_x16(lane_base + kDqColDp + col, dv);
                }
                tc::tmem_st_wait();
                tc::tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    tc::mbar_arrive(&sm.ds_full[grp]);
                    tc::mbar_arrive(&sm.sd_free);
                }
                for (int c = 0; c < 4; ++c) {
                    atc_wait(sm.abort, err, kAtcErrEpilogue, &sm.acc_full[c], u & 1);
                    tc::tc_fence_after();
                    if (atc_chunk_vis(t, q, kb, c, rows_valid)) {
                        uint32_t o[8];
                        tc::tmem_ld_32x32b_x8(lane_base + kDqColAcc + 32 * c + 8 * grp, o);
                        tc::tmem_ld_wait();
#pragma unroll
                        for (int i = 0; i < 8; ++i) dq[i] = __fadd_rn(dq[i], __uint_as_float(o[i]));
                    }
                    tc::tc_fence_before();
                    __syncwarp();
                    if (lane == 0) tc::mbar_arrive(&sm.acc_empty[c]);
                }
            }
            if (valid) {
                float* dst = dqkv + grow * ld3 + h * kAtcDH + 8 * grp;
                *reinterpret_cast<float4*>(dst) = make_float4(dq[0] * scale, dq[1] * scale, dq[2] * scale, dq[3] * scale);
                *reinterpret_cast<float4*>(dst + 4) =
                    make_float4(dq[4] * scale, dq[5] * scale, dq[6] * scale, dq[7] * scale);
                if (grp == 0) {
                    const long si = ((long)b * H + h) * T + r;
                    bstat[2 * si] = sumf;
                    bstat[2 * si + 1] = dr;
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

// ---- dK / dV kernel ----------------------------------------------------------

constexpr uint32_t kKvColS = 0, kKvColDp = 128, kKvColRing = 256, kKvColAcc = 384;
// 16 softmax warps and four MMA-issuing warps, one per warp scheduler: issuer
// r takes product chain r & 1 (0: S^T and dV, 1: dP^T and dK) for the chunks
// of parity r >> 1; issuers 0 and 1 also issue S^T and dP^T, issuer 0 the
// loads.
constexpr int kAtcKvIssuers = 4;
constexpr int kAtcKvThreads = kAtcSoftThreads + 32 * kAtcKvIssuers;

struct AtcKvSmem {
    float kh[kAtcTileFloats], kl[kAtcTileFloats];        // K of the key block, K-major
    float vh[kAtcTileFloats], vl[kAtcTileFloats];        // V of the key block, K-major
    float qh[kAtcTileFloats], ql[kAtcTileFloats];        // Q of the query block, K-major
    float oh[kAtcTileFloats], ol[kAtcTileFloats];        // dO of the query block, K-major
    float qmh[kAtcTileFloats], qml[kAtcTileFloats];      // Q, MN-major
    float omh[kAtcTileFloats], oml[kAtcTileFloats];      // dO, MN-major
    float negml[kAtcTile], inv[kAtcTile], dr[kAtcTile];  // per-query statistics of the block
    uint64_t ld_kv, ld_q, conv_kv, conv_q, sd_ready, blk_done, drained, drain;
    uint64_t ring_full[2], ring_empty[2], kv_chunk[2];
    uint32_t tmem_addr;
    int abort;
};
constexpr size_t kAtcKvSmemBytes = sizeof(AtcKvSmem) + 1024;
static_assert(kAtcKvSmemBytes <= 232448, "attention dK/dV kernel shared memory exceeds the 227 KB per-CTA limit");

// TMEM column of chunk c's dV (dk = false) or dK accumulator: chunks 0 and 1
// in the two dedicated 64-column slots, chunk c >= 2 over the S^T (dV) or
// dP^T (dK) columns of chunk c - 2, whose MMAs have completed by then.
__device__ __forceinline__ uint32_t atc_kv_acc(int c, bool dk) {
    return c < 2 ? kKvColAcc + 64u * c + (dk ? 32u : 0u) : (dk ? kKvColDp : kKvColS) + 32u * (c - 2);
}

// Visibility of a 32-query chunk (queries 128 qb + 32 c ..) to the 32 keys
// 128 kb + 32 q .. of a warp: 2 all visible, 1 diagonal or ragged, 0 none.
__device__ __forceinline__ int atc_kv_chunk_vis(int kb, int q, int qb, int c, bool cols_valid) {
    if (qb > kb) return cols_valid ? 2 : 1;
    if (c > q) return cols_valid ? 2 : 1;
    return c == q ? 1 : 0;
}

__global__ void __launch_bounds__(kAtcKvThreads, 1)
attention_bwd_dkdv_tc_kernel(const __grid_constant__ CUtensorMap map_qk, const __grid_constant__ CUtensorMap map_mn,
                             const __grid_constant__ CUtensorMap map_do, const __grid_constant__ CUtensorMap map_do_mn,
                             int T, int D, int H, float scale, const float* __restrict__ qkv,
                             const float* __restrict__ dctx, const float* __restrict__ row_max,
                             const float* __restrict__ bstat, float* __restrict__ dqkv, int* __restrict__ err)
{
    HX_PDL_PROLOGUE();
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    const uint32_t pad = (1024u - (tc::smem_u32(smem_raw) & 1023u)) & 1023u;
    AtcKvSmem& sm = *reinterpret_cast<AtcKvSmem*>(smem_raw + pad);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int h = blockIdx.x, b = blockIdx.y, kb = blockIdx.z;
    const int ntile = T > kAtcTile ? 2 : 1;
    const int nqb = ntile - kb;  // query blocks kb .. ntile-1
    const int y0 = b * T;

    if (threadIdx.x == 0) {
        tc::mbar_init(&sm.ld_kv, 1);
        tc::mbar_init(&sm.ld_q, 1);
        tc::mbar_init(&sm.conv_kv, kAtcSoftThreads);
        tc::mbar_init(&sm.conv_q, kAtcSoftThreads);
        tc::mbar_init(&sm.sd_ready, 2);              // the S^T and dP^T issuers
        tc::mbar_init(&sm.blk_done, kAtcKvIssuers);  // every issuer
        tc::mbar_init(&sm.drained, kAtcSoftWarps);
        tc::mbar_init(&sm.drain, kAtcKvIssuers);
        for (int i = 0; i < 2; ++i) {
            tc::mbar_init(&sm.ring_full[i], 4);
            tc::mbar_init(&sm.ring_empty[i], 2);  // the two chains' issuers of slot i's parity
            tc::mbar_init(&sm.kv_chunk[i], 2);
        }
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
        // this CTA's later query blocks (their TMA loads wait for the
        // previous block) and the next wave's first Q/dO block and K/V
        // block, into L2
        if (nqb > 1) {
            atc_prefetch_rows(qkv, 3L * D, h * kAtcDH, y0 + kAtcTile * (kb + 1), min(y0 + T, y0 + kAtcTile * (kb + nqb)),
                              threadIdx.x, kAtcSoftThreads);
            atc_prefetch_rows(dctx, D, h * kAtcDH, y0 + kAtcTile * (kb + 1), min(y0 + T, y0 + kAtcTile * (kb + nqb)),
                              threadIdx.x, kAtcSoftThreads);
        }
        const int nb = atc_next_wave_block();
        if (nb >= 0) {
            const int nh = nb % H, nbb = (nb / H) % gridDim.y, nkb = nb / (H * (int)gridDim.y);
            const int r0 = nbb * T + kAtcTile * nkb, r1 = min(nbb * T + T, r0 + kAtcTile);
            for (int part = 0; part < 3; ++part)
                atc_prefetch_rows(qkv, 3L * D, part * D + nh * kAtcDH, r0, r1, threadIdx.x, kAtcSoftThreads);
            atc_prefetch_rows(dctx, D, nh * kAtcDH, r0, r1, threadIdx.x, kAtcSoftThreads);
        }
    }
    if (warp >= kAtcSoftWarps) {
        // Four issuers on the four warp schedulers.  Chain role & 1: 0 is
        // S^T = K Q^T and dV_c = P^T_c dO_c, 1 is dP^T = V dO^T and
        // dK_c = dS^T_c Q_c; issuers 0 and 1 issue S^T and dP^T (and 0 the
        // TMA loads), issuer r the chunks c of parity r >> 1, so chunk g's
        // ring slot and accumulator barrier (g & 1) belong to the two
        // issuers of that parity.  Each accumulator's MMAs keep the
        // single-issuer term order, so the results are the same bit for bit.
        const int role = warp - kAtcSoftWarps;
        const int chain = role & 1, par = role >> 1;
        if (lane == 0) {
            const int yk = y0 + kAtcTile * kb;
            if (role == 0) {
                tc::prefetch_tensormap(&map_qk);
                tc::prefetch_tensormap(&map_mn);
                tc::prefetch_tensormap(&map_do);
                tc::prefetch_tensormap(&map_do_mn);
                tc::mbar_arrive_expect_tx(&sm.ld_kv, 2 * kAtcTileFloats * 4);
                tc::tma_load_2d(sm.kh, &map_qk, &sm.ld_kv, D + h * kAtcDH, yk);
                tc::tma_load_2d(sm.vh, &map_qk, &sm.ld_kv, 2 * D + h * kAtcDH, yk);
            }
            // this chain's A operand of the S^T / dP^T product (K or V) and
            // B operand (Q or dO, K-major); its chunk products' B (dO or Q,
            // MN-major)
            const uint32_t ah = tc::smem_u32(chain ? sm.vh : sm.kh), al = tc::smem_u32(chain ? sm.vl : sm.kl);
            const uint32_t bh = tc::smem_u32(chain ? sm.oh : sm.qh), bl = tc::smem_u32(chain ? sm.ol : sm.ql);
            const uint32_t mh = tc::smem_u32(chain ? sm.qmh : sm.omh), ml = tc::smem_u32(chain ? sm.qml : sm.oml);
            const uint32_t col_sd = chain ? kKvColDp : kKvColS;
            constexpr uint32_t idesc_s = tc::idesc_tf32(kAtcTile, kAtcTile, false, false);
            uint32_t g0 = 0;  // chunks of earlier blocks (ring and accumulator position)
            for (int i = 0; i < nqb; ++i) {
                const int qb = kb + i;
                // the previous block's MMAs are done before its tiles are overwritten
                if (i > 0) atc_wait(sm.abort, err, kAtcErrMma, &sm.blk_done, (i - 1) & 1);
                if (role == 0) {
                    const int yq = y0 + kAtcTile * qb;
                    tc::mbar_arrive_expect_tx(&sm.ld_q, 4 * kAtcTileFloats * 4);
                    tc::tma_load_2d(sm.qh, &map_qk, &sm.ld_q, h * kAtcDH, yq);
                    tc::tma_load_2d(sm.qmh, &map_mn, &sm.ld_q, h * kAtcDH, yq);
                    tc::tma_load_2d(sm.oh, &map_do, &sm.ld_q, h * kAtcDH, yq);
                    tc::tma_load_2d(sm.omh, &map_do_mn, &sm.ld_q, h * kAtcDH, yq);
                }
                if (i == 0) atc_wait(sm.abort, err, kAtcErrMma, &sm.conv_kv, 0);
                atc_wait(sm.abort, err, kAtcErrMma, &sm.conv_q, i & 1);
                // the previous block's accumulators, over S^T / dP^T, are read
                if (i > 0) atc_wait(sm.abort, err, kAtcErrMma, &sm.drained, (i - 1) & 1);
                tc::tc_fence_after();
                // S^T = K Q^T or dP^T = V dO^T (A from shared memory; hi*lo
                // and lo*hi per k-step, then hi*hi; descriptors built once,
                // k-step k at + 2 k in the start address field)
                if (role < 2) {
                    const uint64_t dah = tc::smem_desc(ah, 16, 1024, tc::kLayoutSw128);
                    const uint64_t dal = tc::smem_desc(al, 16, 1024, tc::kLayoutSw128);
                    const uint64_t dbh = tc::smem_desc(bh, 16, 1024, tc::kLayoutSw128);
                    const uint64_t dbl = tc::smem_desc(bl, 16, 1024, tc::kLayoutSw128);
                    const uint32_t d = tmem + col_sd;
#pragma unroll
                    for (int k = 0; k < kAtcDH / 8; ++k) {
                        tc::mma_tf32(d, dal + 2 * k, dbh + 2 * k, idesc_s, k > 0 ? 1u : 0u);
                        tc::mma_tf32(d, dah + 2 * k, dbl + 2 * k, idesc_s, 1u);
                    }
#pragma unroll
                    for (int k = 0; k < kAtcDH / 8; ++k) tc::mma_tf32(d, dah + 2 * k, dbh + 2 * k, idesc_s, 1u);
                }
                if (role < 2) tc::mma_commit(&sm.sd_ready);
                // per 32-query chunk of this issuer's parity: dV_c = P^T_c dO_c
                // (chain 0) or dK_c = dS^T_c Q_c (chain 1); chunk c's slot in
                // the 2-slot lo ring is g & 1
                for (int c = par; c < 4; c += 2) {
                    const uint32_t g = g0 + c;
                    const int slot = g & 1;
                    atc_wait(sm.abort, err, kAtcErrMma, &sm.ring_full[slot], (g >> 1) & 1);
                    // chunk g - 2's MMAs (both chains) have completed, so the
                    // S^T / dP^T columns that chunk c - 2 read are free for
                    // chunk c's results while chunk c - 1's MMAs still run
                    if (g >= 2) atc_wait(sm.abort, err, kAtcErrMma, &sm.kv_chunk[g & 1], ((g >> 1) & 1) ^ 1);
                    tc::tc_fence_after();
                    const uint32_t row = uint32_t(32 * c) * 128;
                    const uint32_t d[1] = {tmem + atc_kv_acc(c, chain == 1)};
                    const uint32_t ahi[1] = {tmem + col_sd + 32 * c};
                    const uint32_t alo[1] = {tmem + kKvColRing + 64 * slot + (chain ? 32u : 0u)};
                    const uint32_t bhi[1] = {mh + row}, blo[1] = {ml + row};
                    atc_mma_chunks_mn<1>(d, ahi, alo, bhi, blo);
                    tc::mma_commit(&sm.ring_empty[slot]);
                    tc::mma_commit(&sm.kv_chunk[g & 1]);
                }
                g0 += 4;
                tc::mma_commit(&sm.blk_done);
            }
            tc::mma_commit(&sm.drain);
            tc::mbar_wait(&sm.drain, 0);
            if (role == 0) {
                tc::mbar_wait(&sm.ld_kv, 0);
                if (nqb > 0) tc::mbar_wait(&sm.ld_q, (nqb - 1) & 1);
            }
        }
    } else {
        const int st = threadIdx.x;
        const int q = warp & 3, grp = warp >> 2;
        const uint32_t lane_base = tmem + (uint32_t(32 * q) << 16);
        const int j = kAtcTile * kb + 32 * q + lane;  // this thread's key
        const float c1 = scale * kAtcLog2e;
        atc_wait(sm.abort, err, kAtcErrLoad, &sm.ld_kv, 0);
        atc_split(sm.kh, sm.kl, kAtcTileFloats / 4, st, kAtcSoftThreads);
        atc_split(sm.vh, sm.vl, kAtcTileFloats / 4, st, kAtcSoftThreads);
        tc::fence_proxy_async_smem();
        tc::mbar_arrive(&sm.conv_kv);
        float dv[8], dk[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) { dv[i] = 0.f; dk[i] = 0.f; }
        uint32_t g = 0;
        for (int i = 0; i < nqb; ++i) {
            const int qb = kb + i;
            const int q0 = kAtcTile * qb;
            // query statistics of the block (the previous block's readers are
            // past this point's barrier below)
            if (st < kAtcTile) {
                const int r = q0 + st;
                const long si = ((long)b * H + h) * T + r;
                const bool ok = r < T;
                sm.negml[st] = ok ? __fmul_rn(row_max[si], -kAtcLog2e) : 0.f;
                sm.inv[st] = ok ? __frcp_rn(bstat[2 * si]) : 0.f;
                sm.dr[st] = ok ? bstat[2 * si + 1] : 0.f;
            }
            atc_wait(sm.abort, err, kAtcErrLoad, &sm.ld_q, i & 1);
            atc_split(sm.qh, sm.ql, kAtcTileFloats / 4, st, kAtcSoftThreads);
            atc_split(sm.oh, sm.ol, kAtcTileFloats / 4, st, kAtcSoftThreads);
            atc_split(sm.qmh, sm.qml, kAtcTileFloats / 4, st, kAtcSoftThreads);
            atc_split(sm.omh, sm.oml, kAtcTileFloats / 4, st, kAtcSoftThreads);
            tc::fence_proxy_async_smem();
            tc::mbar_arrive(&sm.conv_q);
            atc_soft_sync();  // statistics visible
            atc_wait(sm.abort, err, kAtcErrSoftmax, &sm.sd_ready, i & 1);
            tc::tc_fence_after();
            // this thread's chunk: queries q0 + 32 grp ..
            const uint32_t gc = g + grp;
            const int slot = gc & 1;
            atc_wait(sm.abort, err, kAtcErrSoftmax, &sm.ring_empty[slot], ((gc >> 1) & 1) ^ 1);
            tc::tc_fence_after();
            const bool cols_valid = q0 + 32 * grp + 31 < T;
            const int vis = atc_kv_chunk_vis(kb, q, qb, grp, cols_valid);
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                const uint32_t col = 32 * grp + 16 * half;
                uint32_t sv[16], pv[16];
                if (vis) {
                    tc::tmem_ld_32x32b_x16(lane_base + kKvColS + col, sv);
                    tc::tmem_ld_32x32b_x16(lane_base + kKvColDp + col, pv);
                    tc::tmem_ld_wait();
                    uint32_t plo[16], dlo[16];
                    // two queries per paired FP32 instruction; the statistics
                    // of four queries per 16-byte shared-memory load
#pragma unroll
                    for (int x = 0; x < 16; x += 4) {
                        const float4 nm = *reinterpret_cast<const float4*>(&sm.negml[col + x]);
                        const float4 iv = *reinterpret_cast<const float4*>(&sm.inv[col + x]);
                        const float4 d4 = *reinterpret_cast<const float4*>(&sm.dr[col + x]);
#pragma unroll
                        for (int y = 0; y < 4; y += 2) {
                            const int rloc = int(col) + x + y;  // queries q0 + rloc, + 1
                            const float2 t = tc::fma2_rn(
                                make_float2(__uint_as_float(sv[x + y]), __uint_as_float(sv[x + y + 1])),
                                make_float2(c1, c1), y ? make_float2(nm.z, nm.w) : make_float2(nm.x, nm.y));
                            float e0 = tc::exp2_approx(t.x), e1 = tc::exp2_approx(t.y);
                            if (vis == 1) {
                                if (j > q0 + rloc || q0 + rloc >= T) e0 = 0.f;
                                if (j > q0 + rloc + 1 || q0 + rloc + 1 >= T) e1 = 0.f;
                            }
                            const float2 p = tc::mul2_rn(make_float2(e0, e1), y ? make_float2(iv.z, iv.w)
                                                                                 : make_float2(iv.x, iv.y));
                            const float2 ds = tc::mul2_rn(
                                p, tc::sub2_rn(make_float2(__uint_as_float(pv[x + y]), __uint_as_float(pv[x + y + 1])),
                                               y ? make_float2(d4.z, d4.w) : make_float2(d4.x, d4.y)));
                            sv[x + y] = tc::tf32_rna_bits(p.x);
                            sv[x + y + 1] = tc::tf32_rna_bits(p.y);
                            pv[x + y] = tc::tf32_rna_bits(ds.x);
                            pv[x + y + 1] = tc::tf32_rna_bits(ds.y);
                            const float2 pl = tc::sub2_rn(p, make_float2(__uint_as_float(sv[x + y]),
                                                                         __uint_as_float(sv[x + y + 1])));
                            const float2 dl = tc::sub2_rn(ds, make_float2(__uint_as_float(pv[x + y]),
                                                                          __uint_as_float(pv[x + y + 1])));
                            plo[x + y] = __float_as_uint(pl.x);
                            plo[x + y + 1] = __float_as_uint(pl.y);
                            dlo[x + y] = __float_as_uint(dl.x);
                            dlo[x + y + 1] = __float_as_uint(dl.y);
                        }
                    }
                    tc::tmem_st_32x32b_x16(lane_base + kKvColRing + 64 * slot + 16 * half, plo);
                    tc::tmem_st_32x32b_x16(lane_base + kKvColRing + 64 * slot + 32 + 16 * half, dlo);
                } else {
#pragma unroll
                    for (int x = 0; x < 16; ++x) { sv[x] = 0u; pv[x] = 0u; }
                    tc::tmem_st_32x32b_x16(lane_base + kKvColRing + 64 * slot + 16 * half, sv);
                    tc::tmem_st_32x32b_x16(lane_base + kKvColRing + 64 * slot + 32 + 16 * half, pv);
                }
                tc::tmem_st_32x32b_x16(lane_base + kKvColS + col, sv);
                tc::tmem_st_32x32b_x16(lane_base + kKvColDp + col, pv);
            }
            tc::tmem_st_wait();
            tc::tc_fence_before();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&sm.ring_full[slot]);
            // the block's four chunks, once its MMAs have completed
            atc_wait(sm.abort, err, kAtcErrEpilogue, &sm.blk_done, i & 1);
            tc::tc_fence_after();
            for (int c = 0; c < 4; ++c) {
                if (atc_kv_chunk_vis(kb, q, qb, c, true)) {
                    uint32_t a[8], k8[8];
                    tc::tmem_ld_32x32b_x8(lane_base + atc_kv_acc(c, false) + 8 * grp, a);
                    tc::tmem_ld_32x32b_x8(lane_base + atc_kv_acc(c, true) + 8 * grp, k8);
                    tc::tmem_ld_wait();
#pragma unroll
                    for (int x = 0; x < 8; ++x) {
                        dv[x] = __fadd_rn(dv[x], __uint_as_float(a[x]));
                        dk[x] = __fadd_rn(dk[x], __uint_as_float(k8[x]));
                    }
                }
            }
            tc::tc_fence_before();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&sm.drained);
            g += 4;
            atc_soft_sync();  // statistics of this block no longer read
        }
        if (j < T) {
            float* dst = dqkv + ((long)y0 + j) * 3 * D + h * kAtcDH + 8 * grp;
            *reinterpret_cast<float4*>(dst + D) = make_float4(dk[0] * scale, dk[1] * scale, dk[2] * scale, dk[3] * scale);
            *reinterpret_cast<float4*>(dst + D + 4) =
                make_float4(dk[4] * scale, dk[5] * scale, dk[6] * scale, dk[7] * scale);
            *reinterpret_cast<float4*>(dst + 2 * D) = make_float4(dv[0], dv[1], dv[2], dv[3]);
            *reinterpret_cast<float4*>(dst + 2 * D + 4) = make_float4(dv[4], dv[5], dv[6], dv[7]);
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
