// gemm.cuh -- GEMM dispatch: picks a tile shape and a K split for a problem
// and launches it on the runtime stream.
#pragma once

#include "gemm_simt.cuh"
#include "hx_internal.cuh"

namespace hx {

template <int BM, int BN, int BK, int TX, int TY, bool AT, bool BT, class Epi>
void launch_simt(hx_runtime* rt, int M, int N, int K, const float* A, long lda, const float* B, long ldb,
                 Epi epi)
{
    using S = SimtShape<BM, BN, BK, TX, TY>;
    const int tiles_m = (M + BM - 1) / BM, tiles_n = (N + BN - 1) / BN;
    const long tiles = (long)tiles_m * tiles_n;
    // Split K when the output alone cannot fill the SMs and K is long.
    int splits = 1;
    const int min_chunk = BK * 8;
    if (tiles < rt->sm_count && K >= 2 * min_chunk) {
        splits = (int)((2 * rt->sm_count + tiles - 1) / tiles);
        splits = std::min(splits, K / min_chunk);
        splits = std::max(1, std::min(splits, 64));
    }
    int chunk = (K + splits - 1) / splits;
    chunk = ((chunk + BK - 1) / BK) * BK;
    splits = (K + chunk - 1) / chunk;
    if (K == 0) { splits = 1; chunk = BK; }
    dim3 grid(tiles_n, tiles_m, splits);
    if (splits == 1) {
        gemm_simt_kernel<S, BM, BN, BK, TX, TY, AT, BT, Epi>
            <<<grid, S::kThreads, 0, rt->stream>>>(M, N, K, A, lda, B, ldb, chunk, epi, nullptr);
        HX_LAUNCHED(rt);
    } else {
        float* ws = rt->workspace(sizeof(float) * (size_t)splits * M * N);
        gemm_simt_kernel<S, BM, BN, BK, TX, TY, AT, BT, Epi>
            <<<grid, S::kThreads, 0, rt->stream>>>(M, N, K, A, lda, B, ldb, chunk, epi, ws);
        HX_LAUNCHED(rt);
        const long total = (long)M * N;
        const int threads = 256;
        const int blocks = (int)std::min<long>((total + threads - 1) / threads, 4L * rt->sm_count * 8);
        splitk_reduce_kernel<Epi><<<blocks, threads, 0, rt->stream>>>(M, N, splits, ws, epi);
        HX_LAUNCHED(rt);
    }
}

// C = op(A) op(B) with the epilogue applied to every element.
template <bool AT, bool BT, class Epi>
void gemm(hx_runtime* rt, int M, int N, int K, const float* A, long lda, const float* B, long ldb, Epi epi)
{
    require(M > 0 && N > 0 && K >= 0, HX_ERR_ARGUMENT, "gemm: bad shape");
    ProfScope prof(rt, kTagGemm, 2.0 * M * N * K, 4.0 * ((double)M * K + (double)K * N + (double)M * N));
    const long mn = (long)M * N;
    if (mn >= 128L * 128 * rt->sm_count / 2)
        launch_simt<128, 128, 8, 16, 16, AT, BT>(rt, M, N, K, A, lda, B, ldb, epi);
    else if (mn >= 64L * 64 * rt->sm_count / 4)
        launch_simt<64, 64, 16, 16, 16, AT, BT>(rt, M, N, K, A, lda, B, ldb, epi);
    else
        launch_simt<32, 32, 32, 8, 8, AT, BT>(rt, M, N, K, A, lda, B, ldb, epi);
}

}  // namespace hx
