// gemm.cuh -- GEMM dispatch: picks a tile shape and a K split for a problem
// and launches it on the runtime stream.
#pragma once

#include "gemm_simt.cuh"
#include "gemm_tc.cuh"
#include "hx_internal.cuh"

namespace hx {

// Sums the split-K partials in split order and applies the epilogue: four
// elements per thread with 16-byte loads when the rows allow it.
template <class Epi>
void launch_splitk_reduce(hx_runtime* rt, int M, int N, int splits, const float* ws, Epi epi)
{
    const long total = (long)M * N;
    const int threads = 256;
    if (N % 4 == 0 && (reinterpret_cast<uintptr_t>(ws) & 15) == 0) {
        const int blocks = (int)std::min<long>((total / 4 + threads - 1) / threads, 4L * rt->sm_count * 8);
        ::hx::pdl_launch(splitk_reduce4_kernel<Epi>, blocks, threads, 0, rt->stream, M, N, splits, ws, epi);
    } else {
        const int blocks = (int)std::min<long>((total + threads - 1) / threads, 4L * rt->sm_count * 8);
        ::hx::pdl_launch(splitk_reduce_kernel<Epi>, blocks, threads, 0, rt->stream, M, N, splits, ws, epi);
    }
    HX_LAUNCHED(rt);
}

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
        ::hx::pdl_launch(gemm_simt_kernel<S, BM, BN, BK, TX, TY, AT, BT, Epi>, grid, S::kThreads, 0, rt->stream, M, N, K, A, lda, B, ldb, chunk, epi, nullptr);
        HX_LAUNCHED(rt);
    } else {
        float* ws = rt->workspace(sizeof(float) * (size_t)splits * M * N);
        ::hx::pdl_launch(gemm_simt_kernel<S, BM, BN, BK, TX, TY, AT, BT, Epi>, grid, S::kThreads, 0, rt->stream, M, N, K, A, lda, B, ldb, chunk, epi, ws);
        HX_LAUNCHED(rt);
        launch_splitk_reduce(rt, M, N, splits, ws, epi);
    }
}

// ---- tensor-core path ------------------------------------------------------

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_tiled() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        check_cuda(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q),
                   "cudaGetDriverEntryPoint(cuTensorMapEncodeTiled)");
        require(q == cudaDriverEntryPointSuccess && p, HX_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
        fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

// Row-major FP32 matrix [outer][inner] with leading dimension ld (elements),
// boxes of box_inner x box_outer, zero fill out of bounds.  K-major operand
// tiles use the 128B swizzle; MN-major tiles the 128B swizzle with 32-byte
// atoms (the layout the MMA requires for MN-major 32-bit operands); output
// tiles written by TMA stores no swizzle.
inline CUtensorMap make_map(const float* base, uint64_t inner, uint64_t outer, uint64_t ld, uint32_t box_inner,
                            uint32_t box_outer, CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_128B) {
    CUtensorMap m;
    const cuuint64_t dims[2] = {inner, outer};
    const cuuint64_t strides[1] = {ld * sizeof(float)};
    const cuuint32_t box[2] = {box_inner, box_outer};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = encode_tiled()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides,
                                      box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    require(r == CUDA_SUCCESS, HX_ERR_CUDA, "cuTensorMapEncodeTiled failed (" + std::to_string(int(r)) + ")");
    return m;
}

// Row-major FP32 [z][outer][inner] (strides ld and zstride elements), box
// box_inner x box_outer x 1.
inline CUtensorMap make_map3(const float* base, uint64_t inner, uint64_t outer, uint64_t depth, uint64_t ld,
                             uint64_t zstride, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swz) {
    CUtensorMap m;
    const cuuint64_t dims[3] = {inner, outer, depth};
    const cuuint64_t strides[2] = {ld * sizeof(float), zstride * sizeof(float)};
    const cuuint32_t box[3] = {box_inner, box_outer, 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    const CUresult r = encode_tiled()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(base), dims, strides,
                                      box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    require(r == CUDA_SUCCESS, HX_ERR_CUDA, "cuTensorMapEncodeTiled (3-D) failed (" + std::to_string(int(r)) + ")");
    return m;
}

inline bool tc_eligible(hx_runtime* rt, int M, int N, int K, const float* A, long lda, const float* B, long ldb) {
    if (rt->gemm_backend == HX_GEMM_CUDA_CORES) return false;
    const bool aligned = ((reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(B)) & 15) == 0 && lda % 4 == 0 &&
                         ldb % 4 == 0 && K >= 8;
    if (!aligned) return false;
    if (rt->gemm_backend == HX_GEMM_TENSOR_CORES) return true;
    return M >= 64 && N >= 64 && 2.0 * M * N * K >= 6.4e7;
}

// B of a GEMM already split for the tensor cores: hi = B rounded to TF32,
// lo = B - hi, both with B's leading dimension (weights are split once per
// step, so their tiles are not split again in every CTA that loads them).
struct BSplit {
    const float* hi = nullptr;
    const float* lo = nullptr;
};

template <bool AT, bool BT, class Epi>
void launch_tc(hx_runtime* rt, int M, int N, int K, const float* A, long lda, const float* B, long ldb, Epi epi,
               BSplit bs)
{
    // A(m,k): AT=false -> K-major rows [M][K];  AT=true -> MN-major [K][M].
    // B(k,n): BT=false -> MN-major [K][N];      BT=true -> K-major [N][K].
    constexpr bool A_MN = AT, B_MN = !BT;
    constexpr CUtensorMapSwizzle mn_swz = CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B;
    const CUtensorMap mx = A_MN ? make_map(A, M, K, lda, 32, 32, mn_swz) : make_map(A, K, M, lda, 32, kTcHalf);
    auto map_w = [&](const float* base) {
        return B_MN ? make_map(base, N, K, ldb, 32, 32, mn_swz) : make_map(base, K, N, ldb, 32, kTcHalf);
    };
    const bool split = bs.hi && bs.lo;
    const CUtensorMap mw = map_w(split ? bs.hi : B);
    const CUtensorMap mw_lo = split ? map_w(bs.lo) : mw;
    const int pairs = tc_pairs<A_MN, B_MN, false, false, Epi>(rt->sm_count);
    const TcGrid g = tc_grid(M, N, K, pairs, 2 * pairs);
    int* err = rt->device_error();
    float* ws = g.splits > 1 ? rt->workspace(sizeof(float) * (size_t)g.splits * M * N) : nullptr;
    // bulk tensor stores for the epilogue when its single output (or the
    // split-K workspace) meets TMA's 16-byte rules
    bool c_tma;
    CUtensorMap mc = mw;
    if (ws) {
        c_tma = N % 4 == 0 && (reinterpret_cast<uintptr_t>(ws) & 15) == 0;
        if (c_tma) mc = make_map3(ws, N, M, g.splits, N, (uint64_t)M * N, 32, kTcStoreRows, CU_TENSOR_MAP_SWIZZLE_NONE);
    } else {
        const float* out = epi.tma_out();
        const long ldc = epi.tma_ld();
        c_tma = epi.tma_ok() && out && (reinterpret_cast<uintptr_t>(out) & 15) == 0 && ldc % 4 == 0;
        if (c_tma) mc = make_map(out, N, M, ldc, 32, kTcStoreRows, CU_TENSOR_MAP_SWIZZLE_NONE);
    }
    cudaError_t rc;
    if (split)
        rc = c_tma ? launch_tc_kernel<A_MN, B_MN, true, true>(rt->stream, pairs, mx, mw, mw_lo, mc, g, epi, ws, err)
                   : launch_tc_kernel<A_MN, B_MN, true, false>(rt->stream, pairs, mx, mw, mw_lo, mc, g, epi, ws, err);
    else
        rc = c_tma ? launch_tc_kernel<A_MN, B_MN, false, true>(rt->stream, pairs, mx, mw, mw_lo, mc, g, epi, ws, err)
                   : launch_tc_kernel<A_MN, B_MN, false, false>(rt->stream, pairs, mx, mw, mw_lo, mc, g, epi, ws, err);
    HX_CUDA(rc);
    ++rt->metrics.kernel_launches;
    if (g.splits > 1) launch_splitk_reduce(rt, M, N, g.splits, ws, epi);
}

// C = op(A) op(B) with the epilogue applied to every element.  `bs`, when
// given, is B's TF32 hi/lo split for the tensor-core path; the CUDA-core path
// always reads B itself.
template <bool AT, bool BT, class Epi>
void gemm(hx_runtime* rt, int M, int N, int K, const float* A, long lda, const float* B, long ldb, Epi epi,
          BSplit bs = BSplit{})
{
    require(M > 0 && N > 0 && K >= 0, HX_ERR_ARGUMENT, "gemm: bad shape");
    ProfScope prof(rt, kTagGemm, 2.0 * M * N * K, 4.0 * ((double)M * K + (double)K * N + (double)M * N));
    if (tc_eligible(rt, M, N, K, A, lda, B, ldb) &&
        (!bs.hi || ((reinterpret_cast<uintptr_t>(bs.hi) | reinterpret_cast<uintptr_t>(bs.lo)) & 15) == 0)) {
        launch_tc<AT, BT>(rt, M, N, K, A, lda, B, ldb, epi, bs);
        return;
    }
    const long mn = (long)M * N;
    if (mn >= 128L * 128 * rt->sm_count / 2)
        launch_simt<128, 128, 8, 16, 16, AT, BT>(rt, M, N, K, A, lda, B, ldb, epi);
    else if (mn >= 64L * 64 * rt->sm_count / 4)
        launch_simt<64, 64, 16, 16, 16, AT, BT>(rt, M, N, K, A, lda, B, ldb, epi);
    else
        launch_simt<32, 32, 32, 8, 8, AT, BT>(rt, M, N, K, A, lda, B, ldb, epi);
}

}  // namespace hx
