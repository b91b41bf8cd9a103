// gemm_simt.cuh -- FP32 CUDA-core GEMM with fused epilogues.
//
// C[M,N] = op(A)[M,K] * op(B)[K,N], FP32 multiply-add, FP32 accumulation.
//   A(m,k) = AT ? A[k*lda + m] : A[m*lda + k]
//   B(k,n) = BT ? B[n*ldb + k] : B[k*ldb + n]
// The epilogue functor receives every output element once: epi(m, n, acc).
// With a K split (gridDim.z > 1) the kernel writes FP32 partial tiles to a
// workspace [split][M][N] and splitk_reduce applies the epilogue to the sums
// taken in split order, so results do not depend on scheduling.
//
// Used for the tiny shapes of the reference configurations (B=8..32,
// D=48..64), where the whole step is launch-latency bound and exact FP32
// products keep the results closest to the reference's double-accumulated
// CPU path.
#pragma once

#include "pdl.cuh"

#include <cuda_runtime.h>
#include <cstdint>

namespace hx {

template <int BM, int BN, int BK, int TX, int TY>
struct SimtShape {
    static constexpr int kThreads = TX * TY;
    static constexpr int kRM = BM / (TY * 4);  // 4-row groups per thread
    static constexpr int kRN = BN / (TX * 4);  // 4-col groups per thread
    static_assert(kRM * TY * 4 == BM && kRN * TX * 4 == BN, "tile/thread mismatch");
    static constexpr int kALoads = (BM * BK + kThreads - 1) / kThreads;
    static constexpr int kBLoads = (BN * BK + kThreads - 1) / kThreads;
};

template <class S, int BM, int BN, int BK, int TX, int TY, bool AT, bool BT, class Epi>
__global__ void __launch_bounds__(TX * TY)
gemm_simt_kernel(int M, int N, int K, const float* __restrict__ A, long lda,
                 const float* __restrict__ B, long ldb, int k_chunk, Epi epi,
                 float* __restrict__ partial)
{
    HX_PDL_PROLOGUE();
    constexpr int NT = S::kThreads;
    __shared__ __align__(16) float As[2][BK][BM];
    __shared__ __align__(16) float Bs[2][BK][BN];

    const int tid = threadIdx.x;
    const int tx = tid % TX, ty = tid / TX;
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
    const int kbeg = blockIdx.z * k_chunk;
    const int kend = min(K, kbeg + k_chunk);

    float regA[S::kALoads], regB[S::kBLoads];

    auto load_a = [&](int k0) {
#pragma unroll
        for (int i = 0; i < S::kALoads; ++i) {
            const int idx = tid + i * NT;
            int mm, kk;
            if (AT) { mm = idx % BM; kk = idx / BM; } else { kk = idx % BK; mm = idx / BK; }
            const int gm = m0 + mm, gk = k0 + kk;
            float v = 0.f;
            if (idx < BM * BK && gm < M && gk < kend)
                v = AT ? A[(long)gk * lda + gm] : A[(long)gm * lda + gk];
            regA[i] = v;
        }
    };
    auto load_b = [&](int k0) {
#pragma unroll
        for (int i = 0; i < S::kBLoads; ++i) {
            const int idx = tid + i * NT;
            int nn, kk;
            if (!BT) { nn = idx % BN; kk = idx / BN; } else { kk = idx % BK; nn = idx / BK; }
            const int gn = n0 + nn, gk = k0 + kk;
            float v = 0.f;
            if (idx < BN * BK && gn < N && gk < kend)
                v = BT ? B[(long)gn * ldb + gk] : B[(long)gk * ldb + gn];
            regB[i] = v;
        }
    };
    auto store_tiles = [&](int buf) {
#pragma unroll
        for (int i = 0; i < S::kALoads; ++i) {
            const int idx = tid + i * NT;
            if (idx < BM * BK) {
                int mm, kk;
                if (AT) { mm = idx % BM; kk = idx / BM; } else { kk = idx % BK; mm = idx / BK; }
                As[buf][kk][mm] = regA[i];
            }
        }
#pragma unroll
        for (int i = 0; i < S::kBLoads; ++i) {
            const int idx = tid + i * NT;
            if (idx < BN * BK) {
                int nn, kk;
                if (!BT) { nn = idx % BN; kk = idx / BN; } else { kk = idx % BK; nn = idx / BK; }
                Bs[buf][kk][nn] = regB[i];
            }
        }
    };

    float acc[S::kRM * 4][S::kRN * 4];
#pragma unroll
    for (int i = 0; i < S::kRM * 4; ++i)
#pragma unroll
        for (int j = 0; j < S::kRN * 4; ++j) acc[i][j] = 0.f;

    int buf = 0;
    if (kbeg < kend) {
        load_a(kbeg);
        load_b(kbeg);
        store_tiles(0);
    }
    __syncthreads();
    for (int k0 = kbeg; k0 < kend; k0 += BK) {
        const bool more = k0 + BK < kend;
        if (more) { load_a(k0 + BK); load_b(k0 + BK); }
#pragma unroll
        for (int kk = 0; kk < BK; ++kk) {
            float a[S::kRM * 4], b[S::kRN * 4];
#pragma unroll
            for (int g = 0; g < S::kRM; ++g) {
                const float4 v = *reinterpret_cast<const float4*>(&As[buf][kk][g * (BM / S::kRM) + ty * 4]);
                a[g * 4 + 0] = v.x; a[g * 4 + 1] = v.y; a[g * 4 + 2] = v.z; a[g * 4 + 3] = v.w;
            }
#pragma unroll
            for (int g = 0; g < S::kRN; ++g) {
                const float4 v = *reinterpret_cast<const float4*>(&Bs[buf][kk][g * (BN / S::kRN) + tx * 4]);
                b[g * 4 + 0] = v.x; b[g * 4 + 1] = v.y; b[g * 4 + 2] = v.z; b[g * 4 + 3] = v.w;
            }
#pragma unroll
            for (int i = 0; i < S::kRM * 4; ++i)
#pragma unroll
                for (int j = 0; j < S::kRN * 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
        if (more) {
            store_tiles(buf ^ 1);
            __syncthreads();
            buf ^= 1;
        }
    }

#pragma unroll
    for (int gi = 0; gi < S::kRM; ++gi)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int m = m0 + gi * (BM / S::kRM) + ty * 4 + i;
            if (m >= M) continue;
#pragma unroll
            for (int gj = 0; gj < S::kRN; ++gj)
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int n = n0 + gj * (BN / S::kRN) + tx * 4 + j;
                    if (n >= N) continue;
                    const float v = acc[gi * 4 + i][gj * 4 + j];
                    if (partial)
                        partial[((long)blockIdx.z * M + m) * N + n] = v;
                    else
                        epi(m, n, v);
                }
        }
}

template <class Epi>
__global__ void splitk_reduce_kernel(int M, int N, int splits, const float* __restrict__ partial, Epi epi)
{
    HX_PDL_PROLOGUE();
    const long total = (long)M * N;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
        float s = 0.f;
        for (int z = 0; z < splits; ++z) s += partial[(long)z * total + i];
        epi(int(i / N), int(i % N), s);
    }
}

// The same for N % 4 == 0 with 16-byte aligned partials: each thread sums
// four consecutive elements of a row with 16-byte loads, in the same split
// order, so the results are bit-identical to splitk_reduce_kernel's.
template <class Epi>
__global__ void splitk_reduce4_kernel(int M, int N, int splits, const float* __restrict__ partial, Epi epi)
{
    HX_PDL_PROLOGUE();
    const long total4 = (long)M * N / 4, stride4 = (long)M * N / 4;
    const float4* p4 = reinterpret_cast<const float4*>(partial);
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total4; i += (long)gridDim.x * blockDim.x) {
        float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int z = 0; z < splits; ++z) {
            const float4 v = __ldcs(p4 + (long)z * stride4 + i);
            s.x += v.x; s.y += v.y; s.z += v.z; s.w += v.w;
        }
        const long e = 4 * i;
        const int m = int(e / N), n = int(e % N);
        epi(m, n, s.x);
        epi(m, n + 1, s.y);
        epi(m, n + 2, s.z);
        epi(m, n + 3, s.w);
    }
}

// ---- epilogues -----------------------------------------------------------
// Each epilogue is split into prefetch(m, n) -- the one global value it reads
// for element (m, n), 0 if none -- and finish(m, n, v, pre).  The tensor-core
// epilogue issues the prefetches of a whole chunk before finishing any of
// them, so those loads are in flight together; operator() is the fused form.
// An epilogue that writes one float array can also hand its results to TMA
// bulk stores: tma_ok() (host) says so for this instance, tma_out()/tma_ld()
// name the array, and value(v, pre) is the element written.  An epilogue that
// reads also names, by pre_addr(m, n), the address prefetch(m, n) reads, so
// that the tensor-core epilogue can pull a tile's inputs into L2 early.

struct EpiStore {  // C[m*ldc + n] = v, with an optional column split:
    static constexpr bool kReads = false;  // prefetch() loads from global memory
    // column n goes to C + (n / split) * split_stride + m*ldc + n % split
    float* c;
    long ldc;
    int split;           // 0 = no split
    long split_stride;
    __device__ float prefetch(int, int) const { return 0.f; }
    __device__ void finish(int m, int n, float v, float) const {
        if (split) c[(long)(n / split) * split_stride + (long)m * ldc + (n % split)] = v;
        else c[(long)m * ldc + n] = v;
    }
    __device__ void operator()(int m, int n, float v) const { finish(m, n, v, 0.f); }
    bool tma_ok() const { return split == 0; }
    float* tma_out() const { return c; }
    __host__ __device__ long tma_ld() const { return ldc; }
    __device__ float value(float v, float) const { return v; }
};

struct EpiAddResidual {  // out = res + v   (r1 = x + ctx*Wo ; out = r1 + relu*W2)
    static constexpr bool kReads = true;  // prefetch() loads from global memory
    const float* res;
    float* out;
    long ld;
    __device__ float prefetch(int m, int n) const { return res[(long)m * ld + n]; }
    __device__ const float* pre_addr(int m, int n) const { return res + (long)m * ld + n; }
    __device__ void finish(int m, int n, float v, float r) const { out[(long)m * ld + n] = __fadd_rn(r, v); }
    __device__ void operator()(int m, int n, float v) const { finish(m, n, v, prefetch(m, n)); }
    bool tma_ok() const { return true; }
    float* tma_out() const { return out; }
    __host__ __device__ long tma_ld() const { return ld; }
    __device__ float value(float v, float r) const { return __fadd_rn(r, v); }
};

struct EpiRelu {  // h = max(0, z) ; optional mask = h > 0
    static constexpr bool kReads = false;  // prefetch() loads from global memory
    float* h;
    uint8_t* mask;
    long ld;
    __device__ float prefetch(int, int) const { return 0.f; }
    __device__ void finish(int m, int n, float v, float) const {
        const long i = (long)m * ld + n;
        const float r = (0.f < v) ? v : 0.f;
        h[i] = r;
        if (mask) mask[i] = r > 0.f ? 1 : 0;
    }
    __device__ void operator()(int m, int n, float v) const { finish(m, n, v, 0.f); }
    bool tma_ok() const { return mask == nullptr; }
    float* tma_out() const { return h; }
    __host__ __device__ long tma_ld() const { return ld; }
    __device__ float value(float v, float) const { return (0.f < v) ? v : 0.f; }
};

struct EpiReluBackward {  // dz = (act > 0) ? v : 0 ; optional raw store of v
    static constexpr bool kReads = true;  // prefetch() loads from global memory
    const float* act;
    float* dz;
    float* raw;
    long ld;
    __device__ float prefetch(int m, int n) const { return act[(long)m * ld + n]; }
    __device__ const float* pre_addr(int m, int n) const { return act + (long)m * ld + n; }
    __device__ void finish(int m, int n, float v, float a) const {
        const long i = (long)m * ld + n;
        if (raw) raw[i] = v;
        dz[i] = a > 0.f ? v : 0.f;
    }
    __device__ void operator()(int m, int n, float v) const { finish(m, n, v, prefetch(m, n)); }
    bool tma_ok() const { return raw == nullptr; }
    float* tma_out() const { return dz; }
    __host__ __device__ long tma_ld() const { return ld; }
    __device__ float value(float v, float a) const { return a > 0.f ? v : 0.f; }
};

struct EpiError {  // P = v ; E = P - Y ; dP = (P - Y) * s
    static constexpr bool kReads = true;  // prefetch() loads from global memory
    const float* y;
    float* p;
    float* e;
    float* dp;
    float s;
    long ld;
    __device__ float prefetch(int m, int n) const { return y[(long)m * ld + n]; }
    __device__ const float* pre_addr(int m, int n) const { return y + (long)m * ld + n; }
    __device__ void finish(int m, int n, float v, float yv) const {
        const long i = (long)m * ld + n;
        const float err = __fsub_rn(v, yv);
        if (p) p[i] = v;
        if (e) e[i] = err;
        dp[i] = __fmul_rn(err, s);
    }
    __device__ void operator()(int m, int n, float v) const { finish(m, n, v, prefetch(m, n)); }
    bool tma_ok() const { return false; }
    float* tma_out() const { return dp; }
    __host__ __device__ long tma_ld() const { return ld; }
    __device__ float value(float v, float) const { return v; }
};

struct EpiSgd {  // dW = v (optional) ; W_next = W - lr*dW (two roundings, as the reference)
    static constexpr bool kReads = true;  // prefetch() loads from global memory
    const float* w;
    float* dw;
    float* w_next;
    float lr;
    long ld;
    __device__ float prefetch(int m, int n) const { return w[(long)m * ld + n]; }
    __device__ const float* pre_addr(int m, int n) const { return w + (long)m * ld + n; }
    __device__ void finish(int m, int n, float v, float wv) const {
        const long i = (long)m * ld + n;
        if (dw) dw[i] = v;
        w_next[i] = __fsub_rn(wv, __fmul_rn(lr, v));
    }
    __device__ void operator()(int m, int n, float v) const { finish(m, n, v, prefetch(m, n)); }
    bool tma_ok() const { return false; }
    float* tma_out() const { return w_next; }
    __host__ __device__ long tma_ld() const { return ld; }
    __device__ float value(float v, float) const { return v; }
};

}  // namespace hx
