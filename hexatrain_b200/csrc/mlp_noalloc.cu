// mlp_noalloc.cu -- the MLP full step on device buffers without any device
// allocation.
//
// Who needs this: a caller whose process has already handed the GPU's memory
// to its own allocator (a host framework's caching pool that reserved the
// free HBM, or an embedding that forbids cudaMalloc/cudaFree on its step
// path because they synchronise the device and stall its other streams)
// cannot let this library allocate on the step path.  hx_mlp_prepare
// allocates an arena for the step's intermediates, and the first run of a
// shape may grow the split-K workspace, so hx_mlp_execute_device is not
// usable there.  hx_mlp_execute_device_noalloc runs the same step without
// either: the intermediates live in one fixed array of device memory that
// is part of this library's module, reserved on every GPU that loads the
// library for as long as the process runs.
//
// The array (kNoallocScratchBytes = 4 MiB):
//   [0, 4)          error word of the tensor-core pipeline waits
//   [64, 68)        finished-block counter of the loss reduction
//   [256, 4352)     per-block sums of the loss reduction (kMseMaxBlocks doubles)
//   then, each 256-byte aligned:
//                   H   = ReLU(X W1)           B x H floats
//                   dZ1 = dH masked by H > 0   B x H floats
//                   E   = P - Y                B x O floats
//                   dP  = E * 2/(B*O)          B x O floats
// The error word and the counter must be zero when the step starts, so every
// call clears the first 256 bytes before its first launch.  Every element of
// the block sums, H, dZ1, E and dP is written before it is read within a
// call, so their stale contents from the previous call do not matter.  The
// step needs 4352 bytes plus 2*B*H + 2*B*O floats (each tensor rounded up to
// 256 bytes); shapes beyond the array are rejected with HX_ERR_UNSUPPORTED.
// GEMMs here never split K (split-K would need a partial-sum workspace), so a
// shape that the allocating step splits sums its K products in another order
// and may differ from it in the last bits.
//
// Set-up: the first call on a device looks up the array's device address
// with cudaGetSymbolAddress (with that device current; this also loads the
// library's device code on that device if nothing has yet) and caches it
// together with the identity of the device's current CUDA context.  A call
// that finds another context current (the old one was destroyed, for
// example by cudaDeviceReset, and the module was loaded again) repeats the
// set-up.  Make the first call on a device before capturing any stream.
//
// All calls on a device share the one array: two calls whose work overlaps
// on the GPU (different streams, or different runtimes on the same device)
// race on it.  Calls on one stream are ordered and safe.  The call waits
// for its own stream only (not for the caller's other streams) before it
// returns, so that a timed-out pipeline wait is reported by this call.
#include <cmath>
#include <mutex>

#include "gemm.cuh"
#include "plans.cuh"

namespace hx {
namespace {

constexpr size_t kNoallocScratchBytes = size_t(4) << 20;
constexpr size_t kNoallocCounterOffset = 64;
constexpr size_t kNoallocPartOffset = 256;
constexpr size_t kNoallocHeaderBytes = kNoallocPartOffset + sizeof(double) * kMseMaxBlocks;
static_assert(kNoallocHeaderBytes % 256 == 0, "tensors after the header start 256-byte aligned");

static __device__ __align__(256) unsigned char g_mlp_noalloc_scratch[kNoallocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
struct ScratchSetup {
    void* ptr = nullptr;
    unsigned long long context = 0;  // cuCtxGetId of the context the address belongs to
};
ScratchSetup g_scratch[kMaxDevices];

using CtxGetCurrentFn = CUresult (*)(CUcontext*);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long*);

template <class Fn>
Fn driver_fn(const char* name) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    check_cuda(cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q), name);
    require(q == cudaDriverEntryPointSuccess && p, HX_ERR_CUDA, std::string(name) + " unavailable");
    return reinterpret_cast<Fn>(p);
}

// Identity of the current context (unique for the life of the process).
unsigned long long current_context_id() {
    static const CtxGetCurrentFn get_current = driver_fn<CtxGetCurrentFn>("cuCtxGetCurrent");
    static const CtxGetIdFn get_id = driver_fn<CtxGetIdFn>("cuCtxGetId");
    CUcontext ctx = nullptr;
    require(get_current(&ctx) == CUDA_SUCCESS && ctx != nullptr, HX_ERR_CUDA, "no-alloc step: no current CUDA context");
    unsigned long long id = 0;
    require(get_id(ctx, &id) == CUDA_SUCCESS, HX_ERR_CUDA, "no-alloc step: cuCtxGetId failed");
    return id;
}

// Device address of the array on rt's device; the caller has made that
// device current (hx_guard does).  Looked up once per device and context.
unsigned char* scratch_on(hx_runtime* rt) {
    require(rt->device >= 0 && rt->device < kMaxDevices, HX_ERR_ARGUMENT, "no-alloc step: device index out of range");
    const unsigned long long ctx = current_context_id();
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    ScratchSetup& s = g_scratch[rt->device];
    if (!s.ptr || s.context != ctx) {
        void* addr = nullptr;
        check_cuda(cudaGetSymbolAddress(&addr, g_mlp_noalloc_scratch), "cudaGetSymbolAddress(no-alloc scratch)");
        require(addr != nullptr, HX_ERR_CUDA, "no-alloc step: scratch symbol has no device address");
        s.ptr = addr;
        s.context = ctx;
    }
    return static_cast<unsigned char*>(s.ptr);
}

size_t round256(size_t b) { return (b + 255) & ~size_t(255); }

// The three CUDA-core tile shapes gemm() in gemm.cuh chooses between.
template <int BM_, int BN_, int BK_, int TX_, int TY_>
struct SimtTile { static constexpr int BM = BM_, BN = BN_, BK = BK_, TX = TX_, TY = TY_; };
using Big = SimtTile<128, 128, 8, 16, 16>;
using Mid = SimtTile<64, 64, 16, 16, 16>;
using Small = SimtTile<32, 32, 32, 8, 8>;

// One GEMM with the epilogue applied to every element, never splitting K:
// the same kernels and tile choices as gemm() in gemm.cuh, minus the
// workspace.  `err` is the tensor-core kernels' error word.
template <bool AT, bool BT, class Epi>
void gemm_noalloc(hx_runtime* rt, int M, int N, int K, const float* A, long lda, const float* B, long ldb, Epi epi,
                  int* err)
{
    ProfScope prof(rt, kTagGemm, 2.0 * M * N * K, 4.0 * ((double)M * K + (double)K * N + (double)M * N));
    if (tc_eligible(rt, M, N, K, A, lda, B, ldb)) {
        constexpr bool A_MN = AT, B_MN = !BT;
        constexpr CUtensorMapSwizzle mn_swz = CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B;
        const CUtensorMap mx = A_MN ? make_map(A, M, K, lda, 32, 32, mn_swz) : make_map(A, K, M, lda, 32, kTcHalf);
        const CUtensorMap mw = B_MN ? make_map(B, N, K, ldb, 32, 32, mn_swz) : make_map(B, K, N, ldb, 32, kTcHalf);
        const int pairs = tc_pairs<A_MN, B_MN, false, false, Epi>(rt->sm_count);
        const TcGrid g = tc_grid(M, N, K, pairs, 1);
        HX_CUDA((launch_tc_kernel<A_MN, B_MN, false, false>(rt->stream, pairs, mx, mw, mw, mw, g, epi, nullptr, err)));
        ++rt->metrics.kernel_launches;
        return;
    }
    auto simt = [&](auto shape_tag) {
        using T = decltype(shape_tag);
        using S = SimtShape<T::BM, T::BN, T::BK, T::TX, T::TY>;
        const int chunk = K > 0 ? ((K + T::BK - 1) / T::BK) * T::BK : T::BK;
        dim3 grid((N + T::BN - 1) / T::BN, (M + T::BM - 1) / T::BM, 1);
        ::hx::pdl_launch(gemm_simt_kernel<S, T::BM, T::BN, T::BK, T::TX, T::TY, AT, BT, Epi>, grid, S::kThreads, 0, rt->stream, M, N, K, A, lda, B, ldb, chunk, epi, nullptr);
        HX_LAUNCHED(rt);
    };
    const long mn = (long)M * N;
    if (mn >= 128L * 128 * rt->sm_count / 2)
        simt(Big{});
    else if (mn >= 64L * 64 * rt->sm_count / 4)
        simt(Mid{});
    else
        simt(Small{});
}

}  // namespace
}  // namespace hx

using namespace hx;

extern "C" {

int hx_mlp_execute_device_noalloc(hx_runtime* rt, uint32_t B, uint32_t I, uint32_t H, uint32_t O, const float* x,
                                  const float* y, const float* w1, const float* w2, float lr, float* loss,
                                  float* w1_next, float* w2_next) {
    const auto t0 = Clock::now();
    const int rc = hx_guard(rt, [&] {
        require(B && I && H && O, HX_ERR_ARGUMENT, "no-alloc step: empty shape");
        require(x && y && w1 && w2 && loss && w1_next && w2_next, HX_ERR_ARGUMENT, "no-alloc step: null buffer");
        require(std::isfinite(lr), HX_ERR_ARGUMENT, "no-alloc step: learning rate must be finite");
        require(w1 != w1_next && w2 != w2_next, HX_ERR_ARGUMENT,
                "no-alloc step: next weights must not alias current weights");
        const uint64_t lim = uint64_t(1) << 31;
        require(uint64_t(B) * I < lim && uint64_t(I) * H < lim && uint64_t(B) * H < lim && uint64_t(H) * O < lim &&
                    uint64_t(B) * O < lim,
                HX_ERR_ARGUMENT, "no-alloc step: shape exceeds 2^31 elements per tensor");
        const size_t bh = round256(sizeof(float) * size_t(B) * H), bo = round256(sizeof(float) * size_t(B) * O);
        const size_t need = kNoallocHeaderBytes + 2 * bh + 2 * bo;
        require(need <= kNoallocScratchBytes, HX_ERR_UNSUPPORTED,
                "no-alloc step: B=" + std::to_string(B) + " H=" + std::to_string(H) + " O=" + std::to_string(O) +
                    " needs " + std::to_string(need) + " bytes of scratch (4352 + 2*B*H + 2*B*O floats), above the fixed " +
                    std::to_string(kNoallocScratchBytes) + "-byte array; use hx_mlp_prepare/hx_mlp_execute_device");
        unsigned char* s = scratch_on(rt);
        int* err = reinterpret_cast<int*>(s);
        unsigned int* done = reinterpret_cast<unsigned int*>(s + kNoallocCounterOffset);
        double* part = reinterpret_cast<double*>(s + kNoallocPartOffset);
        float* h = reinterpret_cast<float*>(s + kNoallocHeaderBytes);
        float* dz1 = reinterpret_cast<float*>(s + kNoallocHeaderBytes + bh);
        float* e = reinterpret_cast<float*>(s + kNoallocHeaderBytes + 2 * bh);
        float* dp = reinterpret_cast<float*>(s + kNoallocHeaderBytes + 2 * bh + bo);
        HX_CUDA(cudaMemsetAsync(s, 0, kNoallocPartOffset, rt->stream));  // error word and block counter

        const int b = (int)B, i = (int)I, hd = (int)H, o = (int)O;
        const float scale = 2.0f / float(b * o);
        gemm_noalloc<false, false>(rt, b, hd, i, x, i, w1, hd, EpiRelu{h, nullptr, hd}, err);
        gemm_noalloc<false, false>(rt, b, o, hd, h, hd, w2, o, EpiError{y, nullptr, e, dp, scale, o}, err);
        {
            ProfScope prof(rt, kTagReduce, 2.0 * b * o, 4.0 * b * o);
            launch_mse_reduce(rt, e, size_t(b) * o, part, done, loss);
        }
        gemm_noalloc<true, false>(rt, hd, o, b, h, hd, dp, o, EpiSgd{w2, nullptr, w2_next, lr, o}, err);
        gemm_noalloc<false, true>(rt, b, hd, o, dp, o, w2, o, EpiReluBackward{h, dz1, nullptr, hd}, err);
        gemm_noalloc<true, false>(rt, i, hd, b, x, i, dz1, hd, EpiSgd{w1, nullptr, w1_next, lr, hd}, err);

        // Finish here so that a timed-out pipeline wait is reported by this
        // call rather than left in the shared array for the next one.  The
        // read-back is ordered on this runtime's stream only.
        int code = 0;
        HX_CUDA(cudaMemcpyAsync(&code, err, sizeof(int), cudaMemcpyDeviceToHost, rt->stream));
        HX_CUDA(cudaStreamSynchronize(rt->stream));
        if (code)
            fail(HX_ERR_CUDA, "DEVICE_WAIT_TIMEOUT: a bounded pipeline wait in the tensor-core GEMM gave up (role " +
                                  std::to_string(code) + "); results of this call are invalid");
    });
    if (rt) rt->record_execute(rc == HX_OK, us_since(t0));
    return rc;
}

}  // extern "C"
