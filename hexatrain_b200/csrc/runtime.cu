// runtime.cu -- runtime lifecycle: device binding, stream, metrics, errors.
//
// Replaces the reference's QAIRT adapter initialisation
// (qnn/qnn_runtime_qairt.cpp:709-972 Runtime::initialize): instead of loading
// a backend library and creating backend/device/context handles, a runtime
// binds one CUDA device and owns one non-blocking stream.  Plans (MLP, LM,
// Adam) hold their device memory from prepare until destroy.
#include <cstdio>

#include "plans.cuh"
#include "tc_ptx.cuh"

hx_runtime::~hx_runtime() {
    cudaSetDevice(device);
    mlp.reset();
    lm.reset();
    adam.reset();
    momentum.reset();
    scratch.release();
    side_scratch.release();
    if (side_stream) cudaStreamDestroy(side_stream);
    if (own_stream) cudaStreamDestroy(own_stream);
}

namespace {
// One thread waits, with the bounded wait of the tensor-core kernels, on an
// mbarrier that nothing arrives at; when the wait gives up it records the
// self-test code in the error word the way those kernels record theirs.
// Nothing else is in flight in this block (no TMA copy, no MMA, no TMEM).
__global__ void wait_timeout_probe_kernel(long long limit, int* err)
{
    HX_PDL_PROLOGUE();
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x == 0) {
        hx::tc::mbar_init(&bar, 1);
        hx::tc::fence_mbar_init();
        if (!hx::tc::mbar_wait(&bar, 0, limit)) atomicCAS(err, 0, hx::kWaitProbeCode);
    }
}

void write_err(char* err, size_t len, const std::string& msg) {
    if (err && len) {
        std::snprintf(err, len, "%s", msg.c_str());
    }
}
}  // namespace

extern "C" {

int hx_runtime_create(int device, hx_runtime** out, char* err, size_t err_len) {
    if (!out) {
        write_err(err, err_len, "hx_runtime_create: null output pointer");
        return HX_ERR_ARGUMENT;
    }
    *out = nullptr;
    int count = 0;
    cudaError_t e = cudaGetDeviceCount(&count);
    if (e != cudaSuccess || count == 0) {
        write_err(err, err_len, std::string("CUDA_DEVICE_NOT_FOUND: cannot initialize runtime: ") +
                                    (e != cudaSuccess ? cudaGetErrorString(e) : "no CUDA device"));
        return HX_ERR_CUDA;
    }
    if (device < 0 || device >= count) {
        write_err(err, err_len, "CUDA_DEVICE_NOT_FOUND: device index " + std::to_string(device) + " out of range");
        return HX_ERR_ARGUMENT;
    }
    cudaDeviceProp prop{};
    if ((e = cudaGetDeviceProperties(&prop, device)) != cudaSuccess) {
        write_err(err, err_len, std::string("cudaGetDeviceProperties: ") + cudaGetErrorString(e));
        return HX_ERR_CUDA;
    }
    if (prop.major != 10) {
        write_err(err, err_len, "UNSUPPORTED_DEVICE: built for sm_100a (B200); device " + std::to_string(device) +
                                    " is sm_" + std::to_string(prop.major) + std::to_string(prop.minor));
        return HX_ERR_UNSUPPORTED;
    }
    auto* rt = new (std::nothrow) hx_runtime();
    if (!rt) return HX_ERR_MEMORY;
    rt->device = device;
    rt->sm_count = prop.multiProcessorCount;
    rt->metrics.first_failure_call = -1;
    if ((e = cudaSetDevice(device)) != cudaSuccess ||
        (e = cudaStreamCreateWithFlags(&rt->own_stream, cudaStreamNonBlocking)) != cudaSuccess) {
        write_err(err, err_len, std::string("cudaStreamCreate: ") + cudaGetErrorString(e));
        delete rt;
        return HX_ERR_CUDA;
    }
    rt->stream = rt->own_stream;
    *out = rt;
    write_err(err, err_len, "");
    return HX_OK;
}

void hx_runtime_destroy(hx_runtime* rt) { delete rt; }

const char* hx_runtime_last_error(const hx_runtime* rt) { return rt ? rt->last_error.c_str() : "null runtime"; }

int hx_runtime_set_stream(hx_runtime* rt, void* stream) {
    return hx_guard(rt, [&] { rt->stream = stream ? static_cast<cudaStream_t>(stream) : rt->own_stream; });
}

void* hx_runtime_stream(const hx_runtime* rt) { return rt ? static_cast<void*>(rt->stream) : nullptr; }

int hx_runtime_synchronize(hx_runtime* rt) {
    return hx_guard(rt, [&] { rt->check_device_error(); });
}

int hx_runtime_set_gemm_backend(hx_runtime* rt, int backend) {
    return hx_guard(rt, [&] {
        hx::require(backend == HX_GEMM_AUTO || backend == HX_GEMM_CUDA_CORES || backend == HX_GEMM_TENSOR_CORES,
                    HX_ERR_ARGUMENT, "unknown GEMM backend");
        if (rt->gemm_backend != backend) ++rt->graph_epoch;
        rt->gemm_backend = backend;
    });
}

int hx_runtime_set_attention_backend(hx_runtime* rt, int backend) {
    return hx_guard(rt, [&] {
        hx::require(backend == HX_ATTN_AUTO || backend == HX_ATTN_CUDA_CORES, HX_ERR_ARGUMENT,
                    "unknown attention backend");
        if (rt->attention_backend != backend) ++rt->graph_epoch;
        rt->attention_backend = backend;
    });
}

int hx_runtime_metrics(const hx_runtime* rt, hx_metrics* out) {
    if (!rt || !out) return HX_ERR_ARGUMENT;
    *out = rt->metrics;
    out->device_bytes = rt->scratch.bytes + rt->side_scratch.bytes + hx::plan_device_bytes(rt);
    return HX_OK;
}

int hx_runtime_profile(hx_runtime* rt, int enable) {
    return hx_guard(rt, [&] {
        rt->prof.on = enable != 0;
        rt->prof.recs.clear();
        rt->prof.used = 0;
    });
}

int hx_runtime_profile_read(hx_runtime* rt, hx_profile_entry* entries, int capacity, int* count) {
    return hx_guard(rt, [&] {
        hx::require(entries && count && capacity >= 0, HX_ERR_ARGUMENT, "profile_read: null output");
        HX_CUDA(cudaStreamSynchronize(rt->stream));
        hx_profile_entry agg[hx::kTagCount];
        std::memset(agg, 0, sizeof(agg));
        for (int t = 0; t < hx::kTagCount; ++t) std::snprintf(agg[t].name, sizeof(agg[t].name), "%s", hx::prof_tag_name(t));
        for (const auto& r : rt->prof.recs) {
            float ms = 0.f;
            HX_CUDA(cudaEventElapsedTime(&ms, r.a, r.b));
            hx_profile_entry& e = agg[r.tag];
            ++e.launches;
            e.total_ms += ms;
            e.flops += r.flops;
            e.bytes += r.bytes;
        }
        rt->prof.recs.clear();
        rt->prof.used = 0;
        int n = 0;
        for (int t = 0; t < hx::kTagCount && n < capacity; ++t)
            if (agg[t].launches) entries[n++] = agg[t];
        *count = n;
    });
}

int hx_runtime_check_wait_timeout(hx_runtime* rt, long long cycles) {
    return hx_guard(rt, [&] {
        hx::require(cycles > 0 && cycles <= 4000000000LL, HX_ERR_ARGUMENT,
                    "wait self-test: cycles must be in (0, 4e9]");
        ::hx::pdl_launch(wait_timeout_probe_kernel, 1, 32, 0, rt->stream, cycles, rt->device_error());
        HX_LAUNCHED(rt);
        rt->check_device_error();
    });
}

int hx_runtime_inject_execute_failure(hx_runtime* rt, int64_t call_index) {
    return hx_guard(rt, [&] { rt->inject_execute_at = call_index; });
}

}  // extern "C"
