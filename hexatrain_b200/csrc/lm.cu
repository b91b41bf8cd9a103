// lm.cu -- tiny causal Transformer LM training step on B200.
//
// Replaces the generalized L-layer/H-head QNN training graph
// (qnn/qnn_runtime_transformer_training_generalized.inc:4-1260 and its
// execute companion) and the batched Adam driver loop
// (qnn/qnn_transformer_training.cpp:7281-7345).  The reference runs one
// sequence per graph execute and accumulates grad*(1/B) on the host; here the
// B sequences of a step share every kernel (rows r = b*T + t) and the 1/B is
// folded into dlogits, so the weight-gradient GEMMs sum over all B*T rows.
//
// Per layer (pre-LN, no biases, untied head, no final LN -- :44-48):
//   LN1 -> [q|k|v] = n1 W_qkv -> causal attention -> r1 = x + ctx Wo
//   LN2 -> relu = ReLU(n2 W1) -> out = r1 + relu W2
// Backward mirrors :79-82 with the same named gradients in registry order.
#include <cmath>

#include "attention_tc.cuh"
#include "attention_tc_bwd.cuh"
#include "attention_tiled.cuh"
#include "gemm.cuh"
#include "lm_kernels.cuh"
#include "optim.cuh"
#include "plans.cuh"

namespace hx {

AdamScalars adam_scalars(float lr, float gradient_scale, float c1, float c2);
void launch_adam(hx_runtime* rt, bool graph_order, size_t n, const float* w, const float* g, const float* m,
                 const float* v, float* wn, float* mn, float* vn, const AdamScalars& s, const AdamTaps& t,
                 const float* scale_dev = nullptr, const AdamScalars* s_dev = nullptr);
void launch_momentum(hx_runtime* rt, size_t n, const float* w, const float* g, const float* vel, float* wn,
                     float* veln, float lr, float momentum, const float* lr_dev = nullptr);
void launch_clip_scale(hx_runtime* rt, const float* g, const GradTensor* tensors, int count, double* sumsq,
                       float threshold, double* norm_out, float* scale_out);
size_t muon_smem_bytes(int rows, int cols);
void check_muon_shape(int rows, int cols);
void launch_muon(hx_runtime* rt, const MuonMatrix* d_mats, int count, size_t smem, const MuonScalars& s,
                 const float* lr_dev = nullptr, bool tc_shapes = false);
bool muon_tc_shape(int rows, int cols);

struct LayerOffsets {  // offsets (in floats) of one layer's tensors in the flat registry
    size_t g1, b1, wq, wk, wv, wo, g2, b2, w1, w2;
};

struct LayerActs {  // arena offsets (bytes)
    size_t x, n1, mean1, inv1, qkv, ctx, r1, n2, mean2, inv2, relu, rmax, rsum;
};

struct LmPlan {
    hx_lm_config cfg{};
    uint32_t B = 0, V = 0, T = 0, D = 0, F = 0, L = 0, H = 0, dh = 0;
    int M = 0;
    bool diag = false, learned = false;
    size_t P = 0;
    size_t off_E = 0, off_pos = 0, off_out = 0;
    std::vector<LayerOffsets> lo;
    Arena arena;
    // arena offsets (bytes)
    size_t params, exec_params, grads, adam_m, adam_v, muon_buf, pos_fixed, wqkv;
    size_t w_hi, w_lo, wqkv_hi, wqkv_lo;  // TF32 hi/lo splits of the GEMM weights, refreshed every forward
    size_t tokens, in_tok, tgt_tok, in_ids, tgt_ids, bad;
    std::vector<LayerActs> la;
    size_t xL, logits, probs, row_loss, row_correct, seq_loss, seq_correct, loss, acc, scalars;
    size_t dout, dr, dc, dn, df1, dqkv, ln_part;
    size_t attn_bstat;  // tensor-core attention backward: per (sequence, head, row) sum and D
    size_t diag_lig, diag_hp, diag_dout;
    size_t muon_table;
    int ln_parts = 0, ln_rows = 0;
    int emb_chunks = 1, emb_rows = 1;
    size_t emb_part = 0;
    DeviceBuffer onehot;  // lazily sized staging for the one-hot execute API
    hx_optimizer_config opt{};
    int muon_count = 0;
    size_t muon_smem = 0;
    std::vector<std::pair<size_t, size_t>> adam_segments;  // [offset, count) in floats
    // training-stability modes (training_stability.h) and global-norm clip
    uint32_t stab_mode = 0, stab_total = 0;
    float clip_threshold = 0.f;        // > 0: clip the gradient to this global norm before Adam
    int norm_count = 0;                // tensors in the gradient-norm table
    size_t norm_table = 0, norm_sumsq = 0, norm_value = 0, clip_scale = 0;
    bool state_ready = false;
    // Captured step graphs (train step, forward+backward, optimizer step).
    GraphCache graphs;
    // Fork/join events of the backward's second stream (weight gradients).
    static constexpr int kForkEvents = 64;
    cudaEvent_t fork_ev[kForkEvents] = {};
    // Gradient buckets in completion order and their events.
    std::vector<std::pair<size_t, size_t>> buckets;  // [offset, count) in floats
    std::vector<cudaEvent_t> bucket_ev;
    bool bucket_events = false;
    // Per-step optimizer scalars: host values go through a ring of pinned
    // slots into step_scalars (device), which the optimizer kernels read.  A
    // slot is rewritten only after the copy that last read it has run.
    static constexpr int kRing = 16;
    size_t step_scalars = 0;
    LmStepScalars* ring = nullptr;
    cudaEvent_t ring_ev[kRing] = {};
    bool ring_live[kRing] = {};
    unsigned ring_next = 0;
    ~LmPlan() {
        graphs.clear();
        for (cudaEvent_t e : fork_ev)
            if (e) cudaEventDestroy(e);
        for (cudaEvent_t e : bucket_ev)
            if (e) cudaEventDestroy(e);
        for (cudaEvent_t e : ring_ev)
            if (e) cudaEventDestroy(e);
        if (ring) cudaFreeHost(ring);
    }
};

size_t lm_plan_bytes(const LmPlan* p) { return p ? p->arena.block.bytes + p->onehot.bytes : 0; }

bool lm_prepared_config(const hx_runtime* rt, hx_lm_config* cfg, uint32_t* optimizer_kind) {
    if (!rt || !rt->lm) return false;
    if (cfg) *cfg = rt->lm->cfg;
    if (optimizer_kind) *optimizer_kind = rt->lm->opt.kind;
    return true;
}
void LmPlanDeleter::operator()(LmPlan* p) const { delete p; }

namespace {

void validate(const hx_lm_config* c) {
    require(c != nullptr, HX_ERR_ARGUMENT, "APP_CONFIGURATION_VALIDATION: null configuration");
    require(c->vocab && c->tokens && c->dim && c->ffn && c->layers && c->heads, HX_ERR_ARGUMENT,
            "APP_CONFIGURATION_VALIDATION: all Transformer dimensions and counts must be >= 1");
    require(c->dim % c->heads == 0, HX_ERR_ARGUMENT,
            "APP_CONFIGURATION_VALIDATION: embeddingDimension must be divisible by numHeads");
    require(std::isfinite(c->eps) && c->eps > 0.f, HX_ERR_ARGUMENT,
            "APP_CONFIGURATION_VALIDATION: LayerNorm epsilon must be finite and positive");
    require((c->flags & ~uint32_t(HX_LM_LEARNED_POSITION)) == 0, HX_ERR_ARGUMENT,
            "APP_CONFIGURATION_VALIDATION: unknown flag bits");
    const uint64_t lim = uint64_t(1) << 31;
    require(uint64_t(c->vocab) * c->dim < lim && uint64_t(c->dim) * c->ffn < lim && uint64_t(c->tokens) * c->tokens < lim &&
                c->layers <= 4096,
            HX_ERR_ARGUMENT, "APP_RESOURCE_ESTIMATOR: dimension product exceeds 2^31 elements");
}

size_t param_count(const hx_lm_config* c) {
    const size_t V = c->vocab, T = c->tokens, D = c->dim, F = c->ffn;
    return 2 * V * D + ((c->flags & HX_LM_LEARNED_POSITION) ? T * D : 0) + size_t(c->layers) * (4 * D * D + 4 * D + 2 * D * F);
}

bool dh_supported(uint32_t dh) {
    switch (dh) {
        case 1: case 2: case 3: case 4: case 6: case 8: case 12: case 16: case 24: case 32: case 48: case 64:
            return true;
        default:
            return false;
    }
}

size_t attn_fwd_smem(int T, int DH, int nw) { return sizeof(float) * (size_t(2) * T * (DH + 1) + size_t(nw) * T + size_t(nw) * DH); }
size_t attn_bwd_smem(int T, int DH, int nw) { return sizeof(float) * (size_t(4) * T * (DH + 1) + 3 * size_t(T) + size_t(nw) * T); }
constexpr int kAttnThreads = 256;

bool attn_tiled(int T, int DH) { return T <= kAttnMaxT && (DH == 8 || DH == 16 || DH == 32); }

// Tensor-core attention: head dimension 32, T <= 256, no probability
// output, 16-byte aligned rows (the model width is a multiple of 32).
bool attn_tc(hx_runtime* rt, int T, int DH, const float* probs) {
    return rt->attention_backend == HX_ATTN_AUTO && DH == kAtcDH && T <= kAtcMaxT && !probs;
}

void attn_fwd_tc_launch(hx_runtime* rt, const LmPlan& p, const float* qkv, float* ctx, float* rmax, float* rsum) {
    const uint64_t rows = uint64_t(p.B) * p.T, w = 3 * uint64_t(p.D);
    const CUtensorMap mqk = make_map(qkv, w, rows, w, 32, kAtcTile);
    const CUtensorMap mv = make_map(qkv, w, rows, w, 32, kAtcTile, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B);
    HX_CUDA(cudaFuncSetAttribute(attention_fwd_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)kAtcFwdSmemBytes));
    ::hx::pdl_launch(attention_fwd_tc_kernel, dim3(p.H, p.B), kAtcFwdThreads, kAtcFwdSmemBytes, rt->stream, 
        mqk, mv, p.T, p.D, p.H, 1.0f / sqrtf((float)kAtcDH), qkv, ctx, rmax, rsum, rt->device_error());
    HX_LAUNCHED(rt);
}

template <int DH>
void attn_fwd_launch(hx_runtime* rt, const LmPlan& p, const float* qkv, float* ctx, float* rmax, float* rsum, float* probs) {
    const double pairs = double(p.B) * p.H * (double(p.T) * (p.T + 1) / 2);
    ProfScope prof(rt, kTagAttnFwd, 4.0 * pairs * DH, 4.0 * (double(p.M) * 4 * p.D + 2.0 * p.B * p.H * p.T));
    if (attn_tc(rt, p.T, DH, probs)) {
        attn_fwd_tc_launch(rt, p, qkv, ctx, rmax, rsum);
        return;
    }
    if constexpr (DH == 8 || DH == 16 || DH == 32) {
        if (attn_tiled(p.T, DH)) {
            const size_t smem = AttnTiledLayout<DH>::fwd_bytes(p.T);
            HX_CUDA(cudaFuncSetAttribute(attention_fwd_tiled_kernel<DH>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
            ::hx::pdl_launch(attention_fwd_tiled_kernel<DH>, dim3(p.H, p.B), kAttnTiledThreads, smem, rt->stream, 
                p.T, p.D, p.H, 1.0f / sqrtf((float)DH), qkv, ctx, rmax, rsum, probs);
            HX_LAUNCHED(rt);
            return;
        }
    }
    const size_t smem = attn_fwd_smem(p.T, DH, kAttnThreads / 32);
    HX_CUDA(cudaFuncSetAttribute(attention_fwd_kernel<DH>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    ::hx::pdl_launch(attention_fwd_kernel<DH>, dim3(p.H, p.B), kAttnThreads, smem, rt->stream, 
        p.T, p.D, p.H, 1.0f / sqrtf((float)DH), qkv, ctx, rmax, rsum, probs);
    HX_LAUNCHED(rt);
}
// dQ kernel (queries on lanes, writes the backward's row statistics), then
// the dK/dV kernel (keys on lanes, one CTA per 128-key block).
void attn_bwd_tc_launch(hx_runtime* rt, const LmPlan& p, const float* qkv, const float* dctx, const float* rmax,
                        float* dqkv) {
    const uint64_t rows = uint64_t(p.B) * p.T, w = 3 * uint64_t(p.D);
    constexpr CUtensorMapSwizzle mn = CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B;
    const CUtensorMap mqk = make_map(qkv, w, rows, w, 32, kAtcTile);
    const CUtensorMap mmn = make_map(qkv, w, rows, w, 32, kAtcTile, mn);
    const CUtensorMap mdo = make_map(dctx, p.D, rows, p.D, 32, kAtcTile);
    const CUtensorMap mdo_mn = make_map(dctx, p.D, rows, p.D, 32, kAtcTile, mn);
    float* bstat = p.arena.at<float>(p.attn_bstat);
    const float scale = 1.0f / sqrtf((float)kAtcDH);
    HX_CUDA(cudaFuncSetAttribute(attention_bwd_dq_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)kAtcDqSmemBytes));
    ::hx::pdl_launch(attention_bwd_dq_tc_kernel, dim3(p.H, p.B), kAtcDqThreads, kAtcDqSmemBytes, rt->stream, 
        mqk, mmn, p.T, p.D, p.H, scale, qkv, dctx, rmax, bstat, dqkv, rt->device_error());
    HX_LAUNCHED(rt);
    HX_CUDA(cudaFuncSetAttribute(attention_bwd_dkdv_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)kAtcKvSmemBytes));
    const int ntile = p.T > uint32_t(kAtcTile) ? 2 : 1;
    ::hx::pdl_launch(attention_bwd_dkdv_tc_kernel, dim3(p.H, p.B, ntile), kAtcKvThreads, kAtcKvSmemBytes, rt->stream, 
        mqk, mmn, mdo, mdo_mn, p.T, p.D, p.H, scale, qkv, dctx, rmax, bstat, dqkv, rt->device_error());
    HX_LAUNCHED(rt);
}

template <int DH>
void attn_bwd_launch(hx_runtime* rt, const LmPlan& p, const float* qkv, const float* dctx, const float* rmax,
                     const float* rsum, float* dqkv) {
    const double pairs = double(p.B) * p.H * (double(p.T) * (p.T + 1) / 2);
    ProfScope prof(rt, kTagAttnBwd, 8.0 * pairs * DH, 4.0 * (double(p.M) * 6 * p.D + 2.0 * p.B * p.H * p.T));
    if (attn_tc(rt, p.T, DH, nullptr)) {
        attn_bwd_tc_launch(rt, p, qkv, dctx, rmax, dqkv);
        return;
    }
    if constexpr (DH == 8 || DH == 16 || DH == 32) {
        if (attn_tiled(p.T, DH)) {
            const size_t smem = AttnTiledLayout<DH>::bwd_bytes(p.T);
            HX_CUDA(cudaFuncSetAttribute(attention_bwd_tiled_kernel<DH>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
            ::hx::pdl_launch(attention_bwd_tiled_kernel<DH>, dim3(p.H, p.B), kAttnTiledThreads, smem, rt->stream, 
                p.T, p.D, p.H, 1.0f / sqrtf((float)DH), qkv, dctx, rmax, dqkv);
            HX_LAUNCHED(rt);
            return;
        }
    }
    const size_t smem = attn_bwd_smem(p.T, DH, kAttnThreads / 32);
    HX_CUDA(cudaFuncSetAttribute(attention_bwd_kernel<DH>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    ::hx::pdl_launch(attention_bwd_kernel<DH>, dim3(p.H, p.B), kAttnThreads, smem, rt->stream, 
        p.T, p.D, p.H, 1.0f / sqrtf((float)DH), qkv, dctx, rmax, rsum, dqkv);
    HX_LAUNCHED(rt);
}

#define HX_DH_DISPATCH(dh, FN, ...)                                   \
    switch (dh) {                                                     \
        case 1: FN<1>(__VA_ARGS__); break;                            \
        case 2: FN<2>(__VA_ARGS__); break;                            \
        case 3: FN<3>(__VA_ARGS__); break;                            \
        case 4: FN<4>(__VA_ARGS__); break;                            \
        case 6: FN<6>(__VA_ARGS__); break;                            \
        case 8: FN<8>(__VA_ARGS__); break;                            \
        case 12: FN<12>(__VA_ARGS__); break;                          \
        case 16: FN<16>(__VA_ARGS__); break;                          \
        case 24: FN<24>(__VA_ARGS__); break;                          \
        case 32: FN<32>(__VA_ARGS__); break;                          \
        case 48: FN<48>(__VA_ARGS__); break;                          \
        case 64: FN<64>(__VA_ARGS__); break;                          \
        default: fail(HX_ERR_UNSUPPORTED, "unsupported head dimension"); \
    }

int grid_for(long work, int threads, int sms) {
    return (int)std::max<long>(1, std::min<long>((work + threads - 1) / threads, long(sms) * 32));
}

bool aligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0; }

struct DiagOut {
    bool on = false;
};

// Forward + backward over the ids already in the plan.  grads[0..P) receive
// sum over rows of the gradient with dlogits scaled by grad_scale;
// grads[P] receives sum_b loss_b * grad_scale.
// Forward-only variants (executeTinyTransformerForwardOnly): stop after the
// output projection; kHeadLastRow projects only each sequence's last row
// into logits [B][V] (what generation samples from).
enum ForwardMode { kFullStep = 0, kForwardAllRows = 1, kForwardLastRow = 2 };

// hi = w rounded to TF32, lo = w - hi: the tensor-core GEMMs' split of their
// weight operands, done once per forward instead of in every CTA per tile.
__global__ void split_tf32_kernel(long n, const float* __restrict__ w, float* __restrict__ hi, float* __restrict__ lo)
{
    HX_PDL_PROLOGUE();
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
        const float x = w[i];
        const float h = tf32_round(x);
        hi[i] = h;
        lo[i] = x - h;
    }
}

// The backward's weight-gradient GEMMs run on the runtime's second stream,
// beside the main stream's input-gradient GEMMs and attention: both kinds
// are persistent or many-CTA kernels that fill the GPU, so each fills the
// other's last, partial wave.  fork() lets the side stream start after the
// main stream's work so far; join() makes the main stream wait for all side
// work so far.  With the event profiler on, everything stays on the main
// stream (the profile then times each launch alone).
struct SideStream {
    hx_runtime* rt;
    LmPlan& p;
    bool on;
    int k = 0;
    SideStream(hx_runtime* r, LmPlan& plan) : rt(r), p(plan), on(!r->prof.on && r->side_stream != nullptr) {}
    // Events are reused cyclically: a wait takes the event's state when it is
    // enqueued, so a later record of the same event does not affect it.
    cudaEvent_t next() { return p.fork_ev[k++ % LmPlan::kForkEvents]; }
    void fork() {
        if (!on) return;
        cudaEvent_t e = next();
        HX_CUDA(cudaEventRecord(e, rt->stream));
        HX_CUDA(cudaStreamWaitEvent(rt->side_stream, e, 0));
    }
    void join() {
        if (!on) return;
        cudaEvent_t e = next();
        HX_CUDA(cudaEventRecord(e, rt->side_stream));
        HX_CUDA(cudaStreamWaitEvent(rt->stream, e, 0));
    }
    // Runs f's launches on the side stream (on the main one when off).
    template <class F>
    void run(F&& f) {
        if (!on) {
            f();
            return;
        }
        cudaStream_t main = rt->stream;
        rt->stream = rt->side_stream;
        try {
            f();
        } catch (...) {
            rt->stream = main;
            throw;
        }
        rt->stream = main;
    }
};

// Records bucket i's event on `stream` when bucket events are on; an external
// event node when the stream is being captured, so that waits outside the
// graph see each replay's record.
void record_bucket(hx_runtime* rt, LmPlan& p, int i, cudaStream_t stream)
{
    if (!p.bucket_events) return;
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    HX_CUDA(cudaStreamIsCapturing(stream, &cs));
    if (cs == cudaStreamCaptureStatusActive)
        HX_CUDA(cudaEventRecordWithFlags(p.bucket_ev[size_t(i)], stream, cudaEventRecordExternal));
    else
        HX_CUDA(cudaEventRecord(p.bucket_ev[size_t(i)], stream));
}

void forward_backward(hx_runtime* rt, LmPlan& p, const float* W, float* G, float grad_scale, int mode = kFullStep)
{
    const Arena& a = p.arena;
    const int M = p.M, T = p.T, D = p.D, F = p.F, V = p.V, B = p.B;
    const cudaStream_t s = rt->stream;
    const int* in_ids = a.at<int>(p.in_ids);
    const int* tgt_ids = a.at<int>(p.tgt_ids);
    const float* pos = p.learned ? W + p.off_pos : a.at<float>(p.pos_fixed);
    float* wqkv = a.at<float>(p.wqkv);
    const int tpb = 256;

    // pack W_qkv per layer; split the GEMM weights for the tensor cores
    for (uint32_t l = 0; l < p.L; ++l) {
        ::hx::pdl_launch(pack_qkv_kernel, grid_for(3L * D * D, tpb, rt->sm_count), tpb, 0, s, D, W + p.lo[l].wq, wqkv + size_t(l) * 3 * D * D);
        HX_LAUNCHED(rt);
    }
    float* whi = a.at<float>(p.w_hi);
    float* wlo = a.at<float>(p.w_lo);
    float* qhi = a.at<float>(p.wqkv_hi);
    float* qlo = a.at<float>(p.wqkv_lo);
    {
        const long nq = long(p.L) * 3 * D * D;
        ::hx::pdl_launch(split_tf32_kernel, grid_for(long(p.P), tpb, rt->sm_count), tpb, 0, s, long(p.P), W, whi, wlo);
        HX_LAUNCHED(rt);
        ::hx::pdl_launch(split_tf32_kernel, grid_for(nq, tpb, rt->sm_count), tpb, 0, s, nq, wqkv, qhi, qlo);
        HX_LAUNCHED(rt);
    }
    auto wsplit = [&](size_t off) { return BSplit{whi + off, wlo + off}; };
    auto qsplit = [&](uint32_t l) { return BSplit{qhi + size_t(l) * 3 * D * D, qlo + size_t(l) * 3 * D * D}; };
    // embedding
    float* x = a.at<float>(p.la[0].x);
    ProfScope pemb(rt, kTagEmbed, 1.0 * M * D, 4.0 * 3.0 * M * D);
    if (D % 4 == 0 && long(M) * D / 4 < (1L << 31) && aligned16(W + p.off_E) && aligned16(pos) && aligned16(x)) {
        const int D4 = D / 4;
        ::hx::pdl_launch(embed_vec_kernel, grid_for(long(M) * D4, tpb, rt->sm_count), tpb, 0, s, 
            M, T, D4, in_ids, reinterpret_cast<const float4*>(W + p.off_E), reinterpret_cast<const float4*>(pos),
            reinterpret_cast<float4*>(x));
    } else {
        ::hx::pdl_launch(embed_kernel, grid_for(long(M) * D, tpb, rt->sm_count), tpb, 0, s, M, T, D, in_ids, W + p.off_E, pos, x);
    }
    HX_LAUNCHED(rt);
        pemb.end();
    const int rows_per_block = 8;  // warps per block for row kernels
    const int row_grid = (M + rows_per_block - 1) / rows_per_block;
    // LayerNorm forward: the row-in-registers kernel when D = 128, 256 or 512
    // and every row pointer is 16-byte aligned, else the scalar kernel
    auto ln_fwd = [&](const float* xx, const float* gam, const float* bet, float* yy, float* mo, float* io) {
        const int C = (D % 128 == 0) ? D / 128 : 0;
        const bool al = ((reinterpret_cast<uintptr_t>(xx) | reinterpret_cast<uintptr_t>(gam) |
                          reinterpret_cast<uintptr_t>(bet) | reinterpret_cast<uintptr_t>(yy)) & 15) == 0;
        if (al && (C == 1 || C == 2 || C == 4)) {
            auto k = C == 1 ? layernorm_fwd_vec_kernel<1> : C == 2 ? layernorm_fwd_vec_kernel<2> : layernorm_fwd_vec_kernel<4>;
            ::hx::pdl_launch(k, row_grid, 32 * rows_per_block, 0, s, M, p.cfg.eps, xx, gam, bet, yy, mo, io);
        } else {
            ::hx::pdl_launch(layernorm_fwd_kernel, row_grid, 32 * rows_per_block, 0, s, M, D, p.cfg.eps, xx, gam, bet, yy, mo, io);
        }
        HX_LAUNCHED(rt);
    };

    for (uint32_t l = 0; l < p.L; ++l) {
        const LayerActs& A = p.la[l];
        const LayerOffsets& o = p.lo[l];
        const float* xin = a.at<float>(A.x);
        float* xout = (l + 1 < p.L) ? a.at<float>(p.la[l + 1].x) : a.at<float>(p.xL);
        ProfScope pln1(rt, kTagLayerNorm, 8.0 * M * D, 4.0 * (2.0 * M * D + 2.0 * M));
        ln_fwd(xin, W + o.g1, W + o.b1, a.at<float>(A.n1), a.at<float>(A.mean1), a.at<float>(A.inv1));
        pln1.end();
        gemm<false, false>(rt, M, 3 * D, D, a.at<float>(A.n1), D, wqkv + size_t(l) * 3 * D * D, 3 * D,
                           EpiStore{a.at<float>(A.qkv), 3L * D, 0, 0}, qsplit(l));
        float* hp = p.diag ? a.at<float>(p.diag_hp) + size_t(l) * B * p.H * T * T : nullptr;
        HX_DH_DISPATCH(p.dh, attn_fwd_launch, rt, p, a.at<float>(A.qkv), a.at<float>(A.ctx), a.at<float>(A.rmax),
                       a.at<float>(A.rsum), hp);
        gemm<false, false>(rt, M, D, D, a.at<float>(A.ctx), D, W + o.wo, D, EpiAddResidual{xin, a.at<float>(A.r1), D},
                           wsplit(o.wo));
        ProfScope pln2(rt, kTagLayerNorm, 8.0 * M * D, 4.0 * (2.0 * M * D + 2.0 * M));
        ln_fwd(a.at<float>(A.r1), W + o.g2, W + o.b2, a.at<float>(A.n2), a.at<float>(A.mean2), a.at<float>(A.inv2));
        pln2.end();
        gemm<false, false>(rt, M, F, D, a.at<float>(A.n2), D, W + o.w1, F, EpiRelu{a.at<float>(A.relu), nullptr, F},
                           wsplit(o.w1));
        gemm<false, false>(rt, M, D, F, a.at<float>(A.relu), F, W + o.w2, D,
                           EpiAddResidual{a.at<float>(A.r1), xout, D}, wsplit(o.w2));
    }
    const float* xL = a.at<float>(p.xL);
    float* logits = a.at<float>(p.logits);
    if (mode == kForwardLastRow) {
        gemm<false, false>(rt, B, V, D, xL + size_t(T - 1) * D, (long)T * D, W + p.off_out, V,
                           EpiStore{logits, (long)V, 0, 0}, wsplit(p.off_out));
        return;
    }
    gemm<false, false>(rt, M, V, D, xL, D, W + p.off_out, V, EpiStore{logits, (long)V, 0, 0}, wsplit(p.off_out));
    if (mode == kForwardAllRows) return;
    ProfScope pce(rt, kTagSoftmaxCe, 4.0 * M * V, 4.0 * 2.0 * M * V);
    if (V == 1024)
        ::hx::pdl_launch(softmax_ce_vec_kernel<32>, row_grid, 32 * rows_per_block, 0, s, 
            M, T, grad_scale, logits, tgt_ids, p.diag ? a.at<float>(p.probs) : nullptr, logits,
            a.at<double>(p.row_loss), a.at<int>(p.row_correct));
    else
        ::hx::pdl_launch(softmax_ce_kernel, row_grid, 32 * rows_per_block, 0, s, 
            M, V, T, grad_scale, logits, tgt_ids, p.diag ? a.at<float>(p.probs) : nullptr, logits,
            a.at<double>(p.row_loss), a.at<int>(p.row_correct));
    HX_LAUNCHED(rt);
        pce.end();
    ProfScope plr(rt, kTagReduce, 1.0 * M, 12.0 * M);
    ::hx::pdl_launch(loss_seq_kernel, (B + 7) / 8, 256, 0, s, B, T, a.at<double>(p.row_loss), a.at<int>(p.row_correct),
                                               a.at<float>(p.seq_loss), a.at<int>(p.seq_correct));
    HX_LAUNCHED(rt);
    ::hx::pdl_launch(loss_reduce_kernel, 1, 256, 0, s, B, T, a.at<float>(p.seq_loss), a.at<int>(p.seq_correct), grad_scale,
                                         a.at<float>(p.loss), a.at<float>(p.acc), G + p.P);
    HX_LAUNCHED(rt);
        plr.end();

    // ---- backward ----
    const float* dl = logits;  // dlogits, in place
    SideStream side(rt, p);
    side.fork();
    side.run([&] {
        gemm<true, false>(rt, D, V, M, xL, D, dl, V, EpiStore{G + p.off_out, (long)V, 0, 0});
        record_bucket(rt, p, 0, rt->stream);  // the output projection and the loss slot
    });
    float* dout = a.at<float>(p.dout);
    gemm<false, true>(rt, M, D, V, dl, V, W + p.off_out, V, EpiStore{dout, (long)D, 0, 0}, wsplit(p.off_out));
    if (p.diag) copy_d2d(rt, a.at<float>(p.diag_dout), dout, sizeof(float) * size_t(M) * D);
    float* dr = a.at<float>(p.dr);
    float* dc = a.at<float>(p.dc);
    float* dn = a.at<float>(p.dn);
    float* df1 = a.at<float>(p.df1);
    float* dqkv = a.at<float>(p.dqkv);
    float* part = a.at<float>(p.ln_part);
    const int lnw = 8;
    const size_t ln_smem = sizeof(float) * lnw * 2 * D;
    // LayerNorm backward with the residual add; the float4 path for D = 128, 256, 512
    auto ln_bwd = [&](const float* dy, const float* xx, const float* mean, const float* inv, const float* gam,
                      const float* res, float* dxo) {
        const int C = (D % 128 == 0) ? D / 128 : 0;
        if (C == 1 || C == 2 || C == 4) {
            auto k = C == 1 ? layernorm_bwd_vec_kernel<1> : C == 2 ? layernorm_bwd_vec_kernel<2> : layernorm_bwd_vec_kernel<4>;
            if (ln_smem > 48 * 1024) HX_CUDA(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ln_smem));
            ::hx::pdl_launch(k, p.ln_parts, 32 * lnw, ln_smem, s, M, p.ln_rows, dy, xx, mean, inv, gam, res, dxo, part);
        } else {
            if (ln_smem > 48 * 1024)
                HX_CUDA(cudaFuncSetAttribute(layernorm_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ln_smem));
            ::hx::pdl_launch(layernorm_bwd_kernel, p.ln_parts, 32 * lnw, ln_smem, s, M, D, p.ln_rows, dy, xx, mean, inv, gam, res, dxo,
                                                                         part);
        }
        HX_LAUNCHED(rt);
    };
    for (uint32_t li = p.L; li-- > 0;) {
        const LayerActs& A = p.la[li];
        const LayerOffsets& o = p.lo[li];
        const float* xin = a.at<float>(A.x);
        side.fork();  // dout is ready
        side.run([&] {
            gemm<true, false>(rt, F, D, M, a.at<float>(A.relu), F, dout, D, EpiStore{G + o.w2, (long)D, 0, 0});
        });
        gemm<false, true>(rt, M, F, D, dout, D, W + o.w2, D, EpiReluBackward{a.at<float>(A.relu), df1, nullptr, F},
                          wsplit(o.w2));
        side.fork();  // df1 is ready
        side.run([&] {
            gemm<true, false>(rt, D, F, M, a.at<float>(A.n2), D, df1, F, EpiStore{G + o.w1, (long)F, 0, 0});
        });
        gemm<false, true>(rt, M, D, F, df1, F, W + o.w1, F, EpiStore{dn, (long)D, 0, 0}, wsplit(o.w1));
        ProfScope plb2(rt, kTagLayerNorm, 12.0 * M * D, 4.0 * (4.0 * M * D + 2.0 * M));
        ln_bwd(dn, a.at<float>(A.r1), a.at<float>(A.mean2), a.at<float>(A.inv2), W + o.g2, dout, dr);
        plb2.end();
        ::hx::pdl_launch(column_reduce_kernel, (2 * D + 31) / 32, 32 * kColReduceWarps, 0, s, p.ln_parts, D, part, G + o.g2, G + o.b2);
        HX_LAUNCHED(rt);
        side.fork();  // dr is ready
        side.run([&] {
            gemm<true, false>(rt, D, D, M, a.at<float>(A.ctx), D, dr, D, EpiStore{G + o.wo, (long)D, 0, 0});
        });
        gemm<false, true>(rt, M, D, D, dr, D, W + o.wo, D, EpiStore{dc, (long)D, 0, 0}, wsplit(o.wo));
        HX_DH_DISPATCH(p.dh, attn_bwd_launch, rt, p, a.at<float>(A.qkv), dc, a.at<float>(A.rmax), a.at<float>(A.rsum),
                       dqkv);
        side.fork();  // dqkv is ready
        side.run([&] {
            gemm<true, false>(rt, D, 3 * D, M, a.at<float>(A.n1), D, dqkv, 3 * D,
                              EpiStore{G + o.wq, (long)D, (int)D, (long)D * D});
        });
        gemm<false, true>(rt, M, D, 3 * D, dqkv, 3 * D, wqkv + size_t(li) * 3 * D * D, 3 * D, EpiStore{dn, (long)D, 0, 0},
                          qsplit(li));
        // The side stream has read this layer's dout, df1, dr and dqkv before
        // the main stream overwrites them (dout next, the rest in the layer
        // below).
        side.join();
        ProfScope plb1(rt, kTagLayerNorm, 12.0 * M * D, 4.0 * (4.0 * M * D + 2.0 * M));
        ln_bwd(dn, xin, a.at<float>(A.mean1), a.at<float>(A.inv1), W + o.g1, dr, dout);
        plb1.end();
        ::hx::pdl_launch(column_reduce_kernel, (2 * D + 31) / 32, 32 * kColReduceWarps, 0, s, p.ln_parts, D, part, G + o.g1, G + o.b1);
        HX_LAUNCHED(rt);
        record_bucket(rt, p, int(p.L - li), s);  // this layer's ten tensors (its side work was joined above)
        if (p.diag) copy_d2d(rt, a.at<float>(p.diag_lig) + size_t(li) * M * D, dout, sizeof(float) * size_t(M) * D);
    }
    // embedding gradients
    ProfScope pemb2(rt, kTagEmbed, 1.0 * M * D, 4.0 * (2.0 * M * D + (p.emb_chunks + 1.0) * V * D));
    {
        const int tb = std::max(1, std::min<int>(V, kEmbTableFloats / D));
        const size_t esm = embed_bwd_smem_bytes(tb, D, p.emb_rows);
        if (esm > 48 * 1024)
            HX_CUDA(cudaFuncSetAttribute(embed_bwd_partial_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)esm));
        dim3 grid(p.emb_chunks, (V + tb - 1) / tb);
        ::hx::pdl_launch(embed_bwd_partial_kernel, grid, 32 * kEmbWarps, esm, s, M, V, D, p.emb_rows, tb, in_ids, dout,
                                                                    a.at<float>(p.emb_part));
        HX_LAUNCHED(rt);
        ::hx::pdl_launch(embed_bwd_combine_kernel, grid_for(long(V) * D, tpb, rt->sm_count), tpb, 0, s, 
            p.emb_chunks, V, D, a.at<float>(p.emb_part), G + p.off_E);
        HX_LAUNCHED(rt);
    }
    pemb2.end();
    if (p.learned) {
        ::hx::pdl_launch(position_bwd_kernel, (unsigned)((long(T) * D + 31) / 32), 32 * kPosWarps, 0, s, B, T, D, dout, G + p.off_pos);
        HX_LAUNCHED(rt);
    }
    side.join();  // the output projection's gradient, when L = 0
    record_bucket(rt, p, int(p.L + 1), s);  // token (and position) embedding
}

// Host part of the optimizer step: this step's scalars, exactly as the
// reference driver forms them, copied to step_scalars on the stream.
void upload_step_scalars(hx_runtime* rt, LmPlan& p, uint32_t step)
{
    // Bias corrections exactly as the reference driver computes them
    // (qnn/qnn_transformer_training.cpp:1504-1507): double, then float.
    const float c1 = float(1.0 / (1.0 - std::pow(double(p.opt.beta1), double(step))));
    const float c2 = float(1.0 / (1.0 - std::pow(double(p.opt.beta2), double(step))));
    // Scheduled learning rates (training_stability.h stabilityLearningRate).
    const float adam_lr = hx_stability_learning_rate(p.stab_mode, p.opt.adam_lr, step, p.stab_total);
    LmStepScalars v{};
    v.adam = adam_scalars(adam_lr, 1.0f, c1, c2);
    v.adam.beta1 = p.opt.beta1;
    v.adam.beta2 = p.opt.beta2;
    v.adam.one_minus_beta1 = 1.0f - p.opt.beta1;
    v.adam.one_minus_beta2 = 1.0f - p.opt.beta2;
    v.adam.eps = p.opt.adam_eps;
    v.momentum_lr = hx_stability_learning_rate(p.stab_mode, p.opt.momentum_lr, step, p.stab_total);
    v.muon_lr = hx_stability_learning_rate(p.stab_mode, p.opt.muon_lr, step, p.stab_total);
    const int slot = int(p.ring_next++ % LmPlan::kRing);
    if (p.ring_live[slot]) HX_CUDA(cudaEventSynchronize(p.ring_ev[slot]));
    p.ring[slot] = v;
    HX_CUDA(cudaMemcpyAsync(p.arena.at<LmStepScalars>(p.step_scalars), &p.ring[slot], sizeof(LmStepScalars),
                            cudaMemcpyHostToDevice, rt->stream));
    HX_CUDA(cudaEventRecord(p.ring_ev[slot], rt->stream));
    p.ring_live[slot] = true;
}

// Device part of the optimizer step: every launch reads its per-step
// scalars from step_scalars, so the same launches can be captured once and
// replayed for every step.
void optimizer_enqueue(hx_runtime* rt, LmPlan& p)
{
    const Arena& a = p.arena;
    float* W = a.at<float>(p.params);
    const float* G = a.at<float>(p.grads);
    float* m = a.at<float>(p.adam_m);
    float* v = a.at<float>(p.adam_v);
    const LmStepScalars* dyn = a.at<LmStepScalars>(p.step_scalars);
    // the global-norm clip scale, which Adam reads from device memory
    const float* scale_dev = nullptr;
    if (p.clip_threshold > 0.f) {
        launch_clip_scale(rt, G, a.at<GradTensor>(p.norm_table), p.norm_count, a.at<double>(p.norm_sumsq),
                          p.clip_threshold, a.at<double>(p.norm_value), a.at<float>(p.clip_scale));
        scale_dev = a.at<float>(p.clip_scale);
    }
    const AdamScalars host_unused = adam_scalars(0.f, 1.0f, 1.f, 1.f);  // replaced by dyn->adam on the device
    const AdamTaps none{};
    if (p.opt.kind == HX_OPT_MOMENTUM) {
        // velocity lives in the Muon buffer slot (zeroed on state upload)
        float* vel = a.at<float>(p.muon_buf);
        launch_momentum(rt, p.P, W, G, vel, W, vel, 0.f, p.opt.momentum, &dyn->momentum_lr);
    } else if (p.opt.kind == HX_OPT_MUON) {
        MuonScalars ms{0.f, p.opt.muon_momentum, p.opt.ns_a, p.opt.ns_b, p.opt.ns_c,
                       (int)p.opt.muon_nesterov, (int)p.opt.muon_ns_steps, (int)p.opt.muon_bf16_inputs};
        launch_muon(rt, a.at<MuonMatrix>(p.muon_table), p.muon_count, p.muon_smem, ms, &dyn->muon_lr,
                    muon_tc_shape(int(p.D), int(p.D)) && muon_tc_shape(int(p.D), int(p.F)));
        for (const auto& seg : p.adam_segments)
            launch_adam(rt, false, seg.second, W + seg.first, G + seg.first, m + seg.first, v + seg.first,
                        W + seg.first, m + seg.first, v + seg.first, host_unused, none, nullptr, &dyn->adam);
    } else {
        launch_adam(rt, false, p.P, W, G, m, v, W, m, v, host_unused, none, scale_dev, &dyn->adam);
    }
}

// Runs `body` from the plan's graph cache under `key`, or eagerly while the
// event profiler is on (its events need eager launches).
template <class F>
void lm_run(hx_runtime* rt, LmPlan& p, const GraphCache::Key& key, F&& body)
{
    if (rt->prof.on) {
        body();
        return;
    }
    run_cached(rt, p.graphs, key, body);
}

enum LmGraphKind : uintptr_t { kGraphTrainStep = 1, kGraphForwardBackward = 2, kGraphOptimizer = 3 };

GraphCache::Key lm_key(LmGraphKind kind, const void* tokens, float grad_scale) {
    GraphCache::Key k{};
    k[0] = kind;
    k[1] = reinterpret_cast<uintptr_t>(tokens);
    uint32_t bits;
    std::memcpy(&bits, &grad_scale, 4);
    k[2] = bits;
    return k;
}

LmPlan& need_lm(hx_runtime* rt) {
    require(rt->lm != nullptr, HX_ERR_STATE, "generalized tiny training graph not prepared");
    return *rt->lm;
}

void check_bad(hx_runtime* rt, LmPlan& p, const char* what) {
    int bad = 0;
    HX_CUDA(cudaMemcpyAsync(&bad, p.arena.at<int>(p.bad), sizeof(int), cudaMemcpyDeviceToHost, rt->stream));
    HX_CUDA(cudaStreamSynchronize(rt->stream));
    if (bad) fail(HX_ERR_ARGUMENT, what);
}

void default_optimizer(hx_optimizer_config& o) {
    o.kind = HX_OPT_ADAM;
    o.adam_lr = 1e-3f;
    o.beta1 = 0.9f;
    o.beta2 = 0.999f;
    o.adam_eps = 1e-8f;
    o.muon_lr = 0.02f;
    o.muon_momentum = 0.95f;
    o.muon_nesterov = 1;
    o.muon_ns_steps = 5;
    o.ns_a = 3.4445f;
    o.ns_b = -4.7750f;
    o.ns_c = 2.0315f;
    o.muon_bf16_inputs = 1;
    // the reference's momentum candidate (qnn_transformer_training.cpp:1258-1263)
    o.momentum_lr = 0.01f;
    o.momentum = 0.95f;
}

void host_fixed_position(const LmPlan& p, std::vector<float>& out) {
    // tiny_lm::fixedPosition (tiny_language_model_cpu.cpp:68), same float ops.
    out.assign(size_t(p.T) * p.D, 0.f);
    for (uint32_t t = 0; t < p.T; ++t)
        for (uint32_t d = 0; d < p.D; ++d) {
            const float f = std::pow(10000.f, -float(d & ~1u) / float(p.D));
            out[size_t(t) * p.D + d] = ((d & 1u) ? std::cos(float(t) * f) : std::sin(float(t) * f)) * .05f;
        }
}

}  // namespace
}  // namespace hx

using namespace hx;

extern "C" {

size_t hx_lm_param_count(const hx_lm_config* cfg) { return cfg ? hx::param_count(cfg) : 0; }

int hx_lm_validate(const hx_lm_config* cfg, char* err, size_t err_len) {
    try {
        validate(cfg);
        if (err && err_len) err[0] = 0;
        return HX_OK;
    } catch (const Error& e) {
        if (err && err_len) std::snprintf(err, err_len, "%s", e.message.c_str());
        return e.code;
    }
}

int hx_lm_prepare(hx_runtime* rt, const hx_lm_config* cfg, uint32_t batch, int diagnostic) {
    return hx_guard(rt, [&] {
        validate(cfg);
        require(batch >= 1, HX_ERR_ARGUMENT, "APP_CONFIGURATION_VALIDATION: batch must be >= 1");
        auto pp = std::unique_ptr<LmPlan, LmPlanDeleter>(new LmPlan());
        LmPlan& p = *pp;
        p.cfg = *cfg;
        p.B = batch; p.V = cfg->vocab; p.T = cfg->tokens; p.D = cfg->dim; p.F = cfg->ffn;
        p.L = cfg->layers; p.H = cfg->heads; p.dh = p.D / p.H;
        p.learned = (cfg->flags & HX_LM_LEARNED_POSITION) != 0;
        p.diag = diagnostic != 0;
        require(uint64_t(batch) * p.T < (uint64_t(1) << 31) && uint64_t(batch) * p.T * std::max(p.V, 3 * p.D) < (uint64_t(1) << 40),
                HX_ERR_ARGUMENT, "APP_RESOURCE_ESTIMATOR: batch*tokens too large");
        p.M = int(batch * p.T);
        require(dh_supported(p.dh), HX_ERR_UNSUPPORTED,
                "UNSUPPORTED_HEAD_DIMENSION: head dimension " + std::to_string(p.dh) +
                    " (supported: 1,2,3,4,6,8,12,16,24,32,48,64)");
        cudaDeviceProp prop{};
        HX_CUDA(cudaGetDeviceProperties(&prop, rt->device));
        const size_t smem_max = prop.sharedMemPerBlockOptin;
        require(attn_bwd_smem(p.T, p.dh, kAttnThreads / 32) <= smem_max && attn_fwd_smem(p.T, p.dh, kAttnThreads / 32) <= smem_max,
                HX_ERR_UNSUPPORTED, "UNSUPPORTED_ATTENTION_TILE: T*head_dim too large for one CTA's shared memory");
        p.P = param_count(cfg);
        // registry layout
        const size_t V = p.V, T = p.T, D = p.D, F = p.F;
        size_t off = 0;
        p.off_E = off; off += V * D;
        if (p.learned) { p.off_pos = off; off += T * D; }
        p.lo.resize(p.L);
        for (uint32_t l = 0; l < p.L; ++l) {
            LayerOffsets& o = p.lo[l];
            o.g1 = off; off += D;
            o.b1 = off; off += D;
            o.wq = off; off += D * D;
            o.wk = off; off += D * D;
            o.wv = off; off += D * D;
            o.wo = off; off += D * D;
            o.g2 = off; off += D;
            o.b2 = off; off += D;
            o.w1 = off; off += D * F;
            o.w2 = off; off += F * D;
        }
        p.off_out = off; off += D * V;
        require(off == p.P, HX_ERR_STATE, "internal: registry layout mismatch");

        const size_t f = sizeof(float), M = p.M, B = p.B, H = p.H;
        Arena& a = p.arena;
        p.params = a.reserve(f * p.P);
        p.exec_params = a.reserve(f * p.P);
        p.grads = a.reserve(f * (p.P + 1));
        p.adam_m = a.reserve(f * p.P);
        p.adam_v = a.reserve(f * p.P);
        p.muon_buf = a.reserve(f * p.P);
        p.pos_fixed = a.reserve(f * T * D);
        p.wqkv = a.reserve(f * p.L * 3 * D * D);
        p.w_hi = a.reserve(f * p.P);
        p.w_lo = a.reserve(f * p.P);
        p.wqkv_hi = a.reserve(f * p.L * 3 * D * D);
        p.wqkv_lo = a.reserve(f * p.L * 3 * D * D);
        p.tokens = a.reserve(sizeof(uint32_t) * B * (T + 1));
        p.in_tok = a.reserve(sizeof(uint32_t) * M);
        p.tgt_tok = a.reserve(sizeof(uint32_t) * M);
        p.in_ids = a.reserve(sizeof(int) * M);
        p.tgt_ids = a.reserve(sizeof(int) * M);
        p.bad = a.reserve(sizeof(int) * 4);
        p.la.resize(p.L);
        for (uint32_t l = 0; l < p.L; ++l) {
            LayerActs& A = p.la[l];
            A.x = a.reserve(f * M * D);
            A.n1 = a.reserve(f * M * D);
            A.mean1 = a.reserve(f * M);
            A.inv1 = a.reserve(f * M);
            A.qkv = a.reserve(f * M * 3 * D);
            A.ctx = a.reserve(f * M * D);
            A.r1 = a.reserve(f * M * D);
            A.n2 = a.reserve(f * M * D);
            A.mean2 = a.reserve(f * M);
            A.inv2 = a.reserve(f * M);
            A.relu = a.reserve(f * M * F);
            A.rmax = a.reserve(f * B * H * T);
            A.rsum = a.reserve(f * B * H * T);
        }
        p.xL = a.reserve(f * M * D);
        p.logits = a.reserve(f * M * V);
        p.probs = p.diag ? a.reserve(f * M * V) : 0;
        p.row_loss = a.reserve(sizeof(double) * M);
        p.row_correct = a.reserve(sizeof(int) * M);
        p.seq_loss = a.reserve(sizeof(float) * B);
        p.seq_correct = a.reserve(sizeof(int) * B);
        p.loss = a.reserve(f * 4);
        p.acc = a.reserve(f * 4);
        p.scalars = a.reserve(f * 8);
        p.dout = a.reserve(f * M * D);
        p.dr = a.reserve(f * M * D);
        p.dc = a.reserve(f * M * D);
        p.dn = a.reserve(f * M * D);
        p.df1 = a.reserve(f * M * F);
        p.dqkv = a.reserve(f * M * 3 * D);
        p.attn_bstat = a.reserve(f * 2 * B * H * T);
        p.ln_parts = std::max(1, std::min<int>(p.M, 4 * rt->sm_count));  // 32 warps per SM of the LN backward
        p.ln_rows = (p.M + p.ln_parts - 1) / p.ln_parts;
        p.ln_parts = (p.M + p.ln_rows - 1) / p.ln_rows;
        p.ln_part = a.reserve(f * size_t(p.ln_parts) * 2 * D);
        // Short chunks: the CTAs of the most frequent tokens bound the kernel
        // (under Zipf ids most rows fall in the first token block), so the
        // chunk shrinks with the row count, down to 64 rows.
        p.emb_rows = std::max(64, std::min(1024, p.M / 64));
        p.emb_chunks = (p.M + p.emb_rows - 1) / p.emb_rows;
        p.emb_part = a.reserve(f * size_t(p.emb_chunks) * V * D);
        if (p.diag) {
            p.diag_lig = a.reserve(f * p.L * M * D);
            p.diag_hp = a.reserve(f * p.L * B * H * T * T);
            p.diag_dout = a.reserve(f * M * D);
        }
        // Muon matrices: wq, wk, wv, wo, ffn_w1, ffn_w2 of every layer
        p.muon_table = a.reserve(sizeof(MuonMatrix) * 6 * p.L);
        // Global gradient norm: one entry per registry tensor
        p.norm_count = int(2 + (p.learned ? 1 : 0) + 10 * p.L);
        p.norm_table = a.reserve(sizeof(GradTensor) * p.norm_count);
        p.norm_sumsq = a.reserve(sizeof(double) * p.norm_count);
        p.norm_value = a.reserve(sizeof(double));
        p.clip_scale = a.reserve(sizeof(float));
        p.step_scalars = a.reserve(sizeof(LmStepScalars));
        a.commit();
        HX_CUDA(cudaMemsetAsync(a.block.ptr, 0, a.used, rt->stream));
        std::vector<float> pos;
        host_fixed_position(p, pos);
        HX_CUDA(cudaMemcpyAsync(a.at<float>(p.pos_fixed), pos.data(), f * pos.size(), cudaMemcpyHostToDevice, rt->stream));
        default_optimizer(p.opt);
        // Muon table + Adam segments for the non-Muon parameters
        std::vector<MuonMatrix> mats;
        float* W = a.at<float>(p.params);
        float* G = a.at<float>(p.grads);
        float* Bf = a.at<float>(p.muon_buf);
        p.adam_segments.clear();
        p.adam_segments.push_back({0, p.lo.empty() ? p.P : p.lo[0].g1});  // token_embedding (+ position)
        for (uint32_t l = 0; l < p.L; ++l) {
            const LayerOffsets& o = p.lo[l];
            p.adam_segments.push_back({o.g1, 2 * D});
            p.adam_segments.push_back({o.g2, 2 * D});
            const size_t offs[6] = {o.wq, o.wk, o.wv, o.wo, o.w1, o.w2};
            const int rows[6] = {int(D), int(D), int(D), int(D), int(D), int(F)};
            const int cols[6] = {int(D), int(D), int(D), int(D), int(F), int(D)};
            for (int k = 0; k < 6; ++k) mats.push_back(MuonMatrix{W + offs[k], G + offs[k], Bf + offs[k], rows[k], cols[k]});
        }
        p.adam_segments.push_back({p.off_out, D * V});
        p.muon_count = int(mats.size());
        p.muon_smem = std::max(muon_smem_bytes(int(D), int(D)), muon_smem_bytes(int(D), int(F)));
        HX_CUDA(cudaMemcpyAsync(a.at<MuonMatrix>(p.muon_table), mats.data(), sizeof(MuonMatrix) * mats.size(),
                                cudaMemcpyHostToDevice, rt->stream));
        // Tensor order of gradientNorm (qnn/qnn_transformer_training.cpp:920-938):
        // token embedding, per layer wq wk wv wo gamma1 beta1 gamma2 beta2 w1 w2,
        // output projection (the learned position table follows the embedding).
        std::vector<GradTensor> norm;
        norm.push_back({p.off_E, (unsigned long long)V * D});
        if (p.learned) norm.push_back({p.off_pos, (unsigned long long)T * D});
        for (uint32_t l = 0; l < p.L; ++l) {
            const LayerOffsets& o = p.lo[l];
            const unsigned long long dd = (unsigned long long)D * D, df = (unsigned long long)D * F;
            for (const GradTensor t : {GradTensor{o.wq, dd}, GradTensor{o.wk, dd}, GradTensor{o.wv, dd},
                                       GradTensor{o.wo, dd}, GradTensor{o.g1, D}, GradTensor{o.b1, D},
                                       GradTensor{o.g2, D}, GradTensor{o.b2, D}, GradTensor{o.w1, df},
                                       GradTensor{o.w2, df}})
                norm.push_back(t);
        }
        norm.push_back({p.off_out, (unsigned long long)D * V});
        require(int(norm.size()) == p.norm_count, HX_ERR_STATE, "internal: gradient-norm table size");
        HX_CUDA(cudaMemcpyAsync(a.at<GradTensor>(p.norm_table), norm.data(), sizeof(GradTensor) * norm.size(),
                                cudaMemcpyHostToDevice, rt->stream));
        HX_CUDA(cudaHostAlloc(reinterpret_cast<void**>(&p.ring), sizeof(LmStepScalars) * LmPlan::kRing,
                              cudaHostAllocDefault));
        for (cudaEvent_t& e : p.fork_ev) HX_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
        p.buckets.push_back({p.off_out, D * V + 1});  // output projection + the scaled loss slot G[P]
        for (uint32_t l = p.L; l-- > 0;) p.buckets.push_back({p.lo[l].g1, 4 * D * D + 4 * D + 2 * D * F});
        p.buckets.push_back({0, p.L ? p.lo[0].g1 : p.off_out});
        p.bucket_ev.resize(p.buckets.size());
        for (cudaEvent_t& e : p.bucket_ev) HX_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
        if (!rt->side_stream) HX_CUDA(cudaStreamCreateWithFlags(&rt->side_stream, cudaStreamNonBlocking));
        for (cudaEvent_t& e : p.ring_ev) HX_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
        HX_CUDA(cudaStreamSynchronize(rt->stream));
        rt->lm = std::move(pp);
        ++rt->metrics.graph_create_count;
    });
}

int hx_lm_execute_tokens(hx_runtime* rt, const uint32_t* input_tokens, const uint32_t* target_tokens,
                         const float* params, size_t param_count_, const hx_lm_outputs* out);

static void lm_execute_common(hx_runtime* rt, LmPlan& p, const float* params, size_t pc, float lr,
                              const hx_lm_outputs* out) {
    require(params && out && out->loss && out->grads, HX_ERR_ARGUMENT, "generalized tiny training buffer schema");
    require(pc == p.P, HX_ERR_ARGUMENT, "generalized tiny training buffer schema: parameter count " +
                                            std::to_string(pc) + " != " + std::to_string(p.P));
    require(lr == 0.0f, HX_ERR_ARGUMENT, "generalized tiny training requires learningRate=0; use Adam");
    const bool wants_diag = out->logits || out->probabilities || out->d_logits || out->output || out->d_output ||
                            out->layer_input_grads || out->head_probabilities;
    require(!wants_diag || p.diag, HX_ERR_STATE, "diagnostic outputs requested but the graph was prepared without them");
    const Arena& a = p.arena;
    const size_t f = sizeof(float);
    float* W = a.at<float>(p.exec_params);
    float* G = a.at<float>(p.grads);
    HX_CUDA(cudaMemcpyAsync(W, params, f * p.P, cudaMemcpyHostToDevice, rt->stream));
    forward_backward(rt, p, W, G, 1.0f / float(p.B));
    const size_t M = p.M;
    HX_CUDA(cudaMemcpyAsync(out->grads, G, f * p.P, cudaMemcpyDeviceToHost, rt->stream));
    HX_CUDA(cudaMemcpyAsync(out->loss, a.at<float>(p.loss), f, cudaMemcpyDeviceToHost, rt->stream));
    if (out->accuracy) HX_CUDA(cudaMemcpyAsync(out->accuracy, a.at<float>(p.acc), f, cudaMemcpyDeviceToHost, rt->stream));
    auto get = [&](float* dst, size_t off, size_t n) {
        if (dst) HX_CUDA(cudaMemcpyAsync(dst, a.at<float>(off), f * n, cudaMemcpyDeviceToHost, rt->stream));
    };
    if (p.diag) {
        // dlogits live in place of the logits; the logits output is
        // reconstructed only through the probabilities (see docs): report
        // dlogits and probabilities, and recompute logits when asked.
        get(out->d_logits, p.logits, M * p.V);
        get(out->probabilities, p.probs, M * p.V);
        get(out->output, p.xL, M * p.D);
        get(out->d_output, p.diag_dout, M * p.D);
        get(out->layer_input_grads, p.diag_lig, size_t(p.L) * M * p.D);
        get(out->head_probabilities, p.diag_hp, size_t(p.L) * p.B * p.H * p.T * p.T);
        if (out->logits) {
            gemm<false, false>(rt, p.M, p.V, p.D, a.at<float>(p.xL), p.D, W + p.off_out, p.V,
                               EpiStore{a.at<float>(p.logits), (long)p.V, 0, 0});
            get(out->logits, p.logits, M * p.V);
        }
    }
    rt->check_device_error();
}

int hx_lm_execute(hx_runtime* rt, const float* input_one_hot, const float* target_one_hot, const float* params,
                  size_t pc, float lr, const hx_lm_outputs* out) {
    const auto t0 = Clock::now();
    const int rc = hx_guard(rt, [&] {
        LmPlan& p = need_lm(rt);
        require(input_one_hot && target_one_hot, HX_ERR_ARGUMENT, "generalized tiny training buffer schema");
        const size_t n = size_t(p.M) * p.V;
        if (p.onehot.bytes < 2 * n * sizeof(float)) p.onehot.allocate(2 * n * sizeof(float));
        float* dev = p.onehot.as<float>();
        HX_CUDA(cudaMemcpyAsync(dev, input_one_hot, n * sizeof(float), cudaMemcpyHostToDevice, rt->stream));
        HX_CUDA(cudaMemcpyAsync(dev + n, target_one_hot, n * sizeof(float), cudaMemcpyHostToDevice, rt->stream));
        const Arena& a = p.arena;
        HX_CUDA(cudaMemsetAsync(a.at<int>(p.bad), 0, sizeof(int), rt->stream));
        ::hx::pdl_launch(one_hot_decode_kernel, (p.M + 7) / 8, 256, 0, rt->stream, p.M, p.V, dev, a.at<uint32_t>(p.in_tok), a.at<int>(p.bad));
        HX_LAUNCHED(rt);
        ::hx::pdl_launch(one_hot_decode_kernel, (p.M + 7) / 8, 256, 0, rt->stream, p.M, p.V, dev + n, a.at<uint32_t>(p.tgt_tok), a.at<int>(p.bad));
        HX_LAUNCHED(rt);
        check_bad(rt, p, "INVALID_TINY_LM_ONE_HOT: every input/target row must hold exactly one 1.0 and zeros elsewhere");
        ::hx::pdl_launch(copy_ids_kernel, grid_for(p.M, 256, rt->sm_count), 256, 0, rt->stream, 
            p.M, p.V, a.at<uint32_t>(p.in_tok), a.at<uint32_t>(p.tgt_tok), a.at<int>(p.in_ids), a.at<int>(p.tgt_ids), a.at<int>(p.bad));
        HX_LAUNCHED(rt);
        lm_execute_common(rt, p, params, pc, lr, out);
        if (rt->injected_now()) fail(HX_ERR_CUDA, "injected execute failure after device success");
    });
    if (rt) rt->record_execute(rc == HX_OK, us_since(t0));
    return rc;
}

int hx_lm_execute_tokens(hx_runtime* rt, const uint32_t* in, const uint32_t* tgt, const float* params, size_t pc,
                         const hx_lm_outputs* out) {
    const auto t0 = Clock::now();
    const int rc = hx_guard(rt, [&] {
        LmPlan& p = need_lm(rt);
        require(in && tgt, HX_ERR_ARGUMENT, "generalized tiny training buffer schema");
        const Arena& a = p.arena;
        HX_CUDA(cudaMemcpyAsync(a.at<uint32_t>(p.in_tok), in, sizeof(uint32_t) * p.M, cudaMemcpyHostToDevice, rt->stream));
        HX_CUDA(cudaMemcpyAsync(a.at<uint32_t>(p.tgt_tok), tgt, sizeof(uint32_t) * p.M, cudaMemcpyHostToDevice, rt->stream));
        HX_CUDA(cudaMemsetAsync(a.at<int>(p.bad), 0, sizeof(int), rt->stream));
        ::hx::pdl_launch(copy_ids_kernel, grid_for(p.M, 256, rt->sm_count), 256, 0, rt->stream, 
            p.M, p.V, a.at<uint32_t>(p.in_tok), a.at<uint32_t>(p.tgt_tok), a.at<int>(p.in_ids), a.at<int>(p.tgt_ids), a.at<int>(p.bad));
        HX_LAUNCHED(rt);
        check_bad(rt, p, "INVALID_TINY_LM_TOKEN: token id >= vocabulary size");
        lm_execute_common(rt, p, params, pc, 0.0f, out);
        if (rt->injected_now()) fail(HX_ERR_CUDA, "injected execute failure after device success");
    });
    if (rt) rt->record_execute(rc == HX_OK, us_since(t0));
    return rc;
}

int hx_lm_forward_tokens(hx_runtime* rt, const uint32_t* tokens, const float* params, size_t pc, float* logits) {
    const auto t0 = Clock::now();
    const int rc = hx_guard(rt, [&] {
        LmPlan& p = need_lm(rt);
        require(tokens && logits, HX_ERR_ARGUMENT, "generalized tiny training forward-only buffer schema");
        const Arena& a = p.arena;
        const float* W = a.at<float>(p.params);
        if (params) {
            require(pc == p.P, HX_ERR_ARGUMENT, "generalized tiny training forward-only buffer schema");
            for (size_t i = 0; i < pc; ++i)
                require(std::isfinite(params[i]), HX_ERR_ARGUMENT, "generalized tiny training forward-only buffer schema");
            HX_CUDA(cudaMemcpyAsync(a.at<float>(p.exec_params), params, sizeof(float) * p.P, cudaMemcpyHostToDevice,
                                    rt->stream));
            W = a.at<float>(p.exec_params);
        } else {
            require(p.state_ready, HX_ERR_STATE, "forward-only on the device state before state upload");
        }
        HX_CUDA(cudaMemcpyAsync(a.at<uint32_t>(p.in_tok), tokens, sizeof(uint32_t) * p.M, cudaMemcpyHostToDevice,
                                rt->stream));
        HX_CUDA(cudaMemsetAsync(a.at<int>(p.bad), 0, sizeof(int), rt->stream));
        ::hx::pdl_launch(copy_ids_kernel, grid_for(p.M, 256, rt->sm_count), 256, 0, rt->stream, 
            p.M, p.V, a.at<uint32_t>(p.in_tok), a.at<uint32_t>(p.in_tok), a.at<int>(p.in_ids), a.at<int>(p.tgt_ids),
            a.at<int>(p.bad));
        HX_LAUNCHED(rt);
        check_bad(rt, p, "INVALID_TINY_LM_TOKEN: token id >= vocabulary size");
        forward_backward(rt, p, W, a.at<float>(p.grads), 1.0f, kForwardAllRows);
        const size_t n = size_t(p.M) * p.V;
        HX_CUDA(cudaMemcpyAsync(logits, a.at<float>(p.logits), sizeof(float) * n, cudaMemcpyDeviceToHost, rt->stream));
        rt->check_device_error();
        for (size_t i = 0; i < n; ++i)
            require(std::isfinite(logits[i]), HX_ERR_NONFINITE, "QNN_NONFINITE: forward-only logits are not finite");
        if (rt->injected_now()) fail(HX_ERR_CUDA, "injected execute failure after device success");
    });
    if (rt) rt->record_execute(rc == HX_OK, us_since(t0));
    return rc;
}

int hx_lm_generate(hx_runtime* rt, const uint32_t* prompts, uint32_t prompt_len, uint32_t max_new,
                   const hx_sampling* sampling, uint32_t* out) {
    return hx_guard(rt, [&] {
        LmPlan& p = need_lm(rt);
        require(prompts && sampling && out, HX_ERR_ARGUMENT, "generation: null buffer");
        require(prompt_len > 0, HX_ERR_ARGUMENT, "PROMPT_EMPTY: prompt is empty");
        require(p.state_ready, HX_ERR_STATE, "generation before state upload");
        const uint32_t B = p.B, T = p.T, V = p.V;
        std::vector<std::vector<uint32_t>> history(B);
        for (uint32_t b = 0; b < B; ++b) {
            history[b].assign(prompts + size_t(b) * prompt_len, prompts + size_t(b + 1) * prompt_len);
            for (uint32_t t : history[b])
                require(t < V, HX_ERR_ARGUMENT, "INVALID_TINY_LM_TOKEN: token id >= vocabulary size");
        }
        const Arena& a = p.arena;
        std::vector<uint32_t> window(size_t(B) * T);
        std::vector<float> rows(size_t(B) * V);
        for (uint32_t step = 0; step < max_new; ++step) {
            // buildTokenContext (nicopedia_byte_bpe.h:278-291): the last T
            // tokens, right-aligned, left-padded with token 0.
            for (uint32_t b = 0; b < B; ++b) {
                const auto& h = history[b];
                const size_t keep = std::min<size_t>(h.size(), T), pad = T - keep;
                uint32_t* w = window.data() + size_t(b) * T;
                std::fill(w, w + pad, 0u);
                std::copy(h.end() - keep, h.end(), w + pad);
            }
            HX_CUDA(cudaMemcpyAsync(a.at<uint32_t>(p.in_tok), window.data(), sizeof(uint32_t) * p.M,
                                    cudaMemcpyHostToDevice, rt->stream));
            ::hx::pdl_launch(copy_ids_kernel, grid_for(p.M, 256, rt->sm_count), 256, 0, rt->stream, 
                p.M, p.V, a.at<uint32_t>(p.in_tok), a.at<uint32_t>(p.in_tok), a.at<int>(p.in_ids),
                a.at<int>(p.tgt_ids), a.at<int>(p.bad));
            HX_LAUNCHED(rt);
            forward_backward(rt, p, a.at<float>(p.params), a.at<float>(p.grads), 1.0f, kForwardLastRow);
            HX_CUDA(cudaMemcpyAsync(rows.data(), a.at<float>(p.logits), sizeof(float) * rows.size(),
                                    cudaMemcpyDeviceToHost, rt->stream));
            rt->check_device_error();
            for (uint32_t b = 0; b < B; ++b) {
                hx_sampling sb = *sampling;
                sb.seed = sampling->seed + b;  // stream b samples with seed + b
                uint32_t tok = 0;
                if (hx_sample_next_token(rows.data() + size_t(b) * V, V, &sb, step, &tok, nullptr) != HX_OK)
                    fail(HX_ERR_NONFINITE, "generation step produced non-finite logits on prepared graph");
                out[size_t(b) * max_new + step] = tok;
                history[b].push_back(tok);
            }
        }
    });
}

int hx_lm_state_upload(hx_runtime* rt, const float* params, const float* m, const float* v, const float* buf, size_t pc) {
    return hx_guard(rt, [&] {
        LmPlan& p = need_lm(rt);
        require(params && pc == p.P, HX_ERR_ARGUMENT, "state upload: parameter count mismatch");
        const Arena& a = p.arena;
        const size_t b = sizeof(float) * p.P;
        HX_CUDA(cudaMemcpyAsync(a.at<float>(p.params), params, b, cudaMemcpyHostToDevice, rt->stream));
        auto put = [&](const float* src, size_t off) {
            if (src) HX_CUDA(cudaMemcpyAsync(a.at<float>(off), src, b, cudaMemcpyHostToDevice, rt->stream));
            else HX_CUDA(cudaMemsetAsync(a.at<float>(off), 0, b, rt->stream));
        };
        put(m, p.adam_m);
        put(v, p.adam_v);
        put(buf, p.muon_buf);
        HX_CUDA(cudaStreamSynchronize(rt->stream));
        p.state_ready = true;
    });
}

int hx_lm_state_download(hx_runtime* rt, float* params, float* m, float* v, float* buf, size_t pc) {
    return hx_guard(rt, [&] {
        LmPlan& p = need_lm(rt);
        require(pc == p.P, HX_ERR_ARGUMENT, "state download: parameter count mismatch");
        require(p.state_ready, HX_ERR_STATE, "state download before upload");
        const Arena& a = p.arena;
        const size_t b = sizeof(float) * p.P;
        auto get = [&](float* dst, size_t off) {
            if (dst) HX_CUDA(cudaMemcpyAsync(dst, a.at<float>(off), b, cudaMemcpyDeviceToHost, rt->stream));
        };
        get(params, p.params);
        get(m, p.adam_m);
        get(v, p.adam_v);
        get(buf, p.muon_buf);
        HX_CUDA(cudaStreamSynchronize(rt->stream));
    });
}

int hx_lm_set_optimizer(hx_runtime* rt, const hx_optimizer_config* opt) {
    return hx_guard(rt, [&] {
        LmPlan& p = need_lm(rt);
        require(opt != nullptr, HX_ERR_ARGUMENT, "optimizer: null configuration");
        require(opt->kind == HX_OPT_ADAM || opt->kind == HX_OPT_MUON || opt->kind == HX_OPT_MOMENTUM,
                HX_ERR_ARGUMENT, "optimizer: unknown kind");
        require(opt->kind != HX_OPT_MOMENTUM || (std::isfinite(opt->momentum_lr) && std::isfinite(opt->momentum)),
                HX_ERR_ARGUMENT, "momentum optimizer buffer size or scalar");
        require(opt->kind == HX_OPT_ADAM || p.clip_threshold == 0.f, HX_ERR_UNSUPPORTED,
                "gradient clipping scales the Adam gradient input; it needs the Adam optimizer");
        require(std::isfinite(opt->adam_lr) && std::isfinite(opt->beta1) && std::isfinite(opt->beta2) &&
                    std::isfinite(opt->adam_eps) && opt->beta1 >= 0.f && opt->beta1 < 1.f && opt->beta2 >= 0.f &&
                    opt->beta2 < 1.f,
                HX_ERR_ARGUMENT, "optimizer: invalid Adam scalars");
        if (opt->kind == HX_OPT_MUON) {
            check_muon_shape(int(p.D), int(p.D));
            check_muon_shape(int(p.D), int(p.F));
            require(std::isfinite(opt->muon_lr) && std::isfinite(opt->muon_momentum), HX_ERR_ARGUMENT,
                    "optimizer: invalid Muon scalars");
        }
        p.opt = *opt;
        p.graphs.clear();
    });
}

int hx_lm_set_stability(hx_runtime* rt, uint32_t mode, uint32_t total_steps, float clip_threshold) {
    return hx_guard(rt, [&] {
        LmPlan& p = need_lm(rt);
        const char* bad = hx_stability_mode_error(mode);
        require(bad == nullptr, HX_ERR_UNSUPPORTED, bad ? bad : "");
        require(std::isfinite(clip_threshold) && clip_threshold >= 0.f, HX_ERR_ARGUMENT,
                "gradient clip threshold must be finite and >= 0");
        // GRADIENT_CLIP_1 fixes the threshold at 1 (qnn_transformer_training.cpp:1650-1653).
        const float thr = mode == HX_STABILITY_GRADIENT_CLIP_1 ? 1.0f : clip_threshold;
        require(thr == 0.f || p.opt.kind == HX_OPT_ADAM, HX_ERR_UNSUPPORTED,
                "gradient clipping scales the Adam gradient input; it needs the Adam optimizer");
        p.stab_mode = mode;
        p.stab_total = total_steps;
        p.clip_threshold = thr;
        p.graphs.clear();
    });
}

int hx_lm_last_gradient_norm(hx_runtime* rt, double* norm, float* clip_scale) {
    return hx_guard(rt, [&] {
        LmPlan& p = need_lm(rt);
        require(p.clip_threshold > 0.f, HX_ERR_STATE, "no gradient clipping configured");
        HX_CUDA(cudaStreamSynchronize(rt->stream));
        if (norm) HX_CUDA(cudaMemcpy(norm, p.arena.at<double>(p.norm_value), sizeof(double), cudaMemcpyDeviceToHost));
        if (clip_scale)
            HX_CUDA(cudaMemcpy(clip_scale, p.arena.at<float>(p.clip_scale), sizeof(float), cudaMemcpyDeviceToHost));
    });
}

int hx_lm_train_step(hx_runtime* rt, const uint32_t* tokens, uint32_t step, float* loss) {
    const auto t0 = Clock::now();
    const int rc = hx_guard(rt, [&] {
        LmPlan& p = need_lm(rt);
        require(tokens && loss, HX_ERR_ARGUMENT, "train step: null buffer");
        require(step >= 1, HX_ERR_ARGUMENT, "train step: step is 1-based");
        require(p.state_ready, HX_ERR_STATE, "train step before state upload");
        const Arena& a = p.arena;
        const auto tb = Clock::now();
        HX_CUDA(cudaMemcpyAsync(a.at<uint32_t>(p.tokens), tokens, sizeof(uint32_t) * size_t(p.B) * (p.T + 1),
                                cudaMemcpyHostToDevice, rt->stream));
        rt->metrics.last_input_bind_us = us_since(tb);
        upload_step_scalars(rt, p, step);
        const float gs = 1.0f / float(p.B);
        lm_run(rt, p, lm_key(kGraphTrainStep, a.at<uint32_t>(p.tokens), gs), [&] {
            HX_CUDA(cudaMemsetAsync(a.at<int>(p.bad), 0, sizeof(int), rt->stream));
            ::hx::pdl_launch(split_tokens_kernel, grid_for(p.M, 256, rt->sm_count), 256, 0, rt->stream, 
                p.B, p.T, p.V, a.at<uint32_t>(p.tokens), a.at<int>(p.in_ids), a.at<int>(p.tgt_ids), a.at<int>(p.bad));
            HX_LAUNCHED(rt);
            forward_backward(rt, p, a.at<float>(p.params), a.at<float>(p.grads), gs);
            optimizer_enqueue(rt, p);
        });
        const auto to = Clock::now();
        int bad = 0;
        HX_CUDA(cudaMemcpyAsync(loss, a.at<float>(p.loss), sizeof(float), cudaMemcpyDeviceToHost, rt->stream));
        HX_CUDA(cudaMemcpyAsync(&bad, a.at<int>(p.bad), sizeof(int), cudaMemcpyDeviceToHost, rt->stream));
        rt->check_device_error();
        rt->metrics.last_output_bind_us = us_since(to);
        require(!bad, HX_ERR_ARGUMENT, "INVALID_TINY_LM_TOKEN: token id >= vocabulary size (state was updated with id 0)");
        require(std::isfinite(*loss), HX_ERR_NONFINITE, "QNN_NONFINITE: training loss is not finite");
        if (rt->injected_now()) fail(HX_ERR_CUDA, "injected execute failure after device success");
    });
    if (rt) rt->record_execute(rc == HX_OK, us_since(t0));
    return rc;
}

int hx_lm_forward_backward_device(hx_runtime* rt, const uint32_t* tokens, float grad_scale) {
    return hx_guard(rt, [&] {
        LmPlan& p = need_lm(rt);
        require(tokens, HX_ERR_ARGUMENT, "forward_backward: null tokens");
        require(std::isfinite(grad_scale) && grad_scale > 0.f, HX_ERR_ARGUMENT, "forward_backward: invalid grad_scale");
        require(p.state_ready, HX_ERR_STATE, "forward_backward before state upload");
        const Arena& a = p.arena;
        lm_run(rt, p, lm_key(kGraphForwardBackward, tokens, grad_scale), [&] {
            ::hx::pdl_launch(split_tokens_kernel, grid_for(p.M, 256, rt->sm_count), 256, 0, rt->stream, 
                p.B, p.T, p.V, tokens, a.at<int>(p.in_ids), a.at<int>(p.tgt_ids), a.at<int>(p.bad));
            HX_LAUNCHED(rt);
            forward_backward(rt, p, a.at<float>(p.params), a.at<float>(p.grads), grad_scale);
        });
    });
}

int hx_lm_grad_buffer(hx_runtime* rt, float** grads, size_t* count) {
    return hx_guard(rt, [&] {
        LmPlan& p = need_lm(rt);
        require(grads && count, HX_ERR_ARGUMENT, "grad_buffer: null output");
        *grads = p.arena.at<float>(p.grads);
        *count = p.P + 1;
    });
}

int hx_lm_optimizer_step_device(hx_runtime* rt, uint32_t step) {
    return hx_guard(rt, [&] {
        LmPlan& p = need_lm(rt);
        require(step >= 1, HX_ERR_ARGUMENT, "optimizer step is 1-based");
        upload_step_scalars(rt, p, step);
        lm_run(rt, p, lm_key(kGraphOptimizer, nullptr, 0.f), [&] { optimizer_enqueue(rt, p); });
    });
}

int hx_lm_grad_buckets(hx_runtime* rt, size_t* offsets, size_t* counts, int capacity, int* count) {
    return hx_guard(rt, [&] {
        LmPlan& p = need_lm(rt);
        require(count && capacity >= 0 && (capacity == 0 || (offsets && counts)), HX_ERR_ARGUMENT,
                "grad_buckets: null output");
        *count = int(p.buckets.size());
        for (int i = 0; i < capacity && i < int(p.buckets.size()); ++i) {
            offsets[i] = p.buckets[size_t(i)].first;
            counts[i] = p.buckets[size_t(i)].second;
        }
    });
}

int hx_lm_enable_bucket_events(hx_runtime* rt, int enable) {
    return hx_guard(rt, [&] {
        LmPlan& p = need_lm(rt);
        if (p.bucket_events != (enable != 0)) p.graphs.clear();
        p.bucket_events = enable != 0;
    });
}

int hx_lm_bucket_wait(hx_runtime* rt, int bucket, void* stream) {
    return hx_guard(rt, [&] {
        LmPlan& p = need_lm(rt);
        require(p.bucket_events, HX_ERR_STATE, "bucket_wait: bucket events are not enabled");
        require(bucket >= 0 && bucket < int(p.buckets.size()), HX_ERR_ARGUMENT, "bucket_wait: bucket out of range");
        HX_CUDA(cudaStreamWaitEvent(static_cast<cudaStream_t>(stream), p.bucket_ev[size_t(bucket)], 0));
    });
}

int hx_lm_loss_device(hx_runtime* rt, float** loss) {
    return hx_guard(rt, [&] {
        LmPlan& p = need_lm(rt);
        require(loss, HX_ERR_ARGUMENT, "loss_device: null output");
        *loss = p.arena.at<float>(p.loss);
    });
}

}  // extern "C"
