/*
 * hexatrain.h -- C ABI of the HexaTrain B200 runtime (libhexatrain_b200.so).
 *
 * This is the drop-in replacement for the reference's runtime seam, class
 * phonelm::qnn::Runtime (app/src/main/cpp/qnn/qnn_runtime.h:250-451): the
 * same prepare-once / execute-per-step lifecycle, the same named inputs and
 * outputs in the same order, and the same fail-closed error convention
 * (a status plus a human-readable message whose prefix classifies the
 * failure; nothing throws across this boundary).  Plain pointers and sizes
 * only.  "Host" entry points take application-owned host buffers and copy
 * them in and out per call, exactly like the reference's clientBuf binding;
 * "_device" entry points take device pointers and run asynchronously on the
 * runtime's stream.
 *
 * Threading: one runtime is used by one host thread at a time (as the
 * reference's Runtime).  Several runtimes may coexist in one process.
 */
#ifndef HEXATRAIN_H
#define HEXATRAIN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------- */
enum {
    HX_OK = 0,
    HX_ERR_ARGUMENT = 1,   /* null pointer, zero/oversized dimension, size mismatch */
    HX_ERR_STATE = 2,      /* call out of lifecycle order (execute before prepare) */
    HX_ERR_CUDA = 3,       /* a CUDA runtime call failed (message has the CUDA error) */
    HX_ERR_NONFINITE = 4,  /* a result or input was NaN/Inf where the contract forbids it */
    HX_ERR_MEMORY = 5,     /* device allocation failed */
    HX_ERR_UNSUPPORTED = 6 /* a valid request this build does not serve */
};

typedef struct hx_runtime hx_runtime;

/* ---- runtime ------------------------------------------------------------ */

/* Create a runtime bound to CUDA device `device` with its own non-blocking
 * stream.  Replaces Runtime::initialize (qnn/qnn_runtime.h:266).  On failure
 * *out is NULL and `err` (if non-NULL) receives the message. */
int hx_runtime_create(int device, hx_runtime** out, char* err, size_t err_len);
/* Release every device allocation and the stream (Runtime::~Runtime,
 * qnn/qnn_runtime.h:253). */
void hx_runtime_destroy(hx_runtime* rt);
/* Message of the last failed call on this runtime ("" after success).
 * Mirrors the std::string& error out-parameter of every Runtime method. */
const char* hx_runtime_last_error(const hx_runtime* rt);
/* Use `stream` (a cudaStream_t, or NULL for the runtime's own stream) for
 * all subsequent work.  The caller keeps ownership. */
int hx_runtime_set_stream(hx_runtime* rt, void* stream);
void* hx_runtime_stream(const hx_runtime* rt);
/* Block until all work queued on the runtime's stream finished. */
int hx_runtime_synchronize(hx_runtime* rt);

/* Counters mirroring RuntimeMetrics / ApiTrace (qnn/qnn_runtime.h:58-131). */
typedef struct {
    uint64_t graph_create_count;     /* prepare calls that succeeded */
    uint64_t graph_finalize_count;   /* CUDA graphs instantiated */
    uint64_t graph_execute_count;    /* execute / step calls that succeeded */
    uint64_t execute_attempt_count;
    uint64_t execute_failure_count;
    int64_t first_failure_call;      /* -1 if none */
    double last_execute_us;          /* host wall time of the last execute */
    double total_execute_us;
    double last_input_bind_us;       /* host->device copy enqueue time */
    double last_output_bind_us;      /* device->host copy + sync time */
    uint64_t kernel_launches;        /* kernels this runtime launched */
    uint64_t device_bytes;           /* device memory held by this runtime */
} hx_metrics;
int hx_runtime_metrics(const hx_runtime* rt, hx_metrics* out);

/* Host-side failure injection (the reference's failGraphExecuteAt,
 * qnn/qnn_runtime.h:136 and qnn/qnn_runtime_full_step.inc:383-397): the
 * execute call whose attempt index equals `call_index` reports failure with
 * code HX_ERR_CUDA and message "injected execute failure" after its device
 * work finished.  -1 disables.  No device fault is involved. */
int hx_runtime_inject_execute_failure(hx_runtime* rt, int64_t call_index);

/* Failure-path self-test of the device-side bounded waits (no counterpart in
 * the reference).  Every pipeline wait of the tensor-core GEMM and attention
 * kernels gives up after a bounded number of clock cycles, records a code in
 * the runtime's device error word, tears down and returns; the next
 * synchronising call then fails with a "DEVICE_WAIT_TIMEOUT: ..." message.
 * This call runs that path on purpose without any fault: one thread waits,
 * with the same bounded wait, on an mbarrier that nothing arrives at, for
 * `cycles` SM clock cycles (0 < cycles <= 4e9).  It returns HX_ERR_CUDA with
 * the DEVICE_WAIT_TIMEOUT message; the error word is cleared, so the
 * runtime's next call proceeds normally.  Synchronous. */
int hx_runtime_check_wait_timeout(hx_runtime* rt, long long cycles);

/* GEMM engine selection.  AUTO (default) runs large FP32 GEMMs on the
 * tensor cores as 3xTF32 (tcgen05, TMEM accumulators, TMA-fed) and small or
 * unaligned ones on the CUDA cores; the other values force one engine where
 * the problem allows it (tests use this to compare the two). */
enum { HX_GEMM_AUTO = 0, HX_GEMM_CUDA_CORES = 1, HX_GEMM_TENSOR_CORES = 2 };
int hx_runtime_set_gemm_backend(hx_runtime* rt, int backend);

/* Attention engine selection.  AUTO (default) runs causal attention with
 * head dimension 32 and at most 256 tokens on the tensor cores (3xTF32
 * products, softmax on the CUDA cores) unless attention probabilities are
 * requested as a diagnostic output; CUDA_CORES forces the FP32 CUDA-core
 * kernels everywhere (tests use this to compare the two). */
enum { HX_ATTN_AUTO = 0, HX_ATTN_CUDA_CORES = 1 };
int hx_runtime_set_attention_backend(hx_runtime* rt, int backend);

/* Per-kernel-class timing with CUDA events recorded on the runtime stream
 * around every launch while enabled (the counterpart of RuntimeMetrics'
 * executeUs lists, qnn/qnn_runtime.h:68, at kernel granularity).  Steps run
 * eagerly (no CUDA graph replay) while profiling is on.  _read synchronises
 * the stream, aggregates and clears the records. */
typedef struct {
    char name[32];        /* kernel class, e.g. "gemm", "attention_fwd" */
    uint64_t launches;
    double total_ms;      /* sum of event-timed durations */
    double flops;         /* algorithmic FLOPs of those launches */
    double bytes;         /* algorithmic DRAM bytes of those launches */
} hx_profile_entry;
int hx_runtime_profile(hx_runtime* rt, int enable);
int hx_runtime_profile_read(hx_runtime* rt, hx_profile_entry* entries, int capacity, int* count);

/* ---- two-layer ReLU MLP full training step ------------------------------ */
/* Graph phonelm_mlp_training_step (qnn/qnn_runtime_full_step.inc:209-330):
 *   Z1=X W1; H=ReLU(Z1); P=H W2; E=P-Y; loss=mean(E^2); dP=E*2/(B*O);
 *   dW2=H^T dP; dH=dP W2^T (W2 before the update); mask=H>0;
 *   dZ1=mask?dH:0; dW1=X^T dZ1; W1_next=W1-lr*dW1; W2_next=W2-lr*dW2.
 * Shapes: X[B,I] Y[B,O] W1[I,H] W2[H,O], row-major FP32. */

/* Runtime::prepareMlpFullStep (qnn/qnn_runtime.h:422).  diagnostic != 0
 * makes the nine intermediate tensors readable (the reference's APP_READ
 * diagnostic outputs). */
int hx_mlp_prepare(hx_runtime* rt, uint32_t batch, uint32_t input_dim, uint32_t hidden_dim,
                   uint32_t output_dim, int diagnostic);

/* Output bindings, in the reference's output order
 * (qnn/qnn_runtime_full_step.inc:353-354).  loss/w1_next/w2_next are
 * required; the rest are written only when prepared with diagnostic != 0
 * and may be NULL otherwise (NULL skips that output). */
typedef struct {
    float* loss;          /* [1]   */
    float* w1_next;       /* [I*H] */
    float* w2_next;       /* [H*O] */
    float* prediction;    /* [B*O] */
    float* error;         /* [B*O] */
    float* d_prediction;  /* [B*O] */
    float* d_w2;          /* [H*O] */
    float* d_hidden;      /* [B*H] */
    uint8_t* mask;        /* [B*H], 1 where hidden > 0 (BOOL_8) */
    float* d_z1;          /* [B*H] */
    float* d_w1;          /* [I*H] */
    float* hidden;        /* [B*H] */
} hx_mlp_outputs;

/* Runtime::executeMlpFullStep (qnn/qnn_runtime.h:425-430): host buffers in,
 * host buffers out, synchronous.  Element counts are checked against the
 * prepared shape ("full step buffer size mismatch").  Inputs are not
 * modified; outputs must not alias inputs. */
int hx_mlp_execute(hx_runtime* rt, const float* x, size_t x_count, const float* y, size_t y_count,
                   const float* w1, size_t w1_count, const float* w2, size_t w2_count,
                   float learning_rate, const hx_mlp_outputs* out);

/* Same step on device pointers (x,y,w1,w2 and every non-NULL field of
 * `out`), enqueued on the runtime stream without synchronising.  This is the
 * ping-pong form: the caller swaps its two weight buffers between calls, so
 * no weight bytes are copied per step.  `out` itself is a host struct. */
int hx_mlp_execute_device(hx_runtime* rt, const float* x, const float* y, const float* w1,
                          const float* w2, float learning_rate, const hx_mlp_outputs* out);

/* The same step on device pointers for callers that cannot let this library
 * allocate device memory: a process whose GPU memory already belongs to its
 * own allocator (a host framework's caching pool), or a step path on which
 * cudaMalloc/cudaFree are not allowed because they synchronise the device.
 * It has no counterpart in the reference.  No hx_mlp_prepare is needed and
 * nothing is allocated: the intermediates (2*B*H + 2*B*O floats, after a
 * 4352-byte header) live in one fixed 4 MiB array of device memory that every
 * GPU loading this library holds until the process exits; larger shapes fail
 * with HX_ERR_UNSUPPORTED.  The first call on a device (and the first after
 * that device's context was recreated) looks up that array's address (and
 * may load the library's device code); make it before any stream capture.
 * All calls on a device share the array, so calls whose work overlaps on the
 * GPU (other streams or other runtimes on the same device) race; calls on
 * one stream are safe.  Returns after the step has finished on the runtime
 * stream; it waits for that stream only.  K is never split, so shapes that the
 * allocating step splits may differ from it in the last bits. */
int hx_mlp_execute_device_noalloc(hx_runtime* rt, uint32_t batch, uint32_t input_dim,
                                  uint32_t hidden_dim, uint32_t output_dim, const float* x,
                                  const float* y, const float* w1, const float* w2,
                                  float learning_rate, float* loss, float* w1_next,
                                  float* w2_next);

/* ---- tiny causal Transformer LM ----------------------------------------- */

enum {
    HX_LM_LEARNED_POSITION = 1u  /* learned [T,D] table after token_embedding
                                    instead of the fixed sinusoid*0.05 */
};

typedef struct {
    uint32_t vocab;   /* V */
    uint32_t tokens;  /* T (sequence length) */
    uint32_t dim;     /* D */
    uint32_t ffn;     /* F */
    uint32_t layers;  /* L */
    uint32_t heads;   /* H, D % H == 0 */
    float eps;        /* LayerNorm epsilon (the reference uses 1e-5) */
    uint32_t flags;   /* HX_LM_* */
} hx_lm_config;

/* Parameter count of the flat registry-ordered buffer
 * (tiny_language_model_cpu.cpp parameterRegistry; flattening order of
 * qnn/qnn_transformer_training.cpp:1164-1180):
 *   token_embedding[V*D], (position_embedding[T*D] if learned),
 *   per layer {norm1_gamma[D], norm1_beta[D], wq, wk, wv, wo [D*D each],
 *              norm2_gamma[D], norm2_beta[D], ffn_w1[D*F], ffn_w2[F*D]},
 *   output_projection[D*V]. */
size_t hx_lm_param_count(const hx_lm_config* cfg);
/* Validate a configuration (tiny_lm::validateConfig,
 * transformer_resource_estimator.h:76-83).  Returns HX_OK or
 * HX_ERR_ARGUMENT and writes the classified message to err. */
int hx_lm_validate(const hx_lm_config* cfg, char* err, size_t err_len);
/* Deterministic initialisers, host side.  _reference reproduces
 * tiny_lm::initialParameters (tiny_language_model_cpu.cpp:69-70); _normal
 * draws N(0, std) for every matrix and table (gamma=1, beta=0) from a
 * splitmix64 stream seeded by `seed`. */
int hx_lm_init_reference(const hx_lm_config* cfg, uint32_t seed, float* params);
int hx_lm_init_normal(const hx_lm_config* cfg, uint64_t seed, float std, float* params);

/* Runtime::prepareTinyTransformerTraining, generalized builder
 * (qnn/qnn_runtime.h:398-408, qnn/qnn_runtime_transformer_training_generalized.inc:4).
 * `batch` sequences are processed per execute (the reference runs one per
 * graph execute and loops on the host; here the batch is folded into the
 * row dimension of every kernel).  diagnostic != 0 keeps per-sequence
 * logits/probabilities/dlogits/output readable. */
int hx_lm_prepare(hx_runtime* rt, const hx_lm_config* cfg, uint32_t batch, int diagnostic);

/* Outputs of one execute.  loss and grads are required.  The diagnostic
 * fields need diagnostic != 0 at prepare time and may be NULL. Shapes are
 * per batch: [batch*T*V] etc. */
typedef struct {
    float* loss;               /* [1] mean over sequences of the mean CE */
    float* accuracy;           /* [1] optional: argmax accuracy over all rows */
    float* grads;              /* [P] sum_b grad_b / batch, registry order */
    float* logits;             /* [batch*T*V] */
    float* probabilities;      /* [batch*T*V] */
    float* d_logits;           /* [batch*T*V]  (p - onehot)/T (times 1/batch) */
    float* output;             /* [batch*T*D]  last block output */
    float* d_output;           /* [batch*T*D]  dloss/doutput */
    float* layer_input_grads;  /* [L*batch*T*D] */
    float* head_probabilities; /* [L*batch*H*T*T] */
} hx_lm_outputs;

/* Runtime::executeTinyTransformerTraining (qnn/qnn_runtime.h:409-412):
 * one-hot rows in (input/target [batch*T*V], host), current parameters
 * (host, flat registry order), learning_rate must be 0 (the graph stops at
 * gradients, qnn/qnn_runtime_transformer_training_generalized_execute.inc:88-91),
 * outputs to host.  A row that is not exactly one-hot is rejected
 * ("INVALID_TINY_LM_ONE_HOT"). */
int hx_lm_execute(hx_runtime* rt, const float* input_one_hot, const float* target_one_hot,
                  const float* params, size_t param_count, float learning_rate,
                  const hx_lm_outputs* out);
/* Same with token ids [batch*T] instead of one-hot rows. */
int hx_lm_execute_tokens(hx_runtime* rt, const uint32_t* input_tokens, const uint32_t* target_tokens,
                         const float* params, size_t param_count, const hx_lm_outputs* out);

/* -- device-resident training state (the batched driver loop of
 *    qnn/qnn_transformer_training.cpp:7281-7345 in one call per step) ---- */

enum { HX_OPT_ADAM = 0, HX_OPT_MUON = 1, HX_OPT_MOMENTUM = 2 };
typedef struct {
    uint32_t kind;        /* HX_OPT_ADAM: Adam on every parameter.
                             HX_OPT_MUON: Muon on wq,wk,wv,wo,ffn_w1,ffn_w2;
                             Adam on the rest.
                             HX_OPT_MOMENTUM: momentum SGD on every parameter
                             (tiny_lm::momentumUpdate,
                             tiny_language_model_cpu.cpp:123); the velocity
                             occupies the state's Muon-buffer slot. */
    float adam_lr, beta1, beta2, adam_eps;
    float muon_lr, muon_momentum;
    uint32_t muon_nesterov, muon_ns_steps;
    float ns_a, ns_b, ns_c;
    uint32_t muon_bf16_inputs;  /* round Newton-Schulz operands to bf16 */
    float momentum_lr, momentum; /* HX_OPT_MOMENTUM (defaults 0.01, 0.95) */
} hx_optimizer_config;

/* Load parameters (and Adam moments / Muon buffers, or zeros when NULL)
 * into device state.  Requires hx_lm_prepare. */
int hx_lm_state_upload(hx_runtime* rt, const float* params, const float* adam_m, const float* adam_v,
                       const float* muon_buf, size_t param_count);
int hx_lm_state_download(hx_runtime* rt, float* params, float* adam_m, float* adam_v,
                         float* muon_buf, size_t param_count);
int hx_lm_set_optimizer(hx_runtime* rt, const hx_optimizer_config* opt);

/* Training-stability modes (training_stability.h:20-99). */
enum {
    HX_STABILITY_LEGACY = 0,
    HX_STABILITY_WARMUP64 = 1,                     /* lr * min(1, step/64) */
    HX_STABILITY_DECAY_LINEAR = 2,                 /* lr * (1 - (step-1)/total) */
    HX_STABILITY_ZERO_OUTPUT_PROJ_BRANCH_INIT = 3, /* init: Wo, W2 = 0 */
    HX_STABILITY_DEPTH_SCALED_BRANCH_INIT = 4,     /* init: Wo, W1, W2 / sqrt(2L) */
    HX_STABILITY_RESIDUAL_BRANCH_SCALING = 5,      /* reserved; rejected as in the reference */
    HX_STABILITY_GRADIENT_CLIP_1 = 6               /* global-norm clip at 1 before Adam */
};
/* validateTrainingStabilityMode (:77-81): NULL, or the reference's tag
 * (RESIDUAL_BRANCH_SCALING_UNSUPPORTED_ON_DEVICE,
 * UNKNOWN_TRAINING_STABILITY_MODE). */
const char* hx_stability_mode_error(uint32_t mode);
/* stabilityLearningRate (:88-99); `step` is 1-based. */
float hx_stability_learning_rate(uint32_t mode, float base, uint32_t step, uint32_t total_steps);
/* applyInitStability (:104-121) on a flat registry-ordered parameter
 * buffer; modes other than 3 and 4 leave it unchanged.  Host only. */
int hx_lm_apply_init_stability(const hx_lm_config* config, uint32_t mode, float* params);
/* Selects the step-side mode for hx_lm_train_step / optimizer_step_device:
 * the scheduled learning rate over total_steps, and a global-norm gradient
 * clip (the reference's clipThreshold, qnn_transformer_training.cpp:
 * 2432-2445): scale = min(1, threshold/(||g|| + 1e-6)) applied as Adam's
 * gradient-scale input, with ||g|| summed per tensor in double in
 * gradientNorm order (:920-938).  clip_threshold 0 disables the clip;
 * HX_STABILITY_GRADIENT_CLIP_1 sets it to 1.  Clipping needs Adam. */
int hx_lm_set_stability(hx_runtime* rt, uint32_t mode, uint32_t total_steps, float clip_threshold);
/* Pre-clip global gradient norm and the clip scale of the last optimizer
 * step (synchronises the runtime stream).  Requires an active clip. */
int hx_lm_last_gradient_norm(hx_runtime* rt, double* norm, float* clip_scale);

/* One training step on the device state: tokens [batch, T+1] host ids
 * (sequence b reads ids[b][0..T-1], predicts ids[b][1..T]); forward,
 * backward, gradient averaging and the optimizer update with bias
 * corrections for step `step` (1-based).  *loss receives the mean loss
 * (host).  Host in, host out, synchronous. */
int hx_lm_train_step(hx_runtime* rt, const uint32_t* tokens, uint32_t step, float* loss);

/* The same step split for data parallelism, on device pointers, async:
 *  1. hx_lm_forward_backward_device: tokens [batch, T+1] (device uint32)
 *     -> device gradient buffer (sum_b grad_b * grad_scale) and its last
 *     element = sum_b loss_b * grad_scale;
 *  2. the caller all-reduces that buffer (P+1 floats) across ranks;
 *  3. hx_lm_optimizer_step_device applies the optimizer.
 * grad_scale is 1/global_batch. */
int hx_lm_forward_backward_device(hx_runtime* rt, const uint32_t* tokens, float grad_scale);
int hx_lm_grad_buffer(hx_runtime* rt, float** grads, size_t* count);
int hx_lm_optimizer_step_device(hx_runtime* rt, uint32_t step);
/* Device pointer to the mean loss of the last step (1 float). */
int hx_lm_loss_device(hx_runtime* rt, float** loss);

/* Gradient buckets for overlapping the data-parallel all-reduce with the
 * backward pass (no counterpart in the reference, which averages on the
 * host, qnn/qnn_transformer_training.cpp:7322-7330).  The [P+1] gradient
 * buffer splits into contiguous buckets in the order the backward finishes
 * them: the output projection with the loss slot, each layer's ten tensors
 * from the last layer down, then the token (and position) embedding.
 * hx_lm_grad_buckets writes up to `capacity` (offset, count) pairs in that
 * order and their number.  With bucket events enabled, every
 * hx_lm_forward_backward_device records one CUDA event per bucket when the
 * bucket's gradients are final (inside a captured step graph too), and
 * hx_lm_bucket_wait(rt, i, stream) makes `stream` (a cudaStream_t) wait for
 * bucket i of the most recent forward_backward: a communication stream can
 * then reduce bucket i while the backward continues.  The caller must make
 * the runtime's stream wait for that communication stream before
 * hx_lm_optimizer_step_device. */
int hx_lm_grad_buckets(hx_runtime* rt, size_t* offsets, size_t* counts, int capacity, int* count);
int hx_lm_enable_bucket_events(hx_runtime* rt, int enable);
int hx_lm_bucket_wait(hx_runtime* rt, int bucket, void* stream);

/* ---- elementwise Adam ----------------------------------------------------- */
/* Graph phonelm_adam_optimizer (qnn/qnn_runtime_transformer.inc:926-1109):
 *   g'=g*gradient_scale; m'=b1*m+(1-b1)*g'; v'=b2*v+(1-b2)*g'^2;
 *   m^=m'*c1; v^=v'*c2; r=sqrt(v^); den=r+eps; div=m^/den;
 *   norm=(v^>0)?div:0; upd=lr*norm; w'=w-upd
 * with b1=0.9, b2=0.999, eps=1e-8 and the rounding order of
 * tiny_lm::adamUpdate (tiny_language_model_cpu.cpp:124-145). */
int hx_adam_prepare(hx_runtime* rt, uint32_t elements);
typedef struct {
    float* m_next;
    float* v_next;
    float* m_hat;
    float* v_hat;
    float* sqrt_v_hat;
    float* denominator;
    float* divided;
    float* normalized;
    float* scaled_update;
    float* w_next;          /* required; all others may be NULL */
} hx_adam_outputs;
/* Runtime::executeAdamOptimizer (qnn/qnn_runtime.h:361-369), host buffers,
 * synchronous.  Rejects non-finite scalars and gradient_scale outside
 * [0,1] ("Adam optimizer buffer size or scalar"). */
int hx_adam_execute(hx_runtime* rt, const float* current, const float* gradient,
                    const float* first_moment, const float* second_moment, float learning_rate,
                    float gradient_scale, float first_correction, float second_correction,
                    const hx_adam_outputs* out);
/* Device-pointer variant over n elements (w_next, m_next and v_next are
 * required; in-place updates w_next==current etc. are allowed). */
int hx_adam_execute_device(hx_runtime* rt, size_t n, const float* current, const float* gradient,
                           const float* first_moment, const float* second_moment,
                           float learning_rate, float gradient_scale, float first_correction,
                           float second_correction, const hx_adam_outputs* out);

/* ---- forward-only LM and generation -------------------------------------- */
/* executeTinyTransformerForwardOnly (qnn/qnn_runtime.h:418-421,
 * qnn_runtime_transformer_training_generalized_execute.inc:320-...):
 * logits [batch*T, V] for token ids [batch*T] under `params` (host,
 * registry order, checked finite), or under the device state when params is
 * NULL.  No target and no backward.  Non-finite logits fail with
 * HX_ERR_NONFINITE.  Synchronous.  Requires hx_lm_prepare. */
int hx_lm_forward_tokens(hx_runtime* rt, const uint32_t* tokens, const float* params,
                         size_t param_count, float* logits);

typedef struct {
    uint32_t greedy;      /* 1: greedyArgmax (first maximum) */
    float temperature;    /* <= 0 or non-finite: greedy */
    uint32_t top_k;       /* 0: the whole vocabulary */
    uint64_t seed;
} hx_sampling;
typedef struct {
    uint32_t ok, logits_finite;
    double weight_sum, probability_sum;
} hx_sampling_audit;
/* greedyArgmax / sampleTopKChecked (nicopedia_generation.h:286-395) on one
 * logit row: top-K by (logit desc, index asc), temperature softmax in
 * double, u = top 53 bits of splitmix64(seed + step * 0x9E3779B97F4A7C15)
 * / 2^53, first cumulative probability >= u.  Host only.  Non-finite
 * logits or weights fail with HX_ERR_NONFINITE and ok = 0. */
int hx_sample_next_token(const float* logits, uint32_t vocab, const hx_sampling* sampling,
                         uint64_t step, uint32_t* token, hx_sampling_audit* audit);
/* The prepared generation loop (qnn/qnn_prepared_generation.cpp:392-430)
 * for `batch` independent streams on the device state: each step feeds
 * the last T tokens of every stream (left-padded with 0, buildTokenContext),
 * projects only the last row and samples it (stream b with seed + b).
 * prompts [batch*prompt_len], out [batch*max_new].  Synchronous. */
int hx_lm_generate(hx_runtime* rt, const uint32_t* prompts, uint32_t prompt_len, uint32_t max_new,
                   const hx_sampling* sampling, uint32_t* out);

/* ---- momentum SGD optimizer ------------------------------------------------ */
/* Runtime::prepareMomentumOptimizer / executeMomentumOptimizer
 * (qnn/qnn_runtime.h:353-359, graph qnn_runtime_transformer.inc:799-925):
 * velocity' = velocity*momentum + gradient; weight' = weight - velocity'*lr.
 * Host buffers, synchronous ("momentum optimizer buffer size or scalar"). */
int hx_momentum_prepare(hx_runtime* rt, uint32_t elements);
int hx_momentum_execute(hx_runtime* rt, const float* current, const float* gradient,
                        const float* velocity, float learning_rate, float momentum,
                        float* velocity_next, float* weight_next);
/* Device-pointer variant over n elements, async; in place allowed. */
int hx_momentum_execute_device(hx_runtime* rt, size_t n, const float* current, const float* gradient,
                               const float* velocity, float learning_rate, float momentum,
                               float* velocity_next, float* weight_next);

/* ---- Muon (no counterpart in the reference) ------------------------------ */
/* Momentum (+Nesterov) and quintic Newton-Schulz orthogonalisation of one
 * matrix update, Jordan et al. 2024; see hx_optimizer_config.  Host buffers
 * [rows*cols], synchronous.  rows, cols <= 256. */
int hx_muon_execute(hx_runtime* rt, uint32_t rows, uint32_t cols, const float* weight,
                    const float* gradient, const float* momentum_buffer, float learning_rate,
                    float momentum, int nesterov, uint32_t ns_steps, float a, float b, float c,
                    int bf16_inputs, float* weight_next, float* momentum_buffer_next);

/* ---- NPRTCKPTV2 / V3 checkpoint of the LM training state ----------------- */
/* The reference's canonical resume file (qnn/qnn_transformer_training.cpp:
 * 5164-5252 writer nprtSaveCheckpointV2, :5390-5522 reader
 * nprtLoadCheckpointForGeneration): header (magic, V T D F L H seed step,
 * big endian), the V3 tokenizer block at vocabulary 1024, then the
 * parameter, Adam first-moment and Adam second-moment registries in
 * tiny_lm::parameterRegistry order (tiny_language_model_cpu.cpp:63).  The
 * flat buffers here (hx_lm_state_download order) are that order; a
 * learned-position model adds "position_embedding" after
 * "token_embedding".  Codec errors are the reference's NPRT_CKPT_* codes. */
typedef struct {
    uint32_t version;          /* 1, 2 or 3 (NPRTCKPTV1 / V2 / V3) */
    uint32_t seed;
    uint32_t step;
    uint32_t finite;           /* 0 when any stored value is NaN or infinite */
    uint32_t has_adam;         /* 1 for V2 / V3 */
    uint64_t parameter_count;
    char parameter_hash[32];   /* nprtParameterHash: "fnv1a64:" + 16 hex digits */
    char tokenizer_hash[80];   /* V3 only */
} hx_nprt_info;

/* Bytes hx_nprt_encode writes for this configuration and tokenizer identity. */
size_t hx_nprt_encoded_bytes(const hx_lm_config* config, const char* tokenizer_kind,
                             const char* tokenizer_hash);
/* nprtSaveCheckpointV2 (:5171-5252) into memory: refuses step 0 and
 * non-finite state; at vocabulary 1024 writes NPRTCKPTV3 and needs kind
 * "byte_bpe" and a 71-character "sha256:" hash, otherwise NPRTCKPTV2 with
 * both NULL or empty.  Host only; needs no runtime or GPU. */
int hx_nprt_encode(const hx_lm_config* config, uint32_t seed, uint32_t step,
                   const char* tokenizer_kind, const char* tokenizer_hash, const float* params,
                   const float* adam_m, const float* adam_v, uint8_t* out, size_t capacity,
                   size_t* written, char* error, size_t error_capacity);
/* nprtLoadCheckpointForGeneration (:5390-5522) over memory: validates and,
 * where the pointers are non-NULL, copies the registries out.  V1 files
 * decode with has_adam = 0.  Host only. */
int hx_nprt_decode(const hx_lm_config* config, uint32_t expected_seed,
                   const char* expected_tokenizer_hash, const uint8_t* data, size_t size,
                   hx_nprt_info* info, float* params, float* adam_m, float* adam_v, char* error,
                   size_t error_capacity);
/* nicopedia_checkpoint::checkpointName (nicopedia_checkpoint_policy.h):
 * "htp-seed<S>-l<L>[-t<T>-d<D>-f<F>]-step<N>.ckpt". */
int hx_nprt_checkpoint_name(uint32_t seed, uint32_t layers, uint32_t tokens, uint32_t dimension,
                            uint32_t feed_forward_dimension, uint32_t step, char* out,
                            size_t capacity);
/* nprtTrainingOrder (qnn/qnn_transformer_training.cpp:4983-4995): the
 * record index of every (step, batch slot), a pure function of the global
 * step, so a resumed run re-derives its data cursor.  out[steps*batch]. */
int hx_nprt_training_order(uint64_t record_count, uint32_t steps, uint32_t batch, uint64_t* out);
/* Writes the prepared LM's device state (parameters, Adam moments) to
 * `path` via "<path>.tmp" and a rename.  Adam optimizer only: the format
 * has no slot for Muon momentum. */
int hx_lm_checkpoint_save(hx_runtime* rt, const char* path, uint32_t seed, uint32_t step,
                          const char* tokenizer_kind, const char* tokenizer_hash);
/* Canonical resume (:7068-7109): decodes `path`, requires the step
 * (expected_step != 0), finite values and Adam moments (a V1 file fails
 * with RESUME_ADAM_STATE_MISSING), then uploads the state.  Continue with
 * hx_lm_train_step(step + 1, ...). */
int hx_lm_checkpoint_resume(hx_runtime* rt, const char* path, uint32_t expected_seed,
                            uint32_t expected_step, const char* tokenizer_hash, hx_nprt_info* info);

#ifdef __cplusplus
}
#endif
#endif /* HEXATRAIN_H */
