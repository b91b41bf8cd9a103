/*
 * hx_oracle.h -- CPU restatement of HexaTrain's training-step arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker: tests/, the smoke
 * entry and bench.py's cpu_baseline leg call it to produce expected values.
 * The product (hexatrain_b200) never links, loads or calls it, and has no
 * CPU fallback onto it.
 *
 * Each function states the reference routine it restates (paths relative to
 * the HexaTrain source tree).  The restatement keeps the reference's order of
 * floating-point operations (double accumulators where the reference uses
 * them, float where it uses float) so that, built with the same compiler and
 * flags, its results equal the reference's own CPU path value-for-value.  The
 * pin is tests/test_oracle.py against tests/golden/ (generated from the
 * reference itself by tests/golden/make_golden.py).
 *
 * Extensions with no reference counterpart (learned positional embedding,
 * Muon) are marked as such; their parity is pinned by finite differences and
 * by mathematical properties instead.
 */
#ifndef HX_ORACLE_H
#define HX_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- two-layer ReLU MLP full step --------------------------------------
 * Restates the driver's pass() (app/src/main/cpp/qnn/qnn_mlp_training.cpp:53-72)
 * over cpu::matMul / meanSquaredError (app/src/main/cpp/cpu_reference_training.cpp:129-170)
 * followed by cpu::sgdUpdate (:197-204) on both weights.
 * Every output pointer must be non-NULL and sized as documented:
 *   z1,h,dh,dz1 [B,H]; mask [B,H] (1 where h>0); p,e,dp [B,O];
 *   dw2,w2_next [H,O]; dw1,w1_next [I,H].  Returns 0, or -1 on bad sizes. */
int hxo_mlp_step(int B, int I, int H, int O,
                 const float* x, const float* y, const float* w1, const float* w2,
                 float lr, float* loss, float* w1_next, float* w2_next,
                 float* z1, float* h, float* p, float* e, float* dp,
                 float* dw2, float* dh, unsigned char* mask, float* dz1, float* dw1);

/* Plain matMul with double accumulation (cpu_reference_training.cpp:129-142):
 * out[M,N] = lhs[M,K] * rhs[K,N], all row-major. */
void hxo_matmul(int M, int N, int K, const float* lhs, const float* rhs, float* out);
/* meanSquaredError (cpu_reference_training.cpp:163-170). */
float hxo_mse(size_t n, const float* prediction, const float* target);
/* Linear-layer forwardBackward (cpu_reference_training.cpp:172-195):
 * X[B,D], target[B,D], W[D,D]. */
float hxo_linear_forward_backward(int B, int D, const float* x, const float* target,
                                  const float* w, float* prediction, float* error,
                                  float* d_prediction, float* d_weight, float* d_input);
/* sgdUpdate (cpu_reference_training.cpp:197-204): w -= lr * dw, in place. */
void hxo_sgd(size_t n, float* w, const float* dw, float lr);

/* ---- tiny Transformer LM --------------------------------------------- */
typedef struct {
    uint32_t vocab;      /* V */
    uint32_t tokens;     /* T */
    uint32_t dim;        /* D */
    uint32_t ffn;        /* F */
    uint32_t layers;     /* L */
    uint32_t heads;      /* H; D % H == 0 */
    float eps;           /* LayerNorm epsilon (reference: 1e-5) */
    int learned_position;/* 0: fixed sinusoid*0.05 (reference);
                            1: learned [T,D] table stored after token_embedding
                               (extension, no reference counterpart) */
} hxo_lm_config;

/* Flat parameter layout in registry order
 * (tiny_language_model_cpu.cpp:63 parameterRegistry, and the flattening in
 * qnn/qnn_transformer_training.cpp:1164-1180):
 *   token_embedding[V*D], (position_embedding[T*D] when learned),
 *   per layer {norm1_gamma[D], norm1_beta[D], wq[D*D], wk[D*D], wv[D*D],
 *              wo[D*D], norm2_gamma[D], norm2_beta[D], ffn_w1[D*F],
 *              ffn_w2[F*D]},
 *   output_projection[D*V]. */
size_t hxo_lm_param_count(const hxo_lm_config* c);
/* Offsets of each tensor in the flat layout; returns the number of tensors
 * and fills up to `cap` entries of offsets/sizes. */
int hxo_lm_layout(const hxo_lm_config* c, size_t* offsets, size_t* sizes, int cap);

/* fixedPosition (tiny_language_model_cpu.cpp:68): out[T*D]. */
void hxo_lm_fixed_position(const hxo_lm_config* c, float* out);

/* One sequence, forward + explicit backward
 * (tiny_language_model_cpu.cpp:41-49 generalForward, :73-83
 * generalForwardBackward, reached through forwardBackwardGeneralized :84).
 * Inputs are token ids (the reference's one-hot rows, decoded).
 * Required outputs: loss, accuracy, grads[param_count].
 * Optional outputs (NULL to skip): logits/probs/dlogits [T*V],
 * output [T*D] (last block output), dout [T*D] (d loss / d last output),
 * layer_input_grads [L*T*D], head_probs [L*H*T*T].
 * Returns 0, or -1 on invalid configuration/tokens. */
int hxo_lm_forward_backward(const hxo_lm_config* c, const uint32_t* input_tokens,
                            const uint32_t* target_tokens, const float* params,
                            float* loss, float* accuracy, float* grads,
                            float* logits, float* probs, float* dlogits,
                            float* output, float* dout, float* layer_input_grads,
                            float* head_probs);

/* Batched step semantics of the reference driver
 * (qnn/qnn_transformer_training.cpp:7295-7333): for b < B, accumulate
 * grad_b * (1/B) into accum (float, registry order); mean loss in double.
 * tokens: [B, T+1] ids; sequence b uses ids[b][0..T-1] as input and
 * ids[b][1..T] as target.  grad_accum[param_count] is overwritten.
 * threads > 1 runs sequences concurrently (the accumulation stays in
 * sequence order, so results do not depend on the thread count). */
int hxo_lm_batch_gradients(const hxo_lm_config* c, int B, const uint32_t* tokens,
                           const float* params, float* grad_accum, float* mean_loss,
                           int threads);

/* tiny_lm::adamUpdate (tiny_language_model_cpu.cpp:124-145), elementwise over
 * a flat buffer.  Writes m_next, v_next, m_hat, v_hat (NULL allowed for the
 * hats) and w_next. */
void hxo_adam(size_t n, const float* w, const float* g, const float* m, const float* v,
              float lr, float beta1, float beta2, float eps, float c1, float c2,
              float* m_next, float* v_next, float* m_hat, float* v_hat, float* w_next);

/* Bias-correction scalars as the reference driver computes them
 * (qnn/qnn_transformer_training.cpp:1504-1507): c = float(1/(1-beta^t)) in
 * double. */
float hxo_adam_correction(double beta, int step);

/* ---- Muon (extension: no reference counterpart) -------------------------
 * Jordan et al. 2024, "Muon: An optimizer for hidden layers in neural
 * networks": momentum buffer buf = mu*buf + g; Nesterov update
 * u = g + mu*buf (or u = buf); X = u/(||u||_F + 1e-7); if rows > cols work on
 * X^T; 5 quintic Newton-Schulz iterations X <- aX + (bA + cA^2)X with A=XX^T;
 * w_next = w - lr * max(1, rows/cols)^0.5 * X.
 * bf16_inputs != 0 rounds every matrix-product operand to bfloat16
 * (round-to-nearest-even) before the product, with double accumulation. */
void hxo_muon(int rows, int cols, const float* w, const float* g, const float* buf,
              float lr, float momentum, int nesterov, int ns_steps,
              float a, float b, float c, int bf16_inputs,
              float* w_next, float* buf_next);

/* Round a float to the nearest bfloat16 (ties to even), returned as float. */
float hxo_round_bf16(float x);

/* ---- NPRTCKPTV2 / V3 checkpoint writer ------------------------------------
 * nprtSaveCheckpointV2 (qnn/qnn_transformer_training.cpp:5171-5252): magic
 * (V3 at vocabulary 1024 with the tokenizer block, else V2), eight big-endian
 * u32 (V T D F L H seed step), then the parameter, first-moment and
 * second-moment registries (u32 count; per entry u32 name length, name,
 * big-endian u64 count, raw float32) in parameterRegistry order
 * (tiny_language_model_cpu.cpp:63), plus "position_embedding" after
 * "token_embedding" for a learned-position model.  Returns the bytes the
 * file needs and writes them when out has room; returns 0 when the writer
 * refuses (step 0, non-finite state, tokenizer identity). */
size_t hxo_nprt_encode(const hxo_lm_config* c, uint32_t seed, uint32_t step, const char* kind,
                       const char* hash, const float* params, const float* m, const float* v,
                       uint8_t* out, size_t capacity);
/* nprtParameterHash (:5080-5090): FNV-1a 64 over (name, native u64 count,
 * values) of every parameter entry; writes "fnv1a64:%016llx". */
void hxo_nprt_parameter_hash(const hxo_lm_config* c, const float* params, char out[32]);
/* nprtTrainingOrder (:4983-4995): splitmix64 chain from 20260806. */
void hxo_nprt_training_order(uint64_t records, uint32_t steps, uint32_t batch, uint64_t* out);

/* ---- momentum SGD and training-stability modes -----------------------------
 * tiny_lm::momentumUpdate (tiny_language_model_cpu.cpp:123):
 * v' = momentum*v + g; w' = w - lr*v', in float, per element. */
void hxo_momentum(size_t n, const float* w, const float* g, const float* v, float lr, float momentum,
                  float* w_next, float* v_next);
/* stabilityLearningRate (training_stability.h:88-99). */
float hxo_stability_learning_rate(uint32_t mode, float base, uint32_t step, uint32_t total_steps);
/* applyInitStability (training_stability.h:104-121) on the flat layout. */
void hxo_apply_init_stability(const hxo_lm_config* c, uint32_t mode, float* params);
/* gradientNorm (qnn/qnn_transformer_training.cpp:888-938): per tensor a
 * sequential double sum of squares and its square root, summed as squares in
 * the order token_embedding, per layer wq wk wv wo g1 b1 g2 b2 w1 w2,
 * output_projection (a learned position table follows the embedding);
 * returns sqrt of that sum.  *clip receives min(1, threshold/(norm+1e-6))
 * for a finite positive norm and threshold > 0, else 1 (:2432-2439). */
double hxo_gradient_norm(const hxo_lm_config* c, const float* grads, float threshold, float* clip);

#ifdef __cplusplus
}
#endif
#endif
