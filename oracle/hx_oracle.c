/*
 * hx_oracle.c -- CPU restatement of HexaTrain's training-step arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY (the checker).  Only tests/, the smoke entry and
 * bench.py's cpu_baseline leg load this library; the product never does.
 *
 * Numerics: every routine keeps the reference's operation order and its
 * choice of double or float accumulators, so a build with the same flags as
 * the reference (-O2, no fast-math, no FMA contraction) reproduces the
 * reference's values exactly.  Comments name the reference line each block
 * follows (paths relative to the HexaTrain tree).
 */
#include "hx_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

/* ---------------------------------------------------------------------- */
/* Dense products with double accumulation.                                */
/* The reference's three helpers (tiny_language_model_cpu.cpp:15-17 mm/atb/
 * abt, and cpu::matMul in cpu_reference_training.cpp:129-142) all form
 * double(a)*b products and sum them in double over the inner index in
 * ascending order, then round once to float.  One strided kernel covers all
 * of them: out[i][j] = sum_z A(i,z) * B(z,j) with A(i,z) = a[i*ai + z*az] and
 * B(z,j) = b[z*bz + j*bj]. */
static void prod_dd(uint32_t rows, uint32_t cols, uint32_t inner,
                    const float* a, size_t ai, size_t az,
                    const float* b, size_t bz, size_t bj, float* out)
{
    for (uint32_t i = 0; i < rows; ++i) {
        for (uint32_t j = 0; j < cols; ++j) {
            double acc = 0.0;
            const float* pa = a + (size_t)i * ai;
            const float* pb = b + (size_t)j * bj;
            for (uint32_t z = 0; z < inner; ++z)
                acc += (double)pa[(size_t)z * az] * pb[(size_t)z * bz];
            out[(size_t)i * cols + j] = (float)acc;
        }
    }
}

/* out[r,c] = a[r,k] * b[k,c] (mm) */
static void mm(const float* a, const float* b, uint32_t r, uint32_t k, uint32_t c, float* out)
{
    prod_dd(r, c, k, a, k, 1, b, c, 1, out);
}
/* out[ka,cb] = a[r,ka]^T * b[r,cb] (atb) */
static void atb(const float* a, const float* b, uint32_t r, uint32_t ka, uint32_t cb, float* out)
{
    prod_dd(ka, cb, r, a, 1, ka, b, cb, 1, out);
}
/* out[ra,rb] = a[ra,k] * b[rb,k]^T (abt) */
static void abt(const float* a, const float* b, uint32_t ra, uint32_t rb, uint32_t k, float* out)
{
    prod_dd(ra, rb, k, a, k, 1, b, 1, k, out);
}

static void vadd(float* a, const float* b, size_t n)
{
    for (size_t i = 0; i < n; ++i) a[i] += b[i];
}

/* std::max(a, b) is (a < b) ? b : a; keep that exact form. */
static inline float stdmax(float a, float b) { return (a < b) ? b : a; }

/* ---------------------------------------------------------------------- */
/* MLP                                                                     */

void hxo_matmul(int M, int N, int K, const float* lhs, const float* rhs, float* out)
{
    prod_dd((uint32_t)M, (uint32_t)N, (uint32_t)K, lhs, (size_t)K, 1, rhs, (size_t)N, 1, out);
}

float hxo_mse(size_t n, const float* prediction, const float* target)
{
    /* cpu_reference_training.cpp:163-170: subtract in float, square-sum in
     * double, divide in double, round to float. */
    double sum = 0.0;
    for (size_t i = 0; i < n; ++i) {
        const float err = prediction[i] - target[i];
        sum += (double)err * err;
    }
    return (float)(sum / (double)n);
}

void hxo_sgd(size_t n, float* w, const float* dw, float lr)
{
    for (size_t i = 0; i < n; ++i) w[i] -= lr * dw[i];
}

float hxo_linear_forward_backward(int B, int D, const float* x, const float* target,
                                  const float* w, float* prediction, float* error,
                                  float* d_prediction, float* d_weight, float* d_input)
{
    const size_t n = (size_t)B * D;
    hxo_matmul(B, D, D, x, w, prediction);
    for (size_t i = 0; i < n; ++i) error[i] = prediction[i] - target[i];
    const float loss = hxo_mse(n, prediction, target);
    const float scale = 2.0f / (float)(B * D);
    for (size_t i = 0; i < n; ++i) d_prediction[i] = error[i] * scale;
    /* dW = X^T dP ; dX = dP W^T */
    prod_dd((uint32_t)D, (uint32_t)D, (uint32_t)B, x, 1, (size_t)D, d_prediction, (size_t)D, 1, d_weight);
    prod_dd((uint32_t)B, (uint32_t)D, (uint32_t)D, d_prediction, (size_t)D, 1, w, 1, (size_t)D, d_input);
    return loss;
}

int hxo_mlp_step(int B, int I, int H, int O,
                 const float* x, const float* y, const float* w1, const float* w2,
                 float lr, float* loss, float* w1_next, float* w2_next,
                 float* z1, float* h, float* p, float* e, float* dp,
                 float* dw2, float* dh, unsigned char* mask, float* dz1, float* dw1)
{
    if (B <= 0 || I <= 0 || H <= 0 || O <= 0) return -1;
    const size_t bh = (size_t)B * H, bo = (size_t)B * O;
    /* pass(): qnn/qnn_mlp_training.cpp:53-72 */
    hxo_matmul(B, H, I, x, w1, z1);                                   /* Z1 = X W1 */
    for (size_t i = 0; i < bh; ++i) h[i] = stdmax(0.0f, z1[i]);        /* H = ReLU */
    hxo_matmul(B, O, H, h, w2, p);                                    /* P = H W2 */
    for (size_t i = 0; i < bo; ++i) e[i] = p[i] - y[i];               /* E = P - Y */
    *loss = hxo_mse(bo, p, y);                                        /* mean(E^2) */
    const float s = 2.0f / (float)(B * O);
    for (size_t i = 0; i < bo; ++i) dp[i] = (p[i] - y[i]) * s;        /* dP */
    /* dW2 = H^T dP  [H,O] */
    prod_dd((uint32_t)H, (uint32_t)O, (uint32_t)B, h, 1, (size_t)H, dp, (size_t)O, 1, dw2);
    /* dH = dP W2^T  [B,H] with the pre-update W2 */
    prod_dd((uint32_t)B, (uint32_t)H, (uint32_t)O, dp, (size_t)O, 1, w2, 1, (size_t)O, dh);
    for (size_t i = 0; i < bh; ++i) {
        mask[i] = h[i] > 0.0f ? 1 : 0;                                /* full_relu_greater */
        dz1[i] = h[i] > 0 ? dh[i] : 0;                                /* full_relu_select */
    }
    /* dW1 = X^T dZ1 [I,H] */
    prod_dd((uint32_t)I, (uint32_t)H, (uint32_t)B, x, 1, (size_t)I, dz1, (size_t)H, 1, dw1);
    /* SGD on copies of the current weights (cpu::sgdUpdate) */
    memcpy(w1_next, w1, sizeof(float) * (size_t)I * H);
    memcpy(w2_next, w2, sizeof(float) * (size_t)H * O);
    hxo_sgd((size_t)I * H, w1_next, dw1, lr);
    hxo_sgd((size_t)H * O, w2_next, dw2, lr);
    return 0;
}

/* ---------------------------------------------------------------------- */
/* LM layout                                                               */

static int valid_config(const hxo_lm_config* c)
{
    /* transformer_resource_estimator.h:76-83: every dimension >= 1 and
     * D divisible by H. */
    if (!c || !c->vocab || !c->tokens || !c->dim || !c->ffn || !c->layers || !c->heads) return 0;
    if (c->dim % c->heads) return 0;
    return 1;
}

int hxo_lm_layout(const hxo_lm_config* c, size_t* offsets, size_t* sizes, int cap)
{
    const size_t V = c->vocab, T = c->tokens, D = c->dim, F = c->ffn;
    size_t tensor_sizes[4 + 10 * 64];
    int n = 0;
    if (c->layers > 64) return -1;
    tensor_sizes[n++] = V * D;
    if (c->learned_position) tensor_sizes[n++] = T * D;
    for (uint32_t l = 0; l < c->layers; ++l) {
        const size_t per[10] = {D, D, D * D, D * D, D * D, D * D, D, D, D * F, F * D};
        for (int k = 0; k < 10; ++k) tensor_sizes[n++] = per[k];
    }
    tensor_sizes[n++] = D * V;
    size_t off = 0;
    for (int i = 0; i < n; ++i) {
        if (i < cap) {
            if (offsets) offsets[i] = off;
            if (sizes) sizes[i] = tensor_sizes[i];
        }
        off += tensor_sizes[i];
    }
    return n;
}

size_t hxo_lm_param_count(const hxo_lm_config* c)
{
    const size_t V = c->vocab, T = c->tokens, D = c->dim, F = c->ffn;
    return 2 * V * D + (c->learned_position ? T * D : 0) +
           (size_t)c->layers * (4 * D * D + 4 * D + 2 * D * F);
}

typedef struct {
    const float *g1, *b1, *wq, *wk, *wv, *wo, *g2, *b2, *w1, *w2;
} layer_view;

typedef struct {
    float *g1, *b1, *wq, *wk, *wv, *wo, *g2, *b2, *w1, *w2;
} layer_grad_view;

static size_t layer_base(const hxo_lm_config* c, uint32_t l)
{
    const size_t V = c->vocab, T = c->tokens, D = c->dim, F = c->ffn;
    return V * D + (c->learned_position ? T * D : 0) + (size_t)l * (4 * D * D + 4 * D + 2 * D * F);
}

static void make_layer_view(const hxo_lm_config* c, const float* p, uint32_t l, layer_view* v)
{
    const size_t D = c->dim, F = c->ffn;
    const float* q = p + layer_base(c, l);
    v->g1 = q; q += D;
    v->b1 = q; q += D;
    v->wq = q; q += D * D;
    v->wk = q; q += D * D;
    v->wv = q; q += D * D;
    v->wo = q; q += D * D;
    v->g2 = q; q += D;
    v->b2 = q; q += D;
    v->w1 = q; q += D * F;
    v->w2 = q;
}

static void make_grad_view(const hxo_lm_config* c, float* p, uint32_t l, layer_grad_view* v)
{
    layer_view tmp;
    make_layer_view(c, p, l, &tmp);
    v->g1 = (float*)tmp.g1; v->b1 = (float*)tmp.b1; v->wq = (float*)tmp.wq; v->wk = (float*)tmp.wk;
    v->wv = (float*)tmp.wv; v->wo = (float*)tmp.wo; v->g2 = (float*)tmp.g2; v->b2 = (float*)tmp.b2;
    v->w1 = (float*)tmp.w1; v->w2 = (float*)tmp.w2;
}

void hxo_lm_fixed_position(const hxo_lm_config* c, float* out)
{
    /* tiny_language_model_cpu.cpp:68: f = 10000^(-(d&~1)/D) in float,
     * sin for even d, cos for odd d, times 0.05. */
    for (uint32_t t = 0; t < c->tokens; ++t)
        for (uint32_t d = 0; d < c->dim; ++d) {
            const float f = powf(10000.f, -(float)(d & ~1u) / (float)c->dim);
            out[(size_t)t * c->dim + d] =
                ((d & 1u) ? cosf((float)t * f) : sinf((float)t * f)) * .05f;
        }
}

/* ---------------------------------------------------------------------- */
/* LayerNorm forward/backward: tiny_language_model_cpu.cpp:36 (nf), :37 (nb). */

typedef struct {
    float* xhat;   /* [T*D] */
    float* inv;    /* [T]   */
    float* out;    /* [T*D] */
} ln_state;

static void ln_forward(uint32_t T, uint32_t D, float eps, const float* x,
                       const float* g, const float* b, ln_state* n)
{
    for (uint32_t r = 0; r < T; ++r) {
        const float* xr = x + (size_t)r * D;
        double m = 0, v = 0;
        for (uint32_t d = 0; d < D; ++d) m += xr[d];
        m /= D;
        for (uint32_t d = 0; d < D; ++d) {
            const double z = xr[d] - m;
            v += z * z;
        }
        v /= D;
        n->inv[r] = (float)(1 / sqrt(v + eps));
        for (uint32_t d = 0; d < D; ++d) {
            const size_t i = (size_t)r * D + d;
            n->xhat[i] = (x[i] - (float)m) * n->inv[r];
            n->out[i] = n->xhat[i] * g[d] + b[d];
        }
    }
}

/* dx[T*D] is overwritten; dg/db[D] are overwritten (accumulated over rows). */
static void ln_backward(uint32_t T, uint32_t D, const float* dy, const ln_state* n,
                        const float* g, float* dx, float* dg, float* db)
{
    for (uint32_t d = 0; d < D; ++d) { dg[d] = 0; db[d] = 0; }
    for (uint32_t r = 0; r < T; ++r) {
        double s = 0, sx = 0;
        for (uint32_t d = 0; d < D; ++d) {
            const size_t i = (size_t)r * D + d;
            const double z = dy[i] * g[d];
            s += z;
            sx += z * n->xhat[i];
            dg[d] += dy[i] * n->xhat[i];
            db[d] += dy[i];
        }
        for (uint32_t d = 0; d < D; ++d) {
            const size_t i = (size_t)r * D + d;
            const double z = dy[i] * g[d];
            dx[i] = (float)(n->inv[r] / D * (D * z - s - n->xhat[i] * sx));
        }
    }
}

/* ---------------------------------------------------------------------- */
/* LM forward + backward for one sequence.                                 */

typedef struct {
    float *x, *q, *k, *v, *prob, *ctx, *r1, *f1, *relu, *out;
    ln_state n1, n2;
} layer_acts;

static float* alloc_f(size_t n) { return (float*)calloc(n ? n : 1, sizeof(float)); }

int hxo_lm_forward_backward(const hxo_lm_config* c, const uint32_t* input_tokens,
                            const uint32_t* target_tokens, const float* params,
                            float* loss_out, float* accuracy_out, float* grads,
                            float* logits_out, float* probs_out, float* dlogits_out,
                            float* output_out, float* dout_out, float* layer_input_grads,
                            float* head_probs)
{
    if (!valid_config(c)) return -1;
    const uint32_t V = c->vocab, T = c->tokens, D = c->dim, F = c->ffn, L = c->layers, H = c->heads;
    const uint32_t dh = D / H;
    for (uint32_t t = 0; t < T; ++t)
        if (input_tokens[t] >= V || target_tokens[t] >= V) return -1;
    const size_t TD = (size_t)T * D, TF = (size_t)T * F, TV = (size_t)T * V, TT = (size_t)T * T;
    const float* E = params;
    const float* learned_pos = c->learned_position ? params + (size_t)V * D : NULL;
    const float* Wout = params + hxo_lm_param_count(c) - (size_t)D * V;

    layer_acts* acts = (layer_acts*)calloc(L, sizeof(layer_acts));
    for (uint32_t l = 0; l < L; ++l) {
        layer_acts* a = &acts[l];
        a->x = alloc_f(TD); a->q = alloc_f(TD); a->k = alloc_f(TD); a->v = alloc_f(TD);
        a->prob = alloc_f((size_t)H * TT); a->ctx = alloc_f(TD); a->r1 = alloc_f(TD);
        a->f1 = alloc_f(TF); a->relu = alloc_f(TF); a->out = alloc_f(TD);
        a->n1.xhat = alloc_f(TD); a->n1.inv = alloc_f(T); a->n1.out = alloc_f(TD);
        a->n2.xhat = alloc_f(TD); a->n2.inv = alloc_f(T); a->n2.out = alloc_f(TD);
    }
    float* x = alloc_f(TD);
    float* tmp = alloc_f(TD > TF ? (TD > TT ? TD : TT) : (TF > TT ? TF : TT));
    float* logits = alloc_f(TV);
    float* prob = alloc_f(TV);
    float* dlogits = alloc_f(TV);

    /* Embedding: one-hot(tokens) * E is E[token] exactly (each double sum has
     * a single non-zero term), plus the position table
     * (tiny_language_model_cpu.cpp:42). */
    if (learned_pos) {
        for (uint32_t t = 0; t < T; ++t)
            for (uint32_t d = 0; d < D; ++d)
                x[(size_t)t * D + d] = E[(size_t)input_tokens[t] * D + d] + learned_pos[(size_t)t * D + d];
    } else {
        float* pos = alloc_f(TD);
        hxo_lm_fixed_position(c, pos);
        for (uint32_t t = 0; t < T; ++t)
            for (uint32_t d = 0; d < D; ++d)
                x[(size_t)t * D + d] = E[(size_t)input_tokens[t] * D + d] + pos[(size_t)t * D + d];
        free(pos);
    }

    /* Blocks (tiny_language_model_cpu.cpp:44-47). */
    const float scale = 1 / sqrtf((float)dh);
    for (uint32_t l = 0; l < L; ++l) {
        layer_view p;
        make_layer_view(c, params, l, &p);
        layer_acts* z = &acts[l];
        memcpy(z->x, x, sizeof(float) * TD);
        ln_forward(T, D, c->eps, x, p.g1, p.b1, &z->n1);
        mm(z->n1.out, p.wq, T, D, D, z->q);
        mm(z->n1.out, p.wk, T, D, D, z->k);
        mm(z->n1.out, p.wv, T, D, D, z->v);
        if (H == 1) {
            abt(z->q, z->k, T, T, D, tmp); /* scores */
            for (uint32_t r = 0; r < T; ++r) {
                float mx = -INFINITY;
                for (uint32_t j = 0; j <= r; ++j) mx = stdmax(mx, tmp[(size_t)r * T + j] * scale);
                double sum = 0;
                for (uint32_t j = 0; j <= r; ++j) {
                    const float e = expf(tmp[(size_t)r * T + j] * scale - mx);
                    z->prob[(size_t)r * T + j] = e;
                    sum += e;
                }
                for (uint32_t j = 0; j <= r; ++j) z->prob[(size_t)r * T + j] /= (float)sum;
            }
            mm(z->prob, z->v, T, T, D, z->ctx);
        } else {
            for (uint32_t h = 0; h < H; ++h)
                for (uint32_t r = 0; r < T; ++r) {
                    const size_t base = ((size_t)h * T + r) * T;
                    float mx = -INFINITY;
                    for (uint32_t j = 0; j <= r; ++j) {
                        double s = 0;
                        for (uint32_t d = 0; d < dh; ++d)
                            s += (double)z->q[(size_t)r * D + h * dh + d] * z->k[(size_t)j * D + h * dh + d];
                        mx = stdmax(mx, (float)s * scale);
                    }
                    double sum = 0;
                    for (uint32_t j = 0; j <= r; ++j) {
                        double s = 0;
                        for (uint32_t d = 0; d < dh; ++d)
                            s += (double)z->q[(size_t)r * D + h * dh + d] * z->k[(size_t)j * D + h * dh + d];
                        const float e = expf((float)s * scale - mx);
                        z->prob[base + j] = e;
                        sum += e;
                    }
                    for (uint32_t j = 0; j <= r; ++j) {
                        const float a = z->prob[base + j] / (float)sum;
                        z->prob[base + j] = a;
                        for (uint32_t d = 0; d < dh; ++d)
                            z->ctx[(size_t)r * D + h * dh + d] += a * z->v[(size_t)j * D + h * dh + d];
                    }
                }
        }
        memcpy(z->r1, x, sizeof(float) * TD);
        mm(z->ctx, p.wo, T, D, D, tmp);
        vadd(z->r1, tmp, TD);
        ln_forward(T, D, c->eps, z->r1, p.g2, p.b2, &z->n2);
        mm(z->n2.out, p.w1, T, D, F, z->f1);
        for (size_t i = 0; i < TF; ++i) z->relu[i] = stdmax(0.f, z->f1[i]);
        memcpy(z->out, z->r1, sizeof(float) * TD);
        mm(z->relu, p.w2, T, F, D, tmp);
        vadd(z->out, tmp, TD);
        memcpy(x, z->out, sizeof(float) * TD);
    }

    /* Head and softmax (tiny_language_model_cpu.cpp:48). */
    mm(x, Wout, T, D, V, logits);
    for (uint32_t r = 0; r < T; ++r) {
        const size_t b = (size_t)r * V;
        float mx = logits[b];
        for (uint32_t j = 1; j < V; ++j) if (mx < logits[b + j]) mx = logits[b + j];
        double s = 0;
        for (uint32_t j = 0; j < V; ++j) {
            const float e = expf(logits[b + j] - mx);
            prob[b + j] = e;
            s += e;
        }
        for (uint32_t j = 0; j < V; ++j) prob[b + j] /= (float)s;
    }

    /* Loss, accuracy and dLogits (tiny_language_model_cpu.cpp:77). */
    double loss = 0;
    uint32_t correct = 0;
    for (uint32_t row = 0; row < T; ++row) {
        const size_t b = (size_t)row * V;
        float mx = logits[b];
        uint32_t pred = 0;
        const uint32_t truth = target_tokens[row];
        for (uint32_t j = 0; j < V; ++j) {
            if (logits[b + j] > mx) { mx = logits[b + j]; pred = j; }
            const float target = (j == truth) ? 1.0f : 0.0f;
            dlogits[b + j] = (prob[b + j] - target) / (float)T;
        }
        double s = 0;
        for (uint32_t j = 0; j < V; ++j) s += exp((double)(logits[b + j] - mx));
        loss += mx + log(s) - logits[b + truth];
        correct += pred == truth;
    }
    *loss_out = (float)(loss / T);
    if (accuracy_out) *accuracy_out = (float)correct / T;

    /* Backward (tiny_language_model_cpu.cpp:79-82). */
    memset(grads, 0, sizeof(float) * hxo_lm_param_count(c));
    float* gWout = grads + hxo_lm_param_count(c) - (size_t)D * V;
    atb(x, dlogits, T, D, V, gWout);
    float* dout = alloc_f(TD);
    abt(dlogits, Wout, T, D, V, dout);
    if (dout_out) memcpy(dout_out, dout, sizeof(float) * TD);

    float* drelu = alloc_f(TF);
    float* df1 = alloc_f(TF);
    float* dn2 = alloc_f(TD);
    float* drn = alloc_f(TD);
    float* dr = alloc_f(TD);
    float* dc = alloc_f(TD);
    float* dq = alloc_f(TD);
    float* dk = alloc_f(TD);
    float* dv = alloc_f(TD);
    float* dn1 = alloc_f(TD);
    float* dxn = alloc_f(TD);
    float* dap = alloc_f(TT);
    float* ds = alloc_f(TT);

    for (uint32_t li = L; li-- > 0;) {
        const layer_acts* z = &acts[li];
        layer_view p;
        layer_grad_view d;
        make_layer_view(c, params, li, &p);
        make_grad_view(c, grads, li, &d);
        atb(z->relu, dout, T, F, D, d.w2);
        abt(dout, p.w2, T, F, D, drelu);
        for (size_t i = 0; i < TF; ++i) df1[i] = z->f1[i] > 0 ? drelu[i] : 0;
        atb(z->n2.out, df1, T, D, F, d.w1);
        abt(df1, p.w1, T, D, F, dn2);
        ln_backward(T, D, dn2, &z->n2, p.g2, drn, d.g2, d.b2);
        memcpy(dr, dout, sizeof(float) * TD);
        vadd(dr, drn, TD);
        atb(z->ctx, dr, T, D, D, d.wo);
        abt(dr, p.wo, T, D, D, dc);
        memset(dq, 0, sizeof(float) * TD);
        memset(dk, 0, sizeof(float) * TD);
        memset(dv, 0, sizeof(float) * TD);
        if (H == 1) {
            abt(dc, z->v, T, T, D, dap);
            atb(z->prob, dc, T, T, D, dv);
            for (uint32_t rr = 0; rr < T; ++rr) {
                double dot = 0;
                for (uint32_t j = 0; j < T; ++j) dot += dap[(size_t)rr * T + j] * z->prob[(size_t)rr * T + j];
                for (uint32_t j = 0; j < T; ++j)
                    ds[(size_t)rr * T + j] = z->prob[(size_t)rr * T + j] * (dap[(size_t)rr * T + j] - (float)dot);
            }
            mm(ds, z->k, T, T, D, dq);
            atb(ds, z->q, T, T, D, dk);
            const float sc = 1 / sqrtf((float)dh);
            for (size_t i = 0; i < TD; ++i) dq[i] *= sc;
            for (size_t i = 0; i < TD; ++i) dk[i] *= sc;
        } else {
            const float root = sqrtf((float)dh);
            for (uint32_t h = 0; h < H; ++h) {
                memset(dap, 0, sizeof(float) * TT);
                for (uint32_t rr = 0; rr < T; ++rr)
                    for (uint32_t j = 0; j < T; ++j)
                        for (uint32_t e = 0; e < dh; ++e)
                            dap[(size_t)rr * T + j] += dc[(size_t)rr * D + h * dh + e] * z->v[(size_t)j * D + h * dh + e];
                for (uint32_t rr = 0; rr < T; ++rr) {
                    double dot = 0;
                    const size_t pb = ((size_t)h * T + rr) * T;
                    for (uint32_t j = 0; j < T; ++j) dot += dap[(size_t)rr * T + j] * z->prob[pb + j];
                    for (uint32_t j = 0; j < T; ++j) {
                        ds[(size_t)rr * T + j] = z->prob[pb + j] * (dap[(size_t)rr * T + j] - (float)dot);
                        for (uint32_t e = 0; e < dh; ++e)
                            dv[(size_t)j * D + h * dh + e] += z->prob[pb + j] * dc[(size_t)rr * D + h * dh + e];
                    }
                }
                for (uint32_t rr = 0; rr < T; ++rr)
                    for (uint32_t j = 0; j < T; ++j)
                        for (uint32_t e = 0; e < dh; ++e) {
                            dq[(size_t)rr * D + h * dh + e] += ds[(size_t)rr * T + j] * z->k[(size_t)j * D + h * dh + e] / root;
                            dk[(size_t)j * D + h * dh + e] += ds[(size_t)rr * T + j] * z->q[(size_t)rr * D + h * dh + e] / root;
                        }
            }
        }
        atb(z->n1.out, dq, T, D, D, d.wq);
        atb(z->n1.out, dk, T, D, D, d.wk);
        atb(z->n1.out, dv, T, D, D, d.wv);
        abt(dq, p.wq, T, D, D, dn1);
        abt(dk, p.wk, T, D, D, tmp);
        vadd(dn1, tmp, TD);
        abt(dv, p.wv, T, D, D, tmp);
        vadd(dn1, tmp, TD);
        ln_backward(T, D, dn1, &z->n1, p.g1, dxn, d.g1, d.b1);
        memcpy(dout, dr, sizeof(float) * TD);
        vadd(dout, dxn, TD);
        if (layer_input_grads) memcpy(layer_input_grads + (size_t)li * TD, dout, sizeof(float) * TD);
    }

    /* Token embedding gradient: one-hot^T * dX0 (tiny_language_model_cpu.cpp:82),
     * i.e. per vocabulary row the double sum of the matching rows of dX0 in
     * row order.  The learned position table (extension) receives dX0. */
    for (uint32_t vv = 0; vv < V; ++vv)
        for (uint32_t d = 0; d < D; ++d) {
            double acc = 0.0;
            int any = 0;
            for (uint32_t t = 0; t < T; ++t)
                if (input_tokens[t] == vv) { acc += (double)dout[(size_t)t * D + d]; any = 1; }
            grads[(size_t)vv * D + d] = any ? (float)acc : 0.0f;
        }
    if (c->learned_position) memcpy(grads + (size_t)V * D, dout, sizeof(float) * TD);

    if (logits_out) memcpy(logits_out, logits, sizeof(float) * TV);
    if (probs_out) memcpy(probs_out, prob, sizeof(float) * TV);
    if (dlogits_out) memcpy(dlogits_out, dlogits, sizeof(float) * TV);
    if (output_out) memcpy(output_out, x, sizeof(float) * TD);
    if (head_probs)
        for (uint32_t l = 0; l < L; ++l)
            memcpy(head_probs + (size_t)l * H * TT, acts[l].prob, sizeof(float) * H * TT);

    free(drelu); free(df1); free(dn2); free(drn); free(dr); free(dc); free(dq); free(dk);
    free(dv); free(dn1); free(dxn); free(dap); free(ds); free(dout);
    for (uint32_t l = 0; l < L; ++l) {
        layer_acts* a = &acts[l];
        free(a->x); free(a->q); free(a->k); free(a->v); free(a->prob); free(a->ctx); free(a->r1);
        free(a->f1); free(a->relu); free(a->out);
        free(a->n1.xhat); free(a->n1.inv); free(a->n1.out);
        free(a->n2.xhat); free(a->n2.inv); free(a->n2.out);
    }
    free(acts); free(x); free(tmp); free(logits); free(prob); free(dlogits);
    return 0;
}

/* ---------------------------------------------------------------------- */
/* Batched gradients: the reference driver's accumulate loop.              */

typedef struct {
    const hxo_lm_config* c;
    const uint32_t* tokens;
    const float* params;
    float* grads;        /* [B][P] */
    float* losses;       /* [B] */
    int B, first, stride;
    int status;
} batch_job;

static void* batch_worker(void* arg)
{
    batch_job* j = (batch_job*)arg;
    const size_t P = hxo_lm_param_count(j->c);
    const uint32_t T = j->c->tokens;
    for (int b = j->first; b < j->B; b += j->stride) {
        const uint32_t* seq = j->tokens + (size_t)b * (T + 1);
        float acc;
        if (hxo_lm_forward_backward(j->c, seq, seq + 1, j->params, &j->losses[b], &acc,
                                    j->grads + (size_t)b * P, NULL, NULL, NULL, NULL, NULL,
                                    NULL, NULL) != 0)
            j->status = -1;
    }
    return NULL;
}

int hxo_lm_batch_gradients(const hxo_lm_config* c, int B, const uint32_t* tokens,
                           const float* params, float* grad_accum, float* mean_loss,
                           int threads)
{
    if (!valid_config(c) || B <= 0) return -1;
    if (threads < 1) threads = 1;
    if (threads > B) threads = B;
    const size_t P = hxo_lm_param_count(c);
    float* grads = (float*)malloc(sizeof(float) * P * (size_t)B);
    float* losses = (float*)malloc(sizeof(float) * (size_t)B);
    if (!grads || !losses) { free(grads); free(losses); return -1; }
    batch_job* jobs = (batch_job*)calloc((size_t)threads, sizeof(batch_job));
    pthread_t* tids = (pthread_t*)calloc((size_t)threads, sizeof(pthread_t));
    for (int t = 0; t < threads; ++t) {
        jobs[t] = (batch_job){c, tokens, params, grads, losses, B, t, threads, 0};
        if (t > 0) pthread_create(&tids[t], NULL, batch_worker, &jobs[t]);
    }
    batch_worker(&jobs[0]);
    int status = jobs[0].status;
    for (int t = 1; t < threads; ++t) {
        pthread_join(tids[t], NULL);
        if (jobs[t].status) status = jobs[t].status;
    }
    /* accum[j] += grad_b[j] * (1/B) in sequence order
     * (qnn/qnn_transformer_training.cpp:7322-7330); loss mean in double. */
    memset(grad_accum, 0, sizeof(float) * P);
    const float inv = 1.0f / (float)B;
    double loss_sum = 0;
    for (int b = 0; b < B; ++b) {
        const float* g = grads + (size_t)b * P;
        for (size_t i = 0; i < P; ++i) grad_accum[i] += g[i] * inv;
        loss_sum += losses[b];
    }
    *mean_loss = (float)(loss_sum / B);
    free(grads); free(losses); free(jobs); free(tids);
    return status;
}

/* ---------------------------------------------------------------------- */
/* Adam                                                                    */

void hxo_adam(size_t n, const float* w, const float* g, const float* m, const float* v,
              float lr, float beta1, float beta2, float eps, float c1, float c2,
              float* m_next, float* v_next, float* m_hat, float* v_hat, float* w_next)
{
    /* tiny_language_model_cpu.cpp:124-145 */
    for (size_t i = 0; i < n; ++i) {
        const float nm = beta1 * m[i] + (1 - beta1) * g[i];
        const float nv = beta2 * v[i] + (1 - beta2) * g[i] * g[i];
        const float mh = nm * c1;
        const float vh = nv * c2;
        m_next[i] = nm;
        v_next[i] = nv;
        if (m_hat) m_hat[i] = mh;
        if (v_hat) v_hat[i] = vh;
        w_next[i] = w[i] - lr * mh / (sqrtf(vh) + eps);
    }
}

float hxo_adam_correction(double beta, int step)
{
    return (float)(1.0 / (1.0 - pow(beta, (double)step)));
}

/* ---------------------------------------------------------------------- */
/* Muon (extension; restates the published method, no reference code).     */

float hxo_round_bf16(float x)
{
    uint32_t u;
    memcpy(&u, &x, 4);
    if ((u & 0x7f800000u) == 0x7f800000u) { /* inf/nan: truncate, keep nan quiet */
        if (u & 0x007fffffu) u |= 0x00400000u;
        u &= 0xffff0000u;
    } else {
        const uint32_t lsb = (u >> 16) & 1u;
        u += 0x7fffu + lsb;
        u &= 0xffff0000u;
    }
    float r;
    memcpy(&r, &u, 4);
    return r;
}

/* out[m,n] = sum_k op(a)[m,k] op(b)[k,n], double accumulation, operands
 * optionally rounded to bf16.  a: [m,k] row-major, b: [k,n] row-major. */
static void ns_prod(int m, int n, int k, const float* a, const float* b, int bf16, float* out)
{
    for (int i = 0; i < m; ++i)
        for (int j = 0; j < n; ++j) {
            double acc = 0;
            for (int z = 0; z < k; ++z) {
                float x = a[(size_t)i * k + z], y = b[(size_t)z * n + j];
                if (bf16) { x = hxo_round_bf16(x); y = hxo_round_bf16(y); }
                acc += (double)x * y;
            }
            out[(size_t)i * n + j] = (float)acc;
        }
}

void hxo_muon(int rows, int cols, const float* w, const float* g, const float* buf,
              float lr, float momentum, int nesterov, int ns_steps,
              float a, float b, float c, int bf16_inputs,
              float* w_next, float* buf_next)
{
    const size_t n = (size_t)rows * cols;
    float* u = alloc_f(n);
    for (size_t i = 0; i < n; ++i) {
        buf_next[i] = momentum * buf[i] + g[i];
        u[i] = nesterov ? g[i] + momentum * buf_next[i] : buf_next[i];
    }
    double fro = 0;
    for (size_t i = 0; i < n; ++i) fro += (double)u[i] * u[i];
    const float inv = (float)(1.0 / (sqrt(fro) + 1e-7));
    const int tr = rows > cols;
    const int R = tr ? cols : rows, C = tr ? rows : cols; /* X is [R,C], R <= C */
    float* X = alloc_f(n);
    for (int i = 0; i < rows; ++i)
        for (int j = 0; j < cols; ++j) {
            const float val = u[(size_t)i * cols + j] * inv;
            if (tr) X[(size_t)j * C + i] = val; else X[(size_t)i * C + j] = val;
        }
    float* Xt = alloc_f(n);
    float* A = alloc_f((size_t)R * R);
    float* A2 = alloc_f((size_t)R * R);
    float* Bm = alloc_f((size_t)R * R);
    float* BX = alloc_f(n);
    for (int it = 0; it < ns_steps; ++it) {
        for (int i = 0; i < R; ++i)
            for (int j = 0; j < C; ++j) Xt[(size_t)j * R + i] = X[(size_t)i * C + j];
        ns_prod(R, R, C, X, Xt, bf16_inputs, A);          /* A = X X^T */
        ns_prod(R, R, R, A, A, bf16_inputs, A2);          /* A^2 */
        for (size_t i = 0; i < (size_t)R * R; ++i) Bm[i] = b * A[i] + c * A2[i];
        ns_prod(R, C, R, Bm, X, bf16_inputs, BX);         /* B X */
        for (size_t i = 0; i < n; ++i) X[i] = a * X[i] + BX[i];
    }
    const float sc = (float)sqrt(fmax(1.0, (double)rows / (double)cols));
    for (int i = 0; i < rows; ++i)
        for (int j = 0; j < cols; ++j) {
            const float xo = tr ? X[(size_t)j * C + i] : X[(size_t)i * C + j];
            w_next[(size_t)i * cols + j] = w[(size_t)i * cols + j] - lr * (sc * xo);
        }
    free(u); free(X); free(Xt); free(A); free(A2); free(Bm); free(BX);
}

/* ---------------------------------------------------------------------- */
/* NPRTCKPTV2 / V3 writer (qnn/qnn_transformer_training.cpp:5123-5131 for   */
/* the big-endian integers, :5171-5252 for the file).                       */

/* Registry entry k of the layout above: its name and element count;
 * returns 0 past the end. */
static int nprt_entry(const hxo_lm_config* c, uint32_t k, char name[40], uint64_t* count)
{
    static const char* const kLayer[10] = {"norm1_gamma", "norm1_beta", "wq", "wk", "wv",
                                           "wo", "norm2_gamma", "norm2_beta", "ffn_w1", "ffn_w2"};
    const uint64_t V = c->vocab, T = c->tokens, D = c->dim, F = c->ffn;
    const uint64_t sizes[10] = {D, D, D * D, D * D, D * D, D * D, D, D, D * F, F * D};
    if (k == 0) { strcpy(name, "token_embedding"); *count = V * D; return 1; }
    k -= 1;
    if (c->learned_position) {
        if (k == 0) { strcpy(name, "position_embedding"); *count = T * D; return 1; }
        k -= 1;
    }
    if (k < 10u * c->layers) {
        char buf[40];
        snprintf(buf, sizeof buf, "layer_%03u.%s", k / 10, kLayer[k % 10]);
        strcpy(name, buf);
        *count = sizes[k % 10];
        return 1;
    }
    if (k == 10u * c->layers) { strcpy(name, "output_projection"); *count = D * V; return 1; }
    return 0;
}

static void put_be(uint8_t* out, size_t capacity, size_t* at, uint64_t v, int bytes)
{
    for (int s = 8 * (bytes - 1); s >= 0; s -= 8) {
        if (*at < capacity && out) out[*at] = (uint8_t)(v >> s);
        ++*at;
    }
}

static void put_raw(uint8_t* out, size_t capacity, size_t* at, const void* src, size_t n)
{
    if (out && *at + n <= capacity) memcpy(out + *at, src, n);
    *at += n;
}

size_t hxo_nprt_encode(const hxo_lm_config* c, uint32_t seed, uint32_t step, const char* kind,
                       const char* hash, const float* params, const float* m, const float* v,
                       uint8_t* out, size_t capacity)
{
    const size_t n = hxo_lm_param_count(c);
    const int v3 = c->vocab == 1024;
    const char* k = kind ? kind : "";
    const char* h = hash ? hash : "";
    if (step == 0) return 0;
    for (size_t i = 0; i < n; ++i)
        if (!isfinite(params[i]) || !isfinite(m[i]) || !isfinite(v[i])) return 0;
    if (v3 && (strcmp(k, "byte_bpe") != 0 || strlen(h) != 71 || strncmp(h, "sha256:", 7) != 0)) return 0;
    if (!v3 && (*k || *h)) return 0;
    size_t at = 0;
    put_raw(out, capacity, &at, v3 ? "NPRTCKPTV3\n" : "NPRTCKPTV2\n", 11);
    const uint32_t head[8] = {c->vocab, c->tokens, c->dim, c->ffn, c->layers, c->heads, seed, step};
    for (int i = 0; i < 8; ++i) put_be(out, capacity, &at, head[i], 4);
    if (v3) {
        put_be(out, capacity, &at, strlen(k), 4);
        put_raw(out, capacity, &at, k, strlen(k));
        put_be(out, capacity, &at, strlen(h), 4);
        put_raw(out, capacity, &at, h, strlen(h));
    }
    const uint32_t entries = 2 + (c->learned_position ? 1 : 0) + 10 * c->layers;
    const float* regs[3] = {params, m, v};
    for (int r = 0; r < 3; ++r) {
        put_be(out, capacity, &at, entries, 4);
        size_t off = 0;
        char name[40];
        uint64_t count;
        for (uint32_t e = 0; nprt_entry(c, e, name, &count); ++e) {
            put_be(out, capacity, &at, strlen(name), 4);
            put_raw(out, capacity, &at, name, strlen(name));
            put_be(out, capacity, &at, count, 8);
            put_raw(out, capacity, &at, regs[r] + off, count * sizeof(float));
            off += count;
        }
    }
    return at;
}

static uint64_t fnv1a(uint64_t h, const void* p, size_t n)
{
    const uint8_t* b = (const uint8_t*)p;
    for (size_t i = 0; i < n; ++i) {
        h ^= b[i];
        h *= 1099511628211ull;
    }
    return h;
}

void hxo_nprt_parameter_hash(const hxo_lm_config* c, const float* params, char out[32])
{
    uint64_t h = 14695981039346656037ull;
    size_t off = 0;
    char name[40];
    uint64_t count;
    for (uint32_t e = 0; nprt_entry(c, e, name, &count); ++e) {
        h = fnv1a(h, name, strlen(name));
        h = fnv1a(h, &count, sizeof count);
        h = fnv1a(h, params + off, count * sizeof(float));
        off += count;
    }
    snprintf(out, 32, "fnv1a64:%016llx", (unsigned long long)h);
}

void hxo_nprt_training_order(uint64_t records, uint32_t steps, uint32_t batch, uint64_t* out)
{
    uint64_t state = 20260806;
    for (uint64_t i = 0; i < (uint64_t)steps * batch; ++i) {
        uint64_t x = state + i + 0x9e3779b97f4a7c15ull;
        x = (x ^ (x >> 30)) * 0xbf58476d1ce4e5b9ull;
        x = (x ^ (x >> 27)) * 0x94d049bb133111ebull;
        state = x ^ (x >> 31);
        out[i] = state % records;
    }
}

/* ---------------------------------------------------------------------- */
/* Momentum SGD and the training-stability modes.                           */

void hxo_momentum(size_t n, const float* w, const float* g, const float* v, float lr, float momentum,
                  float* w_next, float* v_next)
{
    /* tiny_language_model_cpu.cpp:123: nv = momentum*v + g; nw = w - lr*nv */
    for (size_t i = 0; i < n; ++i) {
        const float nv = momentum * v[i] + g[i];
        v_next[i] = nv;
        w_next[i] = w[i] - lr * nv;
    }
}

float hxo_stability_learning_rate(uint32_t mode, float base, uint32_t step, uint32_t total_steps)
{
    if (mode == 1) {                               /* WARMUP64 */
        const double f = (double)step / 64.0;
        return (float)(base * (f < 1.0 ? f : 1.0));
    }
    if (mode == 2) {                               /* DECAY_LINEAR */
        const double done = total_steps ? (double)total_steps : 1.0;
        return (float)(base * (1.0 - (double)(step - 1) / done));
    }
    return base;
}

/* Offsets of layer l's tensors in the flat layout. */
static void layer_offsets(const hxo_lm_config* c, uint32_t l, size_t o[10])
{
    const size_t V = c->vocab, T = c->tokens, D = c->dim, F = c->ffn;
    size_t off = V * D + (c->learned_position ? T * D : 0) + (size_t)l * (4 * D * D + 4 * D + 2 * D * F);
    const size_t sz[10] = {D, D, D * D, D * D, D * D, D * D, D, D, D * F, F * D};
    for (int k = 0; k < 10; ++k) {  /* g1 b1 wq wk wv wo g2 b2 w1 w2 */
        o[k] = off;
        off += sz[k];
    }
}

void hxo_apply_init_stability(const hxo_lm_config* c, uint32_t mode, float* p)
{
    const size_t D = c->dim, F = c->ffn;
    const float s = 1.0f / sqrtf(2.0f * (float)c->layers);
    for (uint32_t l = 0; l < c->layers; ++l) {
        size_t o[10];
        layer_offsets(c, l, o);
        if (mode == 3) {         /* ZERO_OUTPUT_PROJ_BRANCH_INIT */
            memset(p + o[5], 0, sizeof(float) * D * D);
            memset(p + o[9], 0, sizeof(float) * F * D);
        } else if (mode == 4) {  /* DEPTH_SCALED_BRANCH_INIT */
            for (size_t i = 0; i < D * D; ++i) p[o[5] + i] *= s;
            for (size_t i = 0; i < D * F; ++i) p[o[8] + i] *= s;
            for (size_t i = 0; i < F * D; ++i) p[o[9] + i] *= s;
        }
    }
}

static double tensor_norm(const float* x, size_t n)
{
    double s = 0;
    for (size_t i = 0; i < n; ++i) s += (double)x[i] * x[i];
    return sqrt(s);
}

double hxo_gradient_norm(const hxo_lm_config* c, const float* g, float threshold, float* clip)
{
    const size_t V = c->vocab, T = c->tokens, D = c->dim, F = c->ffn;
    double sum = 0, nrm;
    nrm = tensor_norm(g, V * D);
    sum += nrm * nrm;
    if (c->learned_position) {
        nrm = tensor_norm(g + V * D, T * D);
        sum += nrm * nrm;
    }
    const int order[10] = {2, 3, 4, 5, 0, 1, 6, 7, 8, 9};  /* wq wk wv wo g1 b1 g2 b2 w1 w2 */
    const size_t sz[10] = {D, D, D * D, D * D, D * D, D * D, D, D, D * F, F * D};
    for (uint32_t l = 0; l < c->layers; ++l) {
        size_t o[10];
        layer_offsets(c, l, o);
        for (int k = 0; k < 10; ++k) {
            nrm = tensor_norm(g + o[order[k]], sz[order[k]]);
            sum += nrm * nrm;
        }
    }
    size_t oo[10];
    layer_offsets(c, c->layers, oo);  /* the output projection follows the last layer */
    nrm = tensor_norm(g + oo[0], D * V);
    sum += nrm * nrm;
    const double norm = sqrt(sum);
    if (clip) {
        const double q = (double)threshold / (norm + 1.0e-6);
        *clip = (threshold > 0 && isfinite(norm) && norm > 0) ? (float)(q < 1.0 ? q : 1.0) : 1.0f;
    }
    return norm;
}
