// init.cu -- host-side deterministic parameter initialisers for the LM.
#include <cmath>
#include <cstdio>

#include "hx_internal.cuh"

namespace {

struct Layout {
    size_t E, pos, out;
    std::vector<size_t> g1, b1, wq, wk, wv, wo, g2, b2, w1, w2;
};

Layout layout(const hx_lm_config* c) {
    const size_t V = c->vocab, T = c->tokens, D = c->dim, F = c->ffn;
    Layout l;
    size_t off = 0;
    l.E = off; off += V * D;
    l.pos = SIZE_MAX;
    if (c->flags & HX_LM_LEARNED_POSITION) { l.pos = off; off += T * D; }
    for (uint32_t i = 0; i < c->layers; ++i) {
        l.g1.push_back(off); off += D;
        l.b1.push_back(off); off += D;
        l.wq.push_back(off); off += D * D;
        l.wk.push_back(off); off += D * D;
        l.wv.push_back(off); off += D * D;
        l.wo.push_back(off); off += D * D;
        l.g2.push_back(off); off += D;
        l.b2.push_back(off); off += D;
        l.w1.push_back(off); off += D * F;
        l.w2.push_back(off); off += F * D;
    }
    l.out = off;
    return l;
}

void fixed_position(const hx_lm_config* c, float* out) {
    for (uint32_t t = 0; t < c->tokens; ++t)
        for (uint32_t d = 0; d < c->dim; ++d) {
            const float f = std::pow(10000.f, -float(d & ~1u) / float(c->dim));
            out[size_t(t) * c->dim + d] = ((d & 1u) ? std::cos(float(t) * f) : std::sin(float(t) * f)) * .05f;
        }
}

uint64_t splitmix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

int validate_or(const hx_lm_config* c, float* p) {
    if (!c || !p || !c->vocab || !c->tokens || !c->dim || !c->ffn || !c->layers || !c->heads || c->dim % c->heads)
        return HX_ERR_ARGUMENT;
    return HX_OK;
}

}  // namespace

extern "C" {

// tiny_lm::initialParameters (tiny_language_model_cpu.cpp:69-70): a 32-bit
// LCG per tensor, seeded from (seed, phase), mapped to a uniform value in
// [-scale, scale] through a 16-bit field.  The learned position table (no
// reference counterpart) starts as the fixed sinusoid, so the two position
// modes agree at initialisation.
int hx_lm_init_reference(const hx_lm_config* c, uint32_t seed, float* p) {
    if (int rc = validate_or(c, p)) return rc;
    const size_t D = c->dim, F = c->ffn, V = c->vocab;
    const Layout l = layout(c);
    auto fill = [&](size_t off, size_t n, uint32_t phase, float scale) {
        uint32_t s = seed * 747796405u + phase * 2891336453u;
        for (size_t i = 0; i < n; ++i) {
            s = s * 1664525u + 1013904223u;
            p[off + i] = (float(int((s >> 8) & 65535u)) / 32767.5f - 1) * scale;
        }
    };
    for (uint32_t i = 0; i < c->layers; ++i) {
        for (size_t d = 0; d < D; ++d) {
            p[l.g1[i] + d] = 1.f; p[l.b1[i] + d] = 0.f;
            p[l.g2[i] + d] = 1.f; p[l.b2[i] + d] = 0.f;
        }
    }
    fill(l.E, V * D, 1, .18f);
    fill(l.wq[0], D * D, 2, .12f);
    fill(l.wk[0], D * D, 3, .12f);
    fill(l.wv[0], D * D, 4, .12f);
    fill(l.wo[0], D * D, 5, .12f);
    fill(l.w1[0], D * F, 6, .1f);
    fill(l.w2[0], F * D, 7, .1f);
    fill(l.out, D * V, 8, .16f);
    for (uint32_t i = 1; i < c->layers; ++i) {
        const uint32_t base = 8 + i * 10;
        fill(l.wq[i], D * D, base + 1, .12f);
        fill(l.wk[i], D * D, base + 2, .12f);
        fill(l.wv[i], D * D, base + 3, .12f);
        fill(l.wo[i], D * D, base + 4, .12f);
        fill(l.w1[i], D * F, base + 5, .1f);
        fill(l.w2[i], F * D, base + 6, .1f);
    }
    if (l.pos != SIZE_MAX) fixed_position(c, p + l.pos);
    return HX_OK;
}

// N(0, std) for every matrix and table, gamma = 1, beta = 0.  Element k of
// the flat buffer draws two splitmix64 words from (seed, k) and applies the
// Box-Muller transform, so values do not depend on fill order.
int hx_lm_init_normal(const hx_lm_config* c, uint64_t seed, float std_dev, float* p) {
    if (int rc = validate_or(c, p)) return rc;
    if (!(std_dev >= 0.f) || !std::isfinite(std_dev)) return HX_ERR_ARGUMENT;
    const size_t D = c->dim;
    const Layout l = layout(c);
    const size_t P = l.out + size_t(c->dim) * c->vocab;
    const double two_pi = 6.283185307179586476925286766559;
    const uint64_t key = splitmix64(seed);
    for (size_t k = 0; k < P; ++k) {
        const uint64_t a = splitmix64(key ^ (2 * k)), b = splitmix64(key ^ (2 * k + 1));
        const double u1 = (double((a >> 11) + 1)) * 0x1.0p-53;  // (0, 1]
        const double u2 = double(b >> 11) * 0x1.0p-53;          // [0, 1)
        p[k] = float(std::sqrt(-2.0 * std::log(u1)) * std::cos(two_pi * u2) * std_dev);
    }
    for (uint32_t i = 0; i < c->layers; ++i)
        for (size_t d = 0; d < D; ++d) {
            p[l.g1[i] + d] = 1.f; p[l.b1[i] + d] = 0.f;
            p[l.g2[i] + d] = 1.f; p[l.b2[i] + d] = 0.f;
        }
    return HX_OK;
}

}  // extern "C"
