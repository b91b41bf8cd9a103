// sampling.cu -- next-token selection for generation, on the host.
//
// The reference samples on the CPU from the device's last-row logits
// (nicopedia_generation.h:286-395): greedyArgmax takes the first maximum;
// sampleTopKChecked orders the vocabulary by (logit descending, index
// ascending), keeps the top K (0 = all), forms the temperature softmax of
// those logits in double, and walks the cumulative probabilities to the
// first one at or above u = top53(splitmix64(seed + step * golden)) / 2^53,
// falling back to the last kept index when rounding leaves u above the sum.
// A temperature that is not positive and finite means greedy.  The audit
// flags report non-finite logits or weights and non-positive sums; any of
// them fails the step (qnn_prepared_generation.cpp:406-422).
#include <algorithm>
#include <cmath>
#include <numeric>
#include <vector>

#include "hx_internal.cuh"

namespace {

uint64_t mix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

uint32_t first_max(const float* logits, uint32_t vocab) {
    uint32_t best = 0;
    for (uint32_t i = 1; i < vocab; ++i)
        if (logits[i] > logits[best]) best = i;
    return best;
}

}  // namespace

extern "C" {

int hx_sample_next_token(const float* logits, uint32_t vocab, const hx_sampling* s, uint64_t step,
                         uint32_t* token, hx_sampling_audit* audit) {
    if (!logits || !s || !token || vocab == 0 || vocab > 65536) return HX_ERR_ARGUMENT;
    hx_sampling_audit a{};
    a.ok = 1;
    for (uint32_t i = 0; i < vocab; ++i)
        if (!std::isfinite(logits[i])) a.ok = 0;
    a.logits_finite = a.ok;
    if (!a.ok) {
        if (audit) *audit = a;
        return HX_ERR_NONFINITE;
    }
    if (s->greedy || !(s->temperature > 0.0f) || !std::isfinite(s->temperature)) {
        *token = first_max(logits, vocab);
        if (audit) *audit = a;
        return HX_OK;
    }
    const uint32_t k = (s->top_k == 0 || s->top_k >= vocab) ? vocab : s->top_k;
    std::vector<uint32_t> idx(vocab);
    std::iota(idx.begin(), idx.end(), 0u);
    std::sort(idx.begin(), idx.end(), [&](uint32_t x, uint32_t y) {
        return logits[x] != logits[y] ? logits[x] > logits[y] : x < y;
    });
    const double top = double(logits[idx[0]]);
    std::vector<double> w(k);
    double sum = 0.0;
    bool weights_finite = true;
    for (uint32_t i = 0; i < k; ++i) {
        w[i] = std::exp((double(logits[idx[i]]) - top) / double(s->temperature));
        sum += w[i];
        if (!std::isfinite(w[i])) weights_finite = false;
    }
    a.weight_sum = sum;
    if (!weights_finite || !std::isfinite(sum) || !(sum > 0.0)) {
        a.ok = 0;
        if (audit) *audit = a;
        return HX_ERR_NONFINITE;
    }
    const double u = double(mix64(s->seed + step * 0x9E3779B97F4A7C15ull) >> 11) * 0x1.0p-53;
    double cumulative = 0.0, psum = 0.0;
    bool selected = false, pfinite = true;
    for (uint32_t i = 0; i < k; ++i) {
        const double pr = w[i] / sum;
        if (!std::isfinite(pr)) pfinite = false;
        psum += pr;
        if (!selected && u <= cumulative + pr) {
            *token = idx[i];
            selected = true;
        }
        cumulative += pr;
    }
    a.probability_sum = psum;
    if (!pfinite || !std::isfinite(cumulative) || !std::isfinite(psum) || !(psum > 0.0)) {
        a.ok = 0;
        if (audit) *audit = a;
        return HX_ERR_NONFINITE;
    }
    if (!selected) *token = idx[k - 1];
    if (audit) *audit = a;
    return HX_OK;
}

}  // extern "C"
