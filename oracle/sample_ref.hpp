// TEST INFRASTRUCTURE ONLY: the reference's token sampler restated for the
// sampling parity test (tests/sample_parity.cpp).  Never linked into the
// product.
//
// Follows sample_token of the reference (src/model.cpp:33-63) step for step,
// with the same standard-library algorithms, so that with the same logits and
// the same std::mt19937_64 state it draws the same token:
//   temperature <= 0: std::max_element (first index of the maximum);
//   else the top_k candidates (0 = all) by std::nth_element + std::sort on
//   logit (descending), the softmax of logit * (1 / temperature) in double, the
//   smallest prefix reaching top_p (when 0 < top_p < 1) renormalised, and one
//   std::discrete_distribution draw.
#pragma once
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <limits>
#include <numeric>
#include <random>
#include <stdexcept>
#include <vector>

namespace oracle_ref {

inline uint32_t sample_token(const std::vector<float>& logits, float temperature, uint32_t top_k, float top_p,
                             std::mt19937_64& rng) {
    if (logits.empty()) throw std::runtime_error("empty logits");
    if (temperature <= 0.f)
        return static_cast<uint32_t>(std::max_element(logits.begin(), logits.end()) - logits.begin());
    std::vector<uint32_t> cand(logits.size());
    std::iota(cand.begin(), cand.end(), 0u);
    const size_t k = top_k ? std::min<size_t>(top_k, cand.size()) : cand.size();
    auto by_logit = [&](uint32_t l, uint32_t r) { return logits[l] > logits[r]; };
    if (k < cand.size()) {
        std::nth_element(cand.begin(), cand.begin() + static_cast<std::ptrdiff_t>(k), cand.end(), by_logit);
        cand.resize(k);
    }
    std::sort(cand.begin(), cand.end(), by_logit);
    const float inv_t = 1.f / temperature;
    float mx = -std::numeric_limits<float>::infinity();
    for (uint32_t id : cand) mx = std::max(mx, logits[id] * inv_t);
    std::vector<double> p(cand.size());
    double sum = 0.0;
    for (size_t i = 0; i < cand.size(); ++i) {
        p[i] = std::exp(double(logits[cand[i]] * inv_t - mx));
        sum += p[i];
    }
    for (double& v : p) v /= sum;
    if (top_p > 0.f && top_p < 1.f) {
        double cum = 0.0;
        size_t keep = 0;
        for (; keep < p.size(); ++keep) {
            cum += p[keep];
            if (cum >= top_p) {
                ++keep;
                break;
            }
        }
        keep = std::max<size_t>(1, std::min(keep, p.size()));
        cand.resize(keep);
        p.resize(keep);
        sum = std::accumulate(p.begin(), p.end(), 0.0);
        for (double& v : p) v /= sum;
    }
    std::discrete_distribution<size_t> dist(p.begin(), p.end());
    return cand[dist(rng)];
}

}  // namespace oracle_ref
