// nedo_kernels_cuda.cpp -- drop-in replacement of the two hot-path entry points
// of nedo.cpp's CPU kernels, forwarding to the B200 library (include/nedo_gpu.h):
//
//   void nedo::kernels::matvec(const TensorInfo&, std::span<const std::byte>,
//                              const float* x, float* y);              kernels.hpp:20
//   void nedo::kernels::embedding_row(const TensorInfo&, std::span<const std::byte>,
//                                     uint32_t row, float* out);       kernels.hpp:21
//
// Compiled inside the reference tree (against its include/nedo/*.hpp) it
// replaces the definitions in src/kernels.cpp:162-176; compiled here it uses
// the declaration-compatible headers in cpp/compat.  Behaviour kept from the
// reference:
//   * rank-2 check first: "matvec requires rank-2 tensor: <name>" (src/kernels.cpp:163)
//   * row size via tensor_nbytes, so its exceptions ("Q4_0 elements not block
//     aligned", "tensor type not implemented: N") surface unchanged (src/gguf.cpp:106-114)
//   * an unsupported type throws "matvec tensor type not supported"
//     (src/kernels.cpp:168) -- here always as an exception before any launch,
//     where the reference would terminate inside its OpenMP region for rows >= 256
//   * embedding_row: "bad embedding row" / "embedding type unsupported" (src/kernels.cpp:171,175)
//   * synchronous: y[0..rows) is fully written when the call returns.
// Added: a span shorter than rows*row_bytes throws instead of reading past it.
//
// Added entry point (no reference counterpart, declared in cpp/compat/nedo/kernels.hpp;
// a maintainer adds the same line to the reference's include/nedo/kernels.hpp):
//   void nedo::kernels::matvec_batch(const TensorInfo&, std::span<const std::byte>,
//                                    const float* x, float* y, uint32_t batch);
// `batch` matvecs over one weight, x [batch][cols] -> y [batch][rows], with the
// same checks and messages as matvec.  It replaces the prompt loop of
// src/model.cpp:262-266 (one forward per token, each weight read per token)
// with one pass over each weight for the whole prompt.
//
//   uint32_t nedo::kernels::sample_lm_head(const TensorInfo&, std::span<const std::byte>,
//                                          const float* x, float temperature, uint32_t top_k,
//                                          float top_p, std::mt19937_64& rng);
// The LM head matvec (src/model.cpp:259) followed by the reference's sampler
// (sample_token, src/model.cpp:33-63) with the caller's generator: greedy
// (temperature <= 0) is the fused device argmax; for top_k in [1, 256] the k
// candidates are selected on the device and only they are copied back; other
// top_k (0 = all) read every logit back and select on the host as the
// reference does.  From the candidates on, the steps are the reference's:
// tempered softmax in double, the top_p cut, std::discrete_distribution.
#include <algorithm>
#include <cmath>
#include <cstddef>
#include <cstdint>
#include <limits>
#include <numeric>
#include <random>
#include <span>
#include <stdexcept>
#include <string>
#include <vector>

#include "nedo/kernels.hpp"
#include "nedo_gpu.h"

namespace nedo::kernels {

namespace {
[[noreturn]] void raise_gpu(int) { throw std::runtime_error(nedo_gpu_last_error()); }

bool gpu_type(TensorType t) { return t == TensorType::F16 || t == TensorType::Q4_0 || t == TensorType::Q8_0; }
}  // namespace

void matvec(const TensorInfo& t, std::span<const std::byte> b, const float* x, float* y) {
    if (t.shape.size() != 2) throw std::runtime_error("matvec requires rank-2 tensor: " + t.name);
    const uint64_t cols = t.shape[0], rows = t.shape[1];
    const uint64_t rowbytes = tensor_nbytes(t.type, cols);
    if (rows == 0) return;
    if (!gpu_type(t.type)) throw std::runtime_error("matvec tensor type not supported");
    if (b.size() < rows * rowbytes) throw std::runtime_error("matvec: tensor bytes shorter than its shape: " + t.name);
    const int rc = nedo_gpu_matvec(static_cast<uint32_t>(t.type), rows, cols, b.data(), b.size(), x, y);
    if (rc != NEDO_GPU_OK) raise_gpu(rc);
}

void matvec_batch(const TensorInfo& t, std::span<const std::byte> b, const float* x, float* y, uint32_t batch) {
    if (t.shape.size() != 2) throw std::runtime_error("matvec requires rank-2 tensor: " + t.name);
    const uint64_t cols = t.shape[0], rows = t.shape[1];
    const uint64_t rowbytes = tensor_nbytes(t.type, cols);
    if (rows == 0 || batch == 0) return;
    if (!gpu_type(t.type)) throw std::runtime_error("matvec tensor type not supported");
    if (b.size() < rows * rowbytes) throw std::runtime_error("matvec: tensor bytes shorter than its shape: " + t.name);
    const int rc = nedo_gpu_matvec_batch(static_cast<uint32_t>(t.type), rows, cols, b.data(), b.size(), x, y, batch);
    if (rc != NEDO_GPU_OK) raise_gpu(rc);
}

uint32_t sample_lm_head(const TensorInfo& t, std::span<const std::byte> b, const float* x, float temperature,
                        uint32_t top_k, float top_p, std::mt19937_64& rng) {
    if (t.shape.size() != 2) throw std::runtime_error("matvec requires rank-2 tensor: " + t.name);
    const uint64_t cols = t.shape[0], vocab = t.shape[1];
    const uint64_t rowbytes = tensor_nbytes(t.type, cols);
    if (vocab == 0) throw std::runtime_error("empty logits");
    if (!gpu_type(t.type)) throw std::runtime_error("matvec tensor type not supported");
    if (b.size() < vocab * rowbytes) throw std::runtime_error("matvec: tensor bytes shorter than its shape: " + t.name);
    const auto type = static_cast<uint32_t>(t.type);
    if (temperature <= 0.f) {
        int64_t idx = -1;
        const int rc = nedo_gpu_lm_head_argmax(type, vocab, cols, b.data(), b.size(), x, &idx, nullptr);
        if (rc != NEDO_GPU_OK) raise_gpu(rc);
        return static_cast<uint32_t>(idx);
    }
    const uint64_t k = top_k ? std::min<uint64_t>(top_k, vocab) : vocab;
    std::vector<uint32_t> ids;
    std::vector<float> logit;  // logit[i] is the logit of ids[i]
    if (k <= 256) {
        ids.resize(k);
        logit.resize(k);
        const int rc = nedo_gpu_lm_head_topk(type, vocab, cols, b.data(), b.size(), x, static_cast<uint32_t>(k),
                                             ids.data(), logit.data());
        if (rc != NEDO_GPU_OK) raise_gpu(rc);
    } else {
        std::vector<float> all(vocab);
        const int rc = nedo_gpu_matvec(type, vocab, cols, b.data(), b.size(), x, all.data());
        if (rc != NEDO_GPU_OK) raise_gpu(rc);
        ids.resize(vocab);
        std::iota(ids.begin(), ids.end(), 0u);
        auto larger = [&](uint32_t l, uint32_t r) { return all[l] > all[r]; };
        if (k < ids.size()) {
            std::nth_element(ids.begin(), ids.begin() + static_cast<std::ptrdiff_t>(k), ids.end(), larger);
            ids.resize(k);
        }
        std::sort(ids.begin(), ids.end(), larger);
        logit.resize(ids.size());
        for (size_t i = 0; i < ids.size(); ++i) logit[i] = all[ids[i]];
    }
    // tempered softmax over the candidates, largest first (float products, double exp)
    const float inv_t = 1.f / temperature;
    float top = -std::numeric_limits<float>::infinity();
    for (float l : logit) top = std::max(top, l * inv_t);
    std::vector<double> prob(logit.size());
    double total = 0.0;
    for (size_t i = 0; i < logit.size(); ++i) {
        prob[i] = std::exp(static_cast<double>(logit[i] * inv_t - top));
        total += prob[i];
    }
    for (double& p : prob) p /= total;
    if (top_p > 0.f && top_p < 1.f) {
        // smallest prefix whose mass reaches top_p (at least one candidate)
        double mass = 0.0;
        size_t keep = 0;
        while (keep < prob.size()) {
            mass += prob[keep++];
            if (mass >= top_p) break;
        }
        keep = std::max<size_t>(1, std::min(keep, prob.size()));
        ids.resize(keep);
        prob.resize(keep);
        total = std::accumulate(prob.begin(), prob.end(), 0.0);
        for (double& p : prob) p /= total;
    }
    std::discrete_distribution<size_t> pick(prob.begin(), prob.end());
    return ids[pick(rng)];
}

void embedding_row(const TensorInfo& t, std::span<const std::byte> b, uint32_t row, float* out) {
    if (t.shape.size() != 2 || row >= t.shape[1]) throw std::runtime_error("bad embedding row");
    const uint64_t cols = t.shape[0], rows = t.shape[1];
    const uint64_t rowbytes = tensor_nbytes(t.type, cols);
    if (!gpu_type(t.type)) throw std::runtime_error("embedding type unsupported");
    if (b.size() < rows * rowbytes) throw std::runtime_error("embedding_row: tensor bytes shorter than its shape");
    const int rc = nedo_gpu_embedding_row(static_cast<uint32_t>(t.type), rows, cols, b.data(), b.size(), row, out);
    if (rc != NEDO_GPU_OK) raise_gpu(rc);
}

}  // namespace nedo::kernels
