// Declaration-compatible subset of nedo.cpp's include/nedo/kernels.hpp: the two
// hot-path entry points (kernels.hpp:20-21), the fp16 helpers the kernel
// tests use (kernels.hpp:9-10), and the drop-in's added batched matvec and
// LM-head sampler.
#pragma once
#include <cstddef>
#include <cstdint>
#include <random>
#include <span>

#include "nedo/gguf.hpp"

namespace nedo::kernels {
float fp16_to_fp32(uint16_t h) noexcept;
uint16_t fp32_to_fp16(float f) noexcept;
void matvec(const TensorInfo& t, std::span<const std::byte> bytes, const float* x, float* y);
void embedding_row(const TensorInfo& t, std::span<const std::byte> bytes, uint32_t row, float* out);
// Added by the B200 drop-in (no reference counterpart): `batch` matvecs over one
// weight, x [batch][cols] -> y [batch][rows].
void matvec_batch(const TensorInfo& t, std::span<const std::byte> bytes, const float* x, float* y, uint32_t batch);
// Added by the B200 drop-in (no reference counterpart as a kernel): the LM head
// matvec followed by the reference's sampler (src/model.cpp:33-63) with `rng`.
uint32_t sample_lm_head(const TensorInfo& t, std::span<const std::byte> bytes, const float* x, float temperature,
                        uint32_t top_k, float top_p, std::mt19937_64& rng);
}  // namespace nedo::kernels
