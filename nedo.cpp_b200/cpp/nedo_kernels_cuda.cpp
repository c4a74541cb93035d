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
#include <cstddef>
#include <cstdint>
#include <span>
#include <stdexcept>
#include <string>

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
