// Test infrastructure only: a C-ABI wrapper around the reference CPU kernels.
//
// This file is compiled together with the reference's own src/kernels.cpp and
// src/gguf.cpp (see oracle/Makefile) into oracle/_ref/libnedo_ref*.so.  It lets
// the parity tests and the CPU-baseline leg of bench.py call the unmodified
// reference implementation of nedo::kernels::matvec / embedding_row on exactly
// the same bytes that the CUDA path reads.  Nothing in the product links it.
//
// Reference interfaces wrapped:
//   nedo::kernels::matvec         include/nedo/kernels.hpp:20, src/kernels.cpp:162-169
//   nedo::kernels::embedding_row  include/nedo/kernels.hpp:21, src/kernels.cpp:170-176
//   nedo::kernels::fp16_to_fp32   include/nedo/kernels.hpp:9,  src/kernels.cpp:24-33
//   nedo::kernels::fp32_to_fp16   include/nedo/kernels.hpp:10, src/kernels.cpp:34-42
//   nedo::tensor_nbytes           include/nedo/gguf.hpp:88,    src/gguf.cpp:106-114
#include "nedo/kernels.hpp"
#include "nedo/gguf.hpp"

#include <cstdint>
#include <cstring>
#include <exception>
#include <span>
#include <string>
#ifdef _OPENMP
#include <omp.h>
#endif

namespace {
thread_local std::string g_last_error;

nedo::TensorInfo make_info(uint32_t type, uint64_t rows, uint64_t cols) {
    nedo::TensorInfo t;
    t.name = "w";
    t.shape = {cols, rows};  // GGUF order: shape[0] is the contiguous dimension
    t.type = static_cast<nedo::TensorType>(type);
    t.n_elements = rows * cols;
    return t;
}
}  // namespace

extern "C" {

const char* nedo_ref_last_error(void) { return g_last_error.c_str(); }

int nedo_ref_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void nedo_ref_set_num_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

int nedo_ref_has_openmp(void) {
#ifdef _OPENMP
    return 1;
#else
    return 0;
#endif
}

int nedo_ref_tensor_nbytes(uint32_t type, uint64_t n, uint64_t* out) {
    try {
        *out = nedo::tensor_nbytes(static_cast<nedo::TensorType>(type), n);
        return 0;
    } catch (const std::exception& e) {
        g_last_error = e.what();
        return 1;
    }
}

// y[r] = dot(row r of w, x) for r < rows. Only F16 / Q4_0 / Q8_0 may be passed
// with rows >= 256: the reference throws inside its OpenMP region for any other
// type, which terminates the process (src/kernels.cpp:166-168).
int nedo_ref_matvec(uint32_t type, uint64_t rows, uint64_t cols, const void* w, uint64_t w_bytes,
                    const float* x, float* y) {
    try {
        auto t = make_info(type, rows, cols);
        nedo::kernels::matvec(t, std::span<const std::byte>(static_cast<const std::byte*>(w), w_bytes), x, y);
        return 0;
    } catch (const std::exception& e) {
        g_last_error = e.what();
        return 1;
    }
}

int nedo_ref_embedding_row(uint32_t type, uint64_t rows, uint64_t cols, const void* w, uint64_t w_bytes,
                           uint32_t row, float* out) {
    try {
        auto t = make_info(type, rows, cols);
        nedo::kernels::embedding_row(t, std::span<const std::byte>(static_cast<const std::byte*>(w), w_bytes), row,
                                     out);
        return 0;
    } catch (const std::exception& e) {
        g_last_error = e.what();
        return 1;
    }
}

float nedo_ref_fp16_to_fp32(uint16_t h) { return nedo::kernels::fp16_to_fp32(h); }
uint16_t nedo_ref_fp32_to_fp16(float f) { return nedo::kernels::fp32_to_fp16(f); }

}  // extern "C"
