// Declaration-compatible subset of nedo.cpp's include/nedo/gguf.hpp, enough to
// build the drop-in matvec layer outside the nedo.cpp tree.  Type codes and the
// TensorInfo members follow include/nedo/gguf.hpp:18-39 because the drop-in must
// be ABI-compatible with them; the file parser itself is out of scope.
#pragma once
#include <cstdint>
#include <string>
#include <vector>

namespace nedo {

enum class TensorType : uint32_t {
    F32 = 0, F16 = 1, Q4_0 = 2, Q4_1 = 3, Q5_0 = 6, Q5_1 = 7, Q8_0 = 8,
    Q8_1 = 9, Q2_K = 10, Q3_K = 11, Q4_K = 12, Q5_K = 13, Q6_K = 14, Q8_K = 15,
    IQ2_XXS = 16, IQ2_XS = 17, IQ3_XXS = 18, IQ1_S = 19, IQ4_NL = 20, IQ3_S = 21,
    IQ2_S = 22, IQ4_XS = 23, I8 = 24, I16 = 25, I32 = 26, I64 = 27, F64 = 28,
    IQ1_M = 29, BF16 = 30
};

struct TensorInfo {
    std::string name;
    std::vector<uint64_t> shape;
    TensorType type{};
    uint64_t relative_offset{};
    uint64_t absolute_offset{};
    uint64_t n_elements{};
    uint64_t n_bytes{};
};

// Bytes of n elements of `type` (same contract as src/gguf.cpp:106-114).
uint64_t tensor_nbytes(TensorType type, uint64_t n_elements);

}  // namespace nedo
