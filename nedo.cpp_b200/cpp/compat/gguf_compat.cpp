// Standalone implementations of the helpers the drop-in layer needs when it is
// built outside the nedo.cpp tree (inside the tree, src/gguf.cpp and
// src/kernels.cpp provide them).
#include <cstring>
#include <stdexcept>
#include <string>

#include "nedo/gguf.hpp"
#include "nedo/kernels.hpp"

namespace nedo {

uint64_t tensor_nbytes(TensorType type, uint64_t n) {
    switch (type) {
        case TensorType::F32: return n * 4;
        case TensorType::F16:
        case TensorType::BF16: return n * 2;
        case TensorType::Q4_0:
            if (n % 32) throw std::runtime_error("Q4_0 elements not block aligned");
            return n / 32 * 18;
        case TensorType::Q8_0:
            if (n % 32) throw std::runtime_error("Q8_0 elements not block aligned");
            return n / 32 * 34;
        case TensorType::I8: return n;
        case TensorType::I16: return n * 2;
        case TensorType::I32: return n * 4;
        case TensorType::I64: return n * 8;
        default: throw std::runtime_error("tensor type not implemented: " + std::to_string(static_cast<uint32_t>(type)));
    }
}

namespace kernels {

float fp16_to_fp32(uint16_t h) noexcept {
    const uint32_t sign = static_cast<uint32_t>(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1Fu, man = h & 0x3FFu, bits;
    if (exp == 0x1Fu) {
        bits = sign | 0x7F800000u | (man << 13);
    } else if (exp != 0) {
        bits = sign | ((exp + 112u) << 23) | (man << 13);
    } else if (man == 0) {
        bits = sign;
    } else {
        int e = -1;
        do {
            man <<= 1;
            ++e;
        } while ((man & 0x400u) == 0);
        bits = sign | (static_cast<uint32_t>(112 - e) << 23) | ((man & 0x3FFu) << 13);
    }
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

uint16_t fp32_to_fp16(float f) noexcept {
    // round to nearest, ties to even
    uint32_t x;
    std::memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u, ax = x & 0x7FFFFFFFu;
    if (ax >= 0x7F800000u) return static_cast<uint16_t>(sign | 0x7C00u | (ax > 0x7F800000u ? 0x200u : 0u));
    if (ax >= 0x477FF000u) return static_cast<uint16_t>(sign | 0x7C00u);
    if (ax < 0x38800000u) {
        if (ax < 0x33000000u) return static_cast<uint16_t>(sign);
        const uint32_t e = ax >> 23, m = (ax & 0x7FFFFFu) | 0x800000u, shift = 126u - e;
        uint32_t q = m >> shift;
        const uint32_t rem = m & ((1u << shift) - 1u), half = 1u << (shift - 1u);
        if (rem > half || (rem == half && (q & 1u))) ++q;
        return static_cast<uint16_t>(sign | q);
    }
    uint32_t q = (((ax >> 23) - 112u) << 10) | ((ax & 0x7FFFFFu) >> 13);
    const uint32_t rem = ax & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) ++q;
    return static_cast<uint16_t>(sign | q);
}

}  // namespace kernels
}  // namespace nedo
