// gemv_generic.cu -- shape-agnostic kernels of the matvec path:
//   * gemv_generic_kernel: any row size / alignment the streaming kernel does
//     not take (e.g. a single 34-byte Q8_0 row).  One warp per row, lanes over
//     blocks, byte-granular loads.  Same block semantics as the reference's
//     dot_f16 / dot_q8 / dot_q4 (src/kernels.cpp:109-160).
//   * dequant_rows_kernel: embedding_row (src/kernels.cpp:170-176): one fp32
//     multiply d*q per element, so the result is bit-identical to the reference.
//   * argmax kernels: first index of the maximum (std::max_element,
//     src/model.cpp:36), with its NaN behaviour: NaNs never win, except that
//     a NaN at index 0 is returned (max_element starts from element 0 and no
//     comparison with NaN succeeds).
#include <math.h>

#include "common.cuh"
#include "launch.h"

namespace nedo_gpu {
namespace {

__device__ __forceinline__ float load_half(const uint8_t* p) {
    const uint32_t lo = p[0], hi = p[1];
    return half_bits_to_float(lo | (hi << 8));
}

template <uint32_t TYPE>
__global__ void gemv_generic_kernel(const uint8_t* __restrict__ w, const float* __restrict__ x, float* __restrict__ y,
                                    uint64_t rows, uint64_t cols, uint64_t rb, uint32_t batch, uint64_t ldx,
                                    uint64_t ldy) {
    const uint32_t lane = threadIdx.x & 31u;
    const uint64_t row = static_cast<uint64_t>(blockIdx.x) * (blockDim.x / 32u) + threadIdx.x / 32u;
    if (row >= rows) return;
    const uint8_t* p = w + row * rb;
    for (uint32_t b = 0; b < batch; ++b) {
        const float* xb = x + b * ldx;
        float acc = 0.f;
        if constexpr (TYPE == kF16) {
            for (uint64_t i = lane; i < cols; i += 32u) acc = fmaf(load_half(p + 2u * i), xb[i], acc);
        } else {
            const uint64_t nb = cols / 32u;
            for (uint64_t blk = lane; blk < nb; blk += 32u) {
                const uint8_t* q = p + blk * (TYPE == kQ8_0 ? 34u : 18u);
                const float d = load_half(q);
                const float* xx = xb + blk * 32u;
                float s = 0.f;
                if constexpr (TYPE == kQ8_0) {
                    for (int i = 0; i < 32; ++i) s = fmaf(static_cast<float>(static_cast<int8_t>(q[2 + i])), xx[i], s);
                } else {
                    for (int i = 0; i < 16; ++i) {
                        const uint32_t v = q[2 + i];
                        s = fmaf(static_cast<float>(static_cast<int>(v & 15u) - 8), xx[i], s);
                        s = fmaf(static_cast<float>(static_cast<int>(v >> 4) - 8), xx[i + 16], s);
                    }
                }
                acc = fmaf(d, s, acc);
            }
        }
        acc = warp_sum(acc);
        if (lane == 0) y[b * ldy + row] = acc;
    }
}

template <uint32_t TYPE>
__global__ void dequant_rows_kernel(const uint8_t* __restrict__ w, uint64_t cols, uint64_t rb, uint64_t row_begin,
                                    uint64_t row_count, float* __restrict__ out) {
    const uint64_t total = row_count * cols;
    for (uint64_t e = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; e < total;
         e += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        const uint64_t r = e / cols, i = e % cols;
        const uint8_t* p = w + (row_begin + r) * rb;
        float v;
        if constexpr (TYPE == kF16) {
            v = load_half(p + 2u * i);
        } else if constexpr (TYPE == kQ8_0) {
            const uint8_t* blk = p + (i / 32u) * 34u;
            v = __fmul_rn(load_half(blk), static_cast<float>(static_cast<int8_t>(blk[2 + (i % 32u)])));
        } else {
            const uint8_t* blk = p + (i / 32u) * 18u;
            const uint32_t k = static_cast<uint32_t>(i % 32u);
            const uint32_t byte = blk[2 + (k & 15u)];
            const int n = (k < 16u) ? static_cast<int>(byte & 15u) - 8 : static_cast<int>(byte >> 4) - 8;
            v = __fmul_rn(load_half(blk), static_cast<float>(n));
        }
        out[e] = v;
    }
}

__device__ __forceinline__ bool better(float v, uint32_t i, float bv, uint32_t bi) {
    return v > bv || (v == bv && i < bi);
}

// One pass: each CTA folds a strided slice, the last CTA to finish folds the
// per-CTA candidates (self-resetting counter).
__global__ void argmax_kernel(const float* __restrict__ v, uint64_t n, ArgmaxScratch s) {
    __shared__ float sv[32];
    __shared__ uint32_t si[32];
    float bv = -INFINITY;
    uint32_t bi = 0xFFFFFFFFu;
    for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        const float x = v[i];
        if (better(x, static_cast<uint32_t>(i), bv, bi)) {
            bv = x;
            bi = static_cast<uint32_t>(i);
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xFFFFFFFFu, bv, o);
        const uint32_t oi = __shfl_xor_sync(0xFFFFFFFFu, bi, o);
        if (better(ov, oi, bv, bi)) {
            bv = ov;
            bi = oi;
        }
    }
    const uint32_t warp = threadIdx.x / 32u, lane = threadIdx.x & 31u;
    if (lane == 0) {
        sv[warp] = bv;
        si[warp] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (uint32_t k = 1; k < blockDim.x / 32u; ++k)
            if (better(sv[k], si[k], bv, bi)) {
                bv = sv[k];
                bi = si[k];
            }
        s.cand_val[blockIdx.x] = bv;
        s.cand_idx[blockIdx.x] = bi;
        __threadfence();
        const uint32_t done = atomicAdd(s.counter, 1u);
        if (done == gridDim.x - 1u) {
            __threadfence();
            const volatile float* cv = s.cand_val;
            const volatile uint32_t* ci = s.cand_idx;
            float fv = cv[0];
            uint32_t fi = ci[0];
            for (uint32_t k = 1; k < gridDim.x; ++k)
                if (better(cv[k], ci[k], fv, fi)) {
                    fv = cv[k];
                    fi = ci[k];
                }
            // std::max_element keeps element 0 when it is NaN (nothing compares
            // greater than NaN); otherwise NaNs never win, as in better().
            const float v0 = v[0];
            if (v0 != v0) {
                fv = v0;
                fi = 0u;
            }
            *s.out_index = static_cast<int64_t>(fi);
            if (s.out_value != nullptr) *s.out_value = fv;
            *s.counter = 0u;
        }
    }
}

}  // namespace

cudaError_t launch_generic(uint32_t type, const void* w, const float* x, float* y, uint64_t rows, uint64_t cols,
                           uint32_t batch, uint64_t ldx, uint64_t ldy, cudaStream_t stream) {
    const uint64_t rb = row_bytes_of(type, cols);
    if (rb == 0) return cudaErrorInvalidValue;
    const uint32_t warps = 8;
    const uint64_t blocks = (rows + warps - 1) / warps;
    if (blocks > 0x7FFFFFFFull) return cudaErrorInvalidValue;
    const auto* wb = static_cast<const uint8_t*>(w);
    switch (type) {
        case kF16: gemv_generic_kernel<kF16><<<blocks, warps * 32, 0, stream>>>(wb, x, y, rows, cols, rb, batch, ldx, ldy); break;
        case kQ8_0: gemv_generic_kernel<kQ8_0><<<blocks, warps * 32, 0, stream>>>(wb, x, y, rows, cols, rb, batch, ldx, ldy); break;
        case kQ4_0: gemv_generic_kernel<kQ4_0><<<blocks, warps * 32, 0, stream>>>(wb, x, y, rows, cols, rb, batch, ldx, ldy); break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t launch_dequant_rows(uint32_t type, const void* w, uint64_t rows, uint64_t cols, uint64_t row_begin,
                                uint64_t row_count, float* out, cudaStream_t stream) {
    const uint64_t rb = row_bytes_of(type, cols);
    if (rb == 0 || row_begin + row_count > rows) return cudaErrorInvalidValue;
    const uint64_t total = row_count * cols;
    uint64_t blocks = (total + 255) / 256;
    if (blocks > 4096) blocks = 4096;
    if (blocks == 0) return cudaSuccess;
    const auto* wb = static_cast<const uint8_t*>(w);
    switch (type) {
        case kF16: dequant_rows_kernel<kF16><<<blocks, 256, 0, stream>>>(wb, cols, rb, row_begin, row_count, out); break;
        case kQ8_0: dequant_rows_kernel<kQ8_0><<<blocks, 256, 0, stream>>>(wb, cols, rb, row_begin, row_count, out); break;
        case kQ4_0: dequant_rows_kernel<kQ4_0><<<blocks, 256, 0, stream>>>(wb, cols, rb, row_begin, row_count, out); break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t launch_argmax(const float* v, uint64_t n, ArgmaxScratch* scratch, int num_sms, cudaStream_t stream) {
    if (n == 0 || n > 0xFFFFFFFFull) return cudaErrorInvalidValue;
    uint64_t blocks = (n + 1023) / 1024;
    if (blocks > static_cast<uint64_t>(num_sms)) blocks = num_sms;
    argmax_kernel<<<static_cast<uint32_t>(blocks), 1024, 0, stream>>>(v, n, *scratch);
    return cudaGetLastError();
}

}  // namespace nedo_gpu
