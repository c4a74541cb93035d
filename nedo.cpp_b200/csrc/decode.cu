// decode.cu -- the non-matvec steps of one NedoLM decode forward pass on the
// device (src/model.cpp:212-260 with src/kernels.cpp:43-106 and :170-176):
// embedding row, residual add + RMSNorm, RoPE + KV-cache append, attention over
// the sliding window, SiLU gate (with the MorphFFN masking).  The matvecs of
// the pass are the library's matvec kernels; the host side (nedo_gpu.cu)
// chains everything on one stream and captures it as one CUDA graph.
//
// The token id and the position are read from device memory (`io`), so one
// captured graph serves every step.  Every kernel waits for its predecessor
// with griddepcontrol.wait (programmatic dependent launch) before it reads
// anything that predecessor wrote.
#include <math.h>

#include "common.cuh"
#include "launch.h"

namespace nedo_gpu {
namespace {

__device__ __forceinline__ void dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void dep_launch() { asm volatile("griddepcontrol.launch_dependents;"); }

constexpr uint32_t kF32Type = 0;

// Block-wide sum of one value per thread (blockDim.x a multiple of 32, at most
// 1024), in a fixed order: lanes by xor tree, then warps in index order.
template <typename T>
__device__ T block_sum(T v, T* red) {
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    const uint32_t w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    __syncthreads();
    if ((threadIdx.x & 31u) == 0) red[w] = v;
    __syncthreads();
    T s = red[0];
    for (uint32_t i = 1; i < nw; ++i) s += red[i];
    return s;
}

__device__ float block_max(float v, float* red) {
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
    const uint32_t w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    __syncthreads();
    if ((threadIdx.x & 31u) == 0) red[w] = v;
    __syncthreads();
    float m = red[0];
    for (uint32_t i = 1; i < nw; ++i) m = fmaxf(m, red[i]);
    return m;
}

// x = embedding row io->token of w (src/kernels.cpp:170-176).
__global__ void embed_kernel(uint32_t type, const uint8_t* __restrict__ w, uint64_t cols, uint64_t rows,
                             const DecodeIo* __restrict__ io, float* __restrict__ x, DeviceStatus* st) {
    dep_wait();
    dep_launch();
    const uint32_t tok = io->token;
    if (tok >= rows) {
        if (threadIdx.x == 0 && blockIdx.x == 0) atomicOr(&st->flags, kErrArgument);
        return;
    }
    for (uint64_t i = blockIdx.x * blockDim.x + threadIdx.x; i < cols; i += gridDim.x * blockDim.x) {
        float v;
        if (type == kF16) {
            const uint16_t* r = reinterpret_cast<const uint16_t*>(w + tok * cols * 2u);
            v = half_bits_to_float(r[i]);
        } else {
            const uint64_t bb = type == kQ8_0 ? 34u : 18u;
            const uint8_t* blk = w + tok * (cols / 32u) * bb + (i / 32u) * bb;
            const float d = half_bits_to_float(static_cast<uint32_t>(blk[0]) | (static_cast<uint32_t>(blk[1]) << 8));
            const uint32_t j = i % 32u;
            if (type == kQ8_0) {
                v = d * static_cast<float>(static_cast<int8_t>(blk[2 + j]));
            } else {
                const uint8_t q = blk[2 + (j & 15u)];
                v = d * static_cast<float>((j < 16 ? (q & 15) : (q >> 4)) - 8);
            }
        }
        x[i] = v;
    }
}

// x += delta (when given), then y = x * (1 / sqrt(mean(x^2) + eps)) * w
// (src/kernels.cpp:50-72, the sum of squares in double).  One CTA.
__global__ void add_rmsnorm_kernel(float* __restrict__ x, const float* __restrict__ delta, const void* __restrict__ w,
                                   uint32_t wtype, float* __restrict__ y, uint32_t n, float eps) {
    __shared__ double red[32];
    dep_wait();
    dep_launch();
    double ss = 0.0;
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
        float v = x[i];
        if (delta) {
            v += delta[i];
            x[i] = v;
        }
        ss += static_cast<double>(v) * static_cast<double>(v);
    }
    ss = block_sum(ss, red);
    const float inv = 1.0f / sqrtf(static_cast<float>(ss / n) + eps);
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
        const float wv = wtype == kF32Type ? reinterpret_cast<const float*>(w)[i]
                                            : half_bits_to_float(reinterpret_cast<const uint16_t*>(w)[i]);
        y[i] = x[i] * inv * wv;
    }
}

// RoPE on the q and k heads of the fused projection output qkv = [q | k | v]
// (src/kernels.cpp:93-105), then k and v into cache slot pos % window.
// One CTA per q or k head, hd / 2 threads.
__global__ void rope_kv_kernel(float* __restrict__ qkv, uint32_t nq, uint32_t nkv, uint32_t hd, float theta,
                               const DecodeIo* __restrict__ io, float* __restrict__ kcache,
                               float* __restrict__ vcache, uint32_t window) {
    dep_wait();
    dep_launch();
    const uint64_t pos = io->pos;
    const uint32_t h = blockIdx.x, half = hd / 2u, i = threadIdx.x;
    const uint32_t kvd = nkv * hd;
    float* v = qkv + static_cast<size_t>(h) * hd;  // q heads, then k heads
    if (i < half) {
        const float freq = powf(theta, -2.0f * static_cast<float>(i) / static_cast<float>(hd));
        const float a = static_cast<float>(pos) * freq;
        const float c = cosf(a), s = sinf(a);
        const float x0 = v[i], y0 = v[i + half];
        const float r0 = x0 * c - y0 * s, r1 = x0 * s + y0 * c;
        v[i] = r0;
        v[i + half] = r1;
        if (h >= nq) {
            const size_t slot = static_cast<size_t>(pos % window) * kvd + static_cast<size_t>(h - nq) * hd;
            const float* vv = qkv + static_cast<size_t>(nq) * hd + kvd + static_cast<size_t>(h - nq) * hd;
            kcache[slot + i] = r0;
            kcache[slot + i + half] = r1;
            vcache[slot + i] = vv[i];
            vcache[slot + i + half] = vv[i + half];
        }
    }
}

// One attention head per CTA over the window's keys (src/model.cpp:228-247):
// scores q.k / sqrt(hd) with the dot in double, softmax, weighted sum of the
// values.  Warps take keys round-robin; the value sums of each warp are added
// in warp order.
constexpr uint32_t kAttnThreads = 256;
__global__ void __launch_bounds__(kAttnThreads) attention_kernel(const float* __restrict__ qkv,
                                                                 const float* __restrict__ kcache,
                                                                 const float* __restrict__ vcache,
                                                                 float* __restrict__ att, const DecodeIo* io,
                                                                 uint32_t nq, uint32_t nkv, uint32_t hd,
                                                                 uint32_t window, float inv_sqrt_hd) {
    extern __shared__ float sc[];  // [window] scores, then [8][hd] partial value sums
    __shared__ float red[32];
    dep_wait();
    dep_launch();
    const uint64_t pos = io->pos;
    const uint32_t h = blockIdx.x, kh = h / (nq / nkv), kvd = nkv * hd;
    const uint64_t start = pos + 1 > window ? pos + 1 - window : 0;
    const uint32_t nctx = static_cast<uint32_t>(pos - start + 1);
    const float* q = qkv + static_cast<size_t>(h) * hd;
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u, nw = kAttnThreads / 32u;
    for (uint32_t j = warp; j < nctx; j += nw) {
        const uint32_t slot = static_cast<uint32_t>((start + j) % window);
        const float* k = kcache + static_cast<size_t>(slot) * kvd + static_cast<size_t>(kh) * hd;
        double s = 0.0;
        for (uint32_t d = lane; d < hd; d += 32u) s += static_cast<double>(q[d]) * static_cast<double>(k[d]);
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xFFFFFFFFu, s, o);
        if (lane == 0) sc[j] = static_cast<float>(s) * inv_sqrt_hd;
    }
    __syncthreads();
    float m = -INFINITY;
    for (uint32_t j = threadIdx.x; j < nctx; j += kAttnThreads) m = fmaxf(m, sc[j]);
    m = block_max(m, red);
    float part = 0.f;
    for (uint32_t j = threadIdx.x; j < nctx; j += kAttnThreads) {
        const float e = expf(sc[j] - m);
        sc[j] = e;
        part += e;
    }
    const float inv = 1.0f / block_sum(part, red);
    __syncthreads();
    float* pv = sc + window;  // [nw][hd]
    for (uint32_t d = lane; d < hd; d += 32u) {
        float acc = 0.f;
        for (uint32_t j = warp; j < nctx; j += nw) {
            const uint32_t slot = static_cast<uint32_t>((start + j) % window);
            acc = fmaf(sc[j] * inv, vcache[static_cast<size_t>(slot) * kvd + static_cast<size_t>(kh) * hd + d], acc);
        }
        pv[warp * hd + d] = acc;
    }
    __syncthreads();
    for (uint32_t d = threadIdx.x; d < hd; d += kAttnThreads) {
        float s = pv[d];
        for (uint32_t w = 1; w < nw; ++w) s += pv[w * hd + d];
        att[static_cast<size_t>(h) * hd + d] = s;
    }
}

// gate = silu(gate) * up with gu = [gate | up] (src/kernels.cpp:88-91), then
// the MorphFFN masking of the trailing layers (src/model.cpp:196-209): the
// root and suffix neuron ranges are zeroed when the token's routing flags are
// below 0.5.
__global__ void silu_mul_kernel(float* __restrict__ gu, uint32_t f, const float* __restrict__ route,
                                const DecodeIo* __restrict__ io, uint32_t shared_w, uint32_t root_w,
                                uint32_t suffix_w) {
    dep_wait();
    dep_launch();
    bool mask_root = false, mask_suffix = false;
    if (route) {
        const uint32_t tok = io->token;
        mask_root = route[2u * tok] < 0.5f;
        mask_suffix = route[2u * tok + 1u] < 0.5f;
    }
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < f; i += gridDim.x * blockDim.x) {
        const float v = gu[i];
        float g = (v / (1.0f + expf(-v))) * gu[f + i];
        if (route) {
            const bool in_root = i >= shared_w && i < shared_w + root_w;
            const bool in_suffix = i >= shared_w + root_w && i < shared_w + root_w + suffix_w;
            if ((in_root && mask_root) || (in_suffix && mask_suffix)) g = 0.f;
        }
        gu[i] = g;
    }
}

template <typename K, typename... Args>
cudaError_t launch(K kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t stream, bool pdl, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

}  // namespace

cudaError_t launch_embed(uint32_t type, const void* w, uint64_t cols, uint64_t rows, const DecodeIo* io, float* x,
                         DeviceStatus* st, cudaStream_t stream, bool pdl) {
    const uint32_t grid = static_cast<uint32_t>((cols + 1023) / 1024);
    return launch(embed_kernel, dim3(grid), dim3(256), 0, stream, pdl, type, static_cast<const uint8_t*>(w), cols,
                  rows, io, x, st);
}

cudaError_t launch_add_rmsnorm(float* x, const float* delta, const void* w, uint32_t wtype, float* y, uint32_t n,
                               float eps, cudaStream_t stream, bool pdl) {
    return launch(add_rmsnorm_kernel, dim3(1), dim3(1024), 0, stream, pdl, x, delta, w, wtype, y, n, eps);
}

cudaError_t launch_rope_kv(float* qkv, uint32_t nq, uint32_t nkv, uint32_t hd, float theta, const DecodeIo* io,
                           float* kcache, float* vcache, uint32_t window, cudaStream_t stream, bool pdl) {
    const uint32_t threads = (hd / 2u + 31u) / 32u * 32u;
    return launch(rope_kv_kernel, dim3(nq + nkv), dim3(threads), 0, stream, pdl, qkv, nq, nkv, hd, theta, io, kcache,
                  vcache, window);
}

size_t attention_smem_bytes(uint32_t window, uint32_t hd) {
    return (static_cast<size_t>(window) + static_cast<size_t>(kAttnThreads / 32u) * hd) * sizeof(float);
}

cudaError_t launch_attention(const float* qkv, const float* kcache, const float* vcache, float* att,
                             const DecodeIo* io, uint32_t nq, uint32_t nkv, uint32_t hd, uint32_t window,
                             float inv_sqrt_hd, cudaStream_t stream, bool pdl) {
    const size_t smem = attention_smem_bytes(window, hd);
    if (smem > 48u * 1024u) {
        cudaError_t e = cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(smem));
        if (e != cudaSuccess) return e;
    }
    return launch(attention_kernel, dim3(nq), dim3(kAttnThreads), smem, stream, pdl, qkv, kcache, vcache, att, io, nq,
                  nkv, hd, window, inv_sqrt_hd);
}

cudaError_t launch_silu_mul(float* gu, uint32_t f, const float* route, const DecodeIo* io, uint32_t shared_w,
                            uint32_t root_w, uint32_t suffix_w, cudaStream_t stream, bool pdl) {
    const uint32_t grid = (f + 1023u) / 1024u;
    return launch(silu_mul_kernel, dim3(grid), dim3(256), 0, stream, pdl, gu, f, route, io, shared_w, root_w,
                  suffix_w);
}

}  // namespace nedo_gpu
