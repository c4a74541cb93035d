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
// (src/kernels.cpp:50-72, the sum of squares in double).  One CTA of
// kNormThreads: all loads (x, delta, w) are issued in one pass and staged in
// shared memory, so the kernel waits on memory once.
constexpr uint32_t kNormThreads = 256;
__global__ void __launch_bounds__(kNormThreads) add_rmsnorm_kernel(float* __restrict__ x,
                                                                   const float* __restrict__ delta,
                                                                   const void* __restrict__ w, uint32_t wtype,
                                                                   float* __restrict__ y, uint32_t n, float eps) {
    extern __shared__ float xs[];  // [n] x + delta, then [n] w
    __shared__ double red[kNormThreads / 32];
    dep_wait();
    dep_launch();
    float* wsm = xs + n;
    double ss = 0.0;
    for (uint32_t i = threadIdx.x; i < n; i += kNormThreads) {
        float v = x[i];
        const float wv = wtype == kF32Type ? reinterpret_cast<const float*>(w)[i]
                                            : half_bits_to_float(reinterpret_cast<const uint16_t*>(w)[i]);
        if (delta) {
            v += delta[i];
            x[i] = v;
        }
        xs[i] = v;
        wsm[i] = wv;
        ss += static_cast<double>(v) * static_cast<double>(v);
    }
    ss = block_sum(ss, red);
    const float inv = 1.0f / sqrtf(static_cast<float>(ss / n) + eps);
    for (uint32_t i = threadIdx.x; i < n; i += kNormThreads) y[i] = xs[i] * inv * wsm[i];
}

// One attention step of the pass (src/model.cpp:218-247), RoPE
// (src/kernels.cpp:93-105) and the KV-cache write included, split over keys.
// CTA (s, h) takes keys [s * kKeys, (s + 1) * kKeys) of the window of query
// head h:
//   * RoPE of q_h (every CTA of the head computes the same rotated vector);
//   * the current position's key and value (the last key of the window) are
//     rotated / copied from qkv by the CTAs whose split holds that key and used
//     from shared memory; the first query head of each KV group also writes
//     them into cache slot pos % window (no CTA of this pass reads that slot
//     from the cache: its previous occupant is outside the window);
//   * scores q.k / sqrt(hd) with the dot in double (two threads per key, half
//     the dimensions each), the split's maximum m_s, e_j = exp(score_j - m_s),
//     l_s = sum e_j and acc_s[d] = sum_j e_j v_j[d] (keys in order);
//   * the last CTA of the head to finish (a self-resetting counter) adds the
//     splits in split order: out[d] = sum_s acc_s[d] w_s / sum_s l_s w_s with
//     w_s = exp(m_s - M), M = max_s m_s -- the same result whichever CTA is last.
constexpr uint32_t kKeys = 64;
constexpr uint32_t kAttnWarps = 4;
constexpr uint32_t kAttnThreads = 32 * kAttnWarps;
constexpr uint32_t kKeysPerWarp = kKeys / kAttnWarps;
__global__ void __launch_bounds__(kAttnThreads) attention_kernel(
    const float* __restrict__ qkv, float* __restrict__ kcache, float* __restrict__ vcache, float* __restrict__ part,
    float* __restrict__ att, uint32_t* __restrict__ counter, const DecodeIo* io, uint32_t nq, uint32_t nkv, uint32_t hd,
    uint32_t window, float theta, float inv_sqrt_hd) {
    // q rotated [hd], current k [hd], current v [hd], value sums [warps][hd], split weights [nsplit]
    extern __shared__ __align__(16) float sm[];
    __shared__ float sc[kKeys];
    __shared__ float red[kAttnWarps];
    __shared__ uint32_t last;
    dep_wait();
    dep_launch();
    const uint64_t pos = io->pos;
    const uint32_t s = blockIdx.x, h = blockIdx.y, qpk = nq / nkv, kh = h / qpk, kvd = nkv * hd;
    const uint32_t nsplit = gridDim.x, t = threadIdx.x, half = hd / 2u;
    const uint32_t warp = t >> 5, lane = t & 31u, hd4 = hd / 4u;
    float* qs = sm;
    float* kcur = sm + hd;
    float* vcur = sm + 2u * hd;
    float* pv = sm + 3u * hd;
    float* wsp = sm + (3u + kAttnWarps) * hd;
    const uint64_t start = pos + 1 > window ? pos + 1 - window : 0;
    const uint32_t nctx = static_cast<uint32_t>(pos - start + 1);
    const uint32_t j0 = s * kKeys;
    const uint32_t nk = nctx > j0 ? (nctx - j0 < kKeys ? nctx - j0 : kKeys) : 0u;
    const uint32_t jcur = nctx - 1;  // the current position's key
    const bool has_cur = nk > 0 && jcur >= j0 && jcur < j0 + nk;
    const size_t cur_slot = static_cast<size_t>(pos % window) * kvd + static_cast<size_t>(kh) * hd;
    float* out = part + (static_cast<size_t>(h) * nsplit + s) * (hd + 2u);
    if (nk > 0) {
        const float* q = qkv + static_cast<size_t>(h) * hd;
        const float* k = qkv + static_cast<size_t>(nq) * hd + static_cast<size_t>(kh) * hd;
        const float* v = qkv + static_cast<size_t>(nq) * hd + kvd + static_cast<size_t>(kh) * hd;
        for (uint32_t i = t; i < half; i += kAttnThreads) {
            const float freq = powf(theta, -2.0f * static_cast<float>(i) / static_cast<float>(hd));
            const float a = static_cast<float>(pos) * freq;
            const float c = cosf(a), sn = sinf(a);
            const float x0 = q[i], y0 = q[i + half];
            qs[i] = x0 * c - y0 * sn;
            qs[i + half] = x0 * sn + y0 * c;
            if (has_cur) {
                const float kx = k[i], ky = k[i + half];
                kcur[i] = kx * c - ky * sn;
                kcur[i + half] = kx * sn + ky * c;
                vcur[i] = v[i];
                vcur[i + half] = v[i + half];
            }
        }
        __syncthreads();
        if (has_cur && h % qpk == 0) {
            for (uint32_t d = t; d < hd; d += kAttnThreads) {
                kcache[cur_slot + d] = kcur[d];
                vcache[cur_slot + d] = vcur[d];
            }
        }
        // scores: warp w takes keys w * kKeysPerWarp .. + kKeysPerWarp, the lanes a
        // key's dimensions as float4s (coalesced rows, all the warp's keys in flight)
        const float* krow[kKeysPerWarp];
#pragma unroll
        for (uint32_t i = 0; i < kKeysPerWarp; ++i) {
            const uint32_t j = warp * kKeysPerWarp + i;
            const uint32_t slot = static_cast<uint32_t>((start + j0 + j) % window);
            krow[i] = (j0 + j == jcur) ? kcur : kcache + static_cast<size_t>(slot) * kvd + static_cast<size_t>(kh) * hd;
        }
        double pacc[kKeysPerWarp];
#pragma unroll
        for (uint32_t i = 0; i < kKeysPerWarp; ++i) pacc[i] = 0.0;
        for (uint32_t d4 = lane; d4 < hd4; d4 += 32u) {
            const float4 q4 = reinterpret_cast<const float4*>(qs)[d4];
            float4 kk[kKeysPerWarp];
#pragma unroll
            for (uint32_t i = 0; i < kKeysPerWarp; ++i)
                kk[i] = warp * kKeysPerWarp + i < nk ? reinterpret_cast<const float4*>(krow[i])[d4]
                                                     : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (uint32_t i = 0; i < kKeysPerWarp; ++i) {
                pacc[i] += static_cast<double>(q4.x) * kk[i].x;
                pacc[i] += static_cast<double>(q4.y) * kk[i].y;
                pacc[i] += static_cast<double>(q4.z) * kk[i].z;
                pacc[i] += static_cast<double>(q4.w) * kk[i].w;
            }
        }
#pragma unroll
        for (uint32_t i = 0; i < kKeysPerWarp; ++i) {
            double dsum = pacc[i];
            for (int o = 16; o > 0; o >>= 1) dsum += __shfl_xor_sync(0xFFFFFFFFu, dsum, o);
            const uint32_t j = warp * kKeysPerWarp + i;
            if (lane == 0) sc[j] = j < nk ? static_cast<float>(dsum) * inv_sqrt_hd : -INFINITY;
        }
        __syncthreads();
        float m = t < kKeys ? sc[t] : -INFINITY;
        m = block_max(m, red);
        const float e = (t < kKeys && t < nk) ? expf(sc[t] - m) : 0.f;
        __syncthreads();
        if (t < kKeys) sc[t] = e;
        const float l = block_sum(e, red);
        __syncthreads();
        // values: the same split of keys over warps, float4s over the lanes
        for (uint32_t d4 = lane; d4 < hd4; d4 += 32u) {
            float4 vv[kKeysPerWarp];
#pragma unroll
            for (uint32_t i = 0; i < kKeysPerWarp; ++i) {
                const uint32_t j = warp * kKeysPerWarp + i;
                const uint32_t slot = static_cast<uint32_t>((start + j0 + j) % window);
                const float* vr = (j0 + j == jcur) ? vcur
                                                   : vcache + static_cast<size_t>(slot) * kvd + static_cast<size_t>(kh) * hd;
                vv[i] = j < nk ? reinterpret_cast<const float4*>(vr)[d4] : make_float4(0.f, 0.f, 0.f, 0.f);
            }
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (uint32_t i = 0; i < kKeysPerWarp; ++i) {
                const float ej = sc[warp * kKeysPerWarp + i];
                acc.x = fmaf(ej, vv[i].x, acc.x);
                acc.y = fmaf(ej, vv[i].y, acc.y);
                acc.z = fmaf(ej, vv[i].z, acc.z);
                acc.w = fmaf(ej, vv[i].w, acc.w);
            }
            reinterpret_cast<float4*>(pv + warp * hd)[d4] = acc;
        }
        __syncthreads();
        for (uint32_t d = t; d < hd; d += kAttnThreads) {
            float acc = pv[d];
            for (uint32_t w = 1; w < kAttnWarps; ++w) acc += pv[w * hd + d];
            out[d] = acc;
        }
        if (t == 0) {
            out[hd] = m;
            out[hd + 1] = l;
        }
    } else {
        // no keys in this split: m = -inf, l = 0
        for (uint32_t d = t; d < hd; d += kAttnThreads) out[d] = 0.f;
        if (t == 0) {
            out[hd] = -INFINITY;
            out[hd + 1] = 0.f;
        }
    }
    // the last CTA of the head combines the splits
    __threadfence();
    __syncthreads();
    if (t == 0) last = atomicAdd(&counter[h], 1u) == nsplit - 1u ? 1u : 0u;
    __syncthreads();
    if (!last) return;
    __threadfence();
    // every split's (m, l) in one round of loads, the weights w_s = exp(m_s - M)
    // in shared memory, then the value sums (loads of all splits in flight)
    const float* p = part + static_cast<size_t>(h) * nsplit * (hd + 2u);
    float mloc = -INFINITY;
    for (uint32_t i = t; i < nsplit; i += kAttnThreads) {
        const float mi = __ldcg(p + static_cast<size_t>(i) * (hd + 2u) + hd);
        wsp[i] = mi;
        mloc = fmaxf(mloc, mi);
    }
    const float mx = block_max(mloc, red);
    float lloc = 0.f;
    for (uint32_t i = t; i < nsplit; i += kAttnThreads) {
        const float wi = expf(wsp[i] - mx);
        wsp[i] = wi;
        lloc += __ldcg(p + static_cast<size_t>(i) * (hd + 2u) + hd + 1u) * wi;
    }
    const float L = block_sum(lloc, red);
    __syncthreads();
    const float inv = 1.0f / L;
    for (uint32_t d = t; d < hd; d += kAttnThreads) {
        float acc = 0.f;
#pragma unroll 8
        for (uint32_t i = 0; i < nsplit; ++i) acc = fmaf(__ldcg(p + static_cast<size_t>(i) * (hd + 2u) + d), wsp[i], acc);
        att[static_cast<size_t>(h) * hd + d] = acc * inv;
    }
    if (t == 0) counter[h] = 0u;
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

// Greedy generation on the device: the pass's pick becomes the next pass's
// token (io->token), the position advances, and the pick is recorded at
// ids[io->step] (src/model.cpp:271-279 without the host round trip).
__global__ void advance_kernel(DecodeIo* io, const int64_t* __restrict__ pick, uint32_t* __restrict__ ids,
                               uint32_t cap) {
    const uint32_t next = static_cast<uint32_t>(pick[0]);
    const uint32_t k = io->step;
    if (k < cap) ids[k] = next;
    io->step = k + 1u;
    io->token = next;
    io->pos += 1u;
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
    const size_t smem = 2u * static_cast<size_t>(n) * sizeof(float);
    if (smem > 48u * 1024u) {
        if (smem > 200u * 1024u) return cudaErrorInvalidValue;
        cudaError_t e = cudaFuncSetAttribute(add_rmsnorm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(smem));
        if (e != cudaSuccess) return e;
    }
    return launch(add_rmsnorm_kernel, dim3(1), dim3(kNormThreads), smem, stream, pdl, x, delta, w, wtype, y, n, eps);
}

uint32_t attention_splits(uint32_t window) { return (window + kKeys - 1) / kKeys; }

cudaError_t launch_attention(const float* qkv, float* kcache, float* vcache, float* att, float* part,
                             uint32_t* counter, const DecodeIo* io, uint32_t nq, uint32_t nkv, uint32_t hd,
                             uint32_t window, float theta, float inv_sqrt_hd, cudaStream_t stream, bool pdl) {
    const uint32_t ns = attention_splits(window);
    // q, current k and v, the warps' value sums, the split weights
    const size_t smem = ((3u + kAttnWarps) * static_cast<size_t>(hd) + ns) * sizeof(float);
    if (smem > 48u * 1024u) {
        cudaError_t e = cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(smem));
        if (e != cudaSuccess) return e;
    }
    return launch(attention_kernel, dim3(ns, nq), dim3(kAttnThreads), smem, stream, pdl, qkv, kcache, vcache, part,
                  att, counter, io, nq, nkv, hd, window, theta, inv_sqrt_hd);
}

cudaError_t launch_advance(DecodeIo* io, const int64_t* pick, uint32_t* ids, uint32_t cap, cudaStream_t stream) {
    advance_kernel<<<1, 1, 0, stream>>>(io, pick, ids, cap);
    return cudaGetLastError();
}

cudaError_t launch_silu_mul(float* gu, uint32_t f, const float* route, const DecodeIo* io, uint32_t shared_w,
                            uint32_t root_w, uint32_t suffix_w, cudaStream_t stream, bool pdl) {
    const uint32_t grid = (f + 255u) / 256u;
    return launch(silu_mul_kernel, dim3(grid), dim3(256), 0, stream, pdl, gu, f, route, io, shared_w, root_w,
                  suffix_w);
}

}  // namespace nedo_gpu
