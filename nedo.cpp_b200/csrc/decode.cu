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
//   * before the dependency wait, the split's cached keys and values are
//     copied into shared memory (cp.async, L2 only): the cache was written by
//     earlier passes, which completed before the previous kernel of this pass
//     passed its own dependency wait, and the position comes from `io`, which
//     the previous pass's last kernel (or the host) wrote.  The q|k|v
//     projection before this kernel prefetches the same rows into L2, so the
//     copies are L2 hits (copies still in flight delay this kernel's
//     dependency wait: measured ~4.7 us for 6 MB from HBM, ~3.6 us from L2);
//   * RoPE of q_h (every CTA of the head computes the same rotated vector);
//   * the current position's key and value (the last key of the window) are
//     rotated / copied from qkv by the CTA whose split holds that key; the
//     first query head of each KV group also writes them into cache slot
//     pos % window (no CTA of this pass reads that slot from the cache: its
//     previous occupant is outside the window);
//   * scores q.k / sqrt(hd) with the dot in double (lane = key, the warps a
//     quarter of the dimensions each, added in warp order), the split's
//     maximum m_s, e_j = exp(score_j - m_s), l_s = sum e_j and
//     acc_s[d] = sum_j e_j v_j[d] (keys in order);
//   * the last of the head's non-empty splits to finish (a self-resetting
//     counter) adds them in split order, out[d] = sum_s acc_s[d] w_s /
//     sum_s l_s w_s with w_s = exp(m_s - M), M the running maximum over rounds
//     of 32 splits -- the same result whichever CTA is last.  Splits past the
//     window's keys do nothing.
constexpr uint32_t kKeys = 32;  // keys per split: one per lane
constexpr uint32_t kAttnWarps = 4;
constexpr uint32_t kAttnThreads = 32 * kAttnWarps;

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}

// Threads per value dimension: the largest power of two <= kAttnThreads / hd (>= 1).
__host__ __device__ constexpr uint32_t value_parts(uint32_t hd) {
    uint32_t p = 1;
    while (2u * p * hd <= kAttnThreads) p *= 2u;
    return p;
}

// Shared floats of attention_kernel: keys and values [kKeys][hd + 4], q [hd],
// the value partials [max(kAttnThreads, hd)].
__host__ __device__ constexpr size_t attention_smem_floats(uint32_t hd) {
    return 2u * kKeys * static_cast<size_t>(hd + 4u) + static_cast<size_t>(hd) +
           (hd > kAttnThreads ? hd : kAttnThreads);
}

__global__ void __launch_bounds__(kAttnThreads) attention_kernel(
    const float* __restrict__ qkv, float* __restrict__ kcache, float* __restrict__ vcache, float* __restrict__ part,
    float* __restrict__ att, uint32_t* __restrict__ counter, const DecodeIo* io, uint32_t nq, uint32_t nkv, uint32_t hd,
    uint32_t window, float theta, float inv_sqrt_hd) {
    extern __shared__ __align__(16) float sm[];
    __shared__ double dpart[kAttnWarps][kKeys];
    __shared__ float ew[kKeys];
    __shared__ float ml[2];
    __shared__ uint32_t last;
    const uint32_t pitch = hd + 4u;  // an odd number of float4s: lane-per-row reads hit distinct banks
    float* ks = sm;
    float* vs = ks + kKeys * pitch;
    float* qs = vs + kKeys * pitch;
    float* vp = qs + hd;
    const uint64_t pos = __ldcg(reinterpret_cast<const unsigned long long*>(&io->pos));
    const uint32_t s = blockIdx.x, h = blockIdx.y, qpk = nq / nkv, kh = h / qpk, kvd = nkv * hd;
    const uint32_t t = threadIdx.x, half = hd / 2u;
    const uint32_t warp = t >> 5, lane = t & 31u, hd4 = hd / 4u;
    const uint64_t start = pos + 1 > window ? pos + 1 - window : 0;
    const uint32_t nctx = static_cast<uint32_t>(pos - start + 1);
    const uint32_t nused = (nctx + kKeys - 1u) / kKeys;  // splits holding keys
    const uint32_t j0 = s * kKeys;
    if (s >= nused) return;  // reads and writes nothing
    const uint32_t nk = nctx - j0 < kKeys ? nctx - j0 : kKeys;
    const uint32_t jcur = nctx - 1;  // the current position's key
    const bool has_cur = jcur >= j0 && jcur < j0 + nk;
    const size_t cur_slot = static_cast<size_t>(pos % window) * kvd + static_cast<size_t>(kh) * hd;
    for (uint32_t i = t; i < nk * hd4; i += kAttnThreads) {
        const uint32_t j = i / hd4, c = i - j * hd4;
        if (j0 + j == jcur) continue;
        const size_t off = static_cast<size_t>((start + j0 + j) % window) * kvd + static_cast<size_t>(kh) * hd + 4u * c;
        cp_async16(ks + j * pitch + 4u * c, kcache + off);
        cp_async16(vs + j * pitch + 4u * c, vcache + off);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
    dep_wait();
    dep_launch();
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
            const float k0 = kx * c - ky * sn, k1 = kx * sn + ky * c;
            const float v0 = v[i], v1 = v[i + half];
            float* kr = ks + (jcur - j0) * pitch;
            float* vr = vs + (jcur - j0) * pitch;
            kr[i] = k0;
            kr[i + half] = k1;
            vr[i] = v0;
            vr[i + half] = v1;
            if (h % qpk == 0) {
                kcache[cur_slot + i] = k0;
                kcache[cur_slot + i + half] = k1;
                vcache[cur_slot + i] = v0;
                vcache[cur_slot + i + half] = v1;
            }
        }
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();
    // scores: lane = key, warp w the dimension chunks w, w + 4, ...
    {
        double acc = 0.0;
        if (lane < nk) {
            const float4* kr = reinterpret_cast<const float4*>(ks + lane * pitch);
            const float4* q4p = reinterpret_cast<const float4*>(qs);
            for (uint32_t c = warp; c < hd4; c += kAttnWarps) {
                const float4 q4 = q4p[c], k4 = kr[c];
                acc += static_cast<double>(q4.x) * k4.x;
                acc += static_cast<double>(q4.y) * k4.y;
                acc += static_cast<double>(q4.z) * k4.z;
                acc += static_cast<double>(q4.w) * k4.w;
            }
        }
        dpart[warp][lane] = acc;
    }
    __syncthreads();
    if (warp == 0) {
        double d = dpart[0][lane];
        for (uint32_t w = 1; w < kAttnWarps; ++w) d += dpart[w][lane];
        const float sc = lane < nk ? static_cast<float>(d) * inv_sqrt_hd : -INFINITY;
        float m = sc;
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
        const float e = lane < nk ? expf(sc - m) : 0.f;
        float l = e;
        for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xFFFFFFFFu, l, o);
        ew[lane] = e;
        if (lane == 0) {
            ml[0] = m;
            ml[1] = l;
        }
    }
    __syncthreads();
    // values: P threads per dimension, each a contiguous run of kKeys / P keys
    float* out = part + (static_cast<size_t>(h) * gridDim.x + s) * (hd + 2u);
    {
        const uint32_t P = value_parts(hd), run = kKeys / P;
        for (uint32_t i = t; i < hd * P; i += kAttnThreads) {
            const uint32_t d = i % hd, p = i / hd;
            float acc = 0.f;
            for (uint32_t j = p * run; j < p * run + run && j < nk; ++j) acc = fmaf(ew[j], vs[j * pitch + d], acc);
            vp[p * hd + d] = acc;
        }
        __syncthreads();
        for (uint32_t d = t; d < hd; d += kAttnThreads) {
            float acc = vp[d];
            for (uint32_t p = 1; p < P; ++p) acc += vp[p * hd + d];
            out[d] = acc;
        }
        if (t == 0) {
            out[hd] = ml[0];
            out[hd + 1] = ml[1];
        }
    }
    // the last non-empty split of the head combines them.  The CTA barrier orders
    // every thread's partial stores before thread 0's acquire-release add on the
    // counter (cumulative at GPU scope); in the last CTA that add has acquired every
    // other split's release, and the barrier after it passes that on to all threads.
    __syncthreads();
    if (t == 0) {
        uint32_t prev;
        asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(prev) : "l"(counter + h) : "memory");
        last = prev == nused - 1u ? 1u : 0u;
    }
    __syncthreads();
    if (!last) return;
    // each thread's dimension: the splits' (m, l) and value sums, 32 splits per
    // round of loads, folded in split order with a running maximum (the same
    // maxima in every thread)
    const float* p = part + static_cast<size_t>(h) * gridDim.x * (hd + 2u);
    for (uint32_t d = t; d < hd; d += kAttnThreads) {
        float M = -INFINITY, L = 0.f, O = 0.f;
        for (uint32_t i0 = 0; i0 < nused; i0 += 32u) {
            const uint32_t nb = nused - i0 < 32u ? nused - i0 : 32u;
            float mi[32], li[32], ai[32];
#pragma unroll
            for (uint32_t k2 = 0; k2 < 32; ++k2) {
                if (k2 < nb) {
                    const float* pk = p + static_cast<size_t>(i0 + k2) * (hd + 2u);
                    mi[k2] = __ldcg(pk + hd);
                    li[k2] = __ldcg(pk + hd + 1u);
                    ai[k2] = __ldcg(pk + d);
                }
            }
            float mb = M;
#pragma unroll
            for (uint32_t k2 = 0; k2 < 32; ++k2)
                if (k2 < nb) mb = fmaxf(mb, mi[k2]);
            const float sc = expf(M - mb);  // 0 on the first round
            L *= sc;
            O *= sc;
#pragma unroll
            for (uint32_t k2 = 0; k2 < 32; ++k2) {
                if (k2 < nb) {
                    const float w = expf(mi[k2] - mb);
                    L = fmaf(li[k2], w, L);
                    O = fmaf(ai[k2], w, O);
                }
            }
            M = mb;
        }
        att[static_cast<size_t>(h) * hd + d] = O / L;
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
    const size_t smem = attention_smem_floats(hd) * sizeof(float);
    if (smem > 200u * 1024u) return cudaErrorInvalidValue;
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
