// topk.cu -- the k largest logits on the device, for the sampling step of the
// LM head (reference src/model.cpp:33-63, sample_token).
//
// sample_token keeps the top_k logits (nth_element + sort by logit, largest
// first) and draws from their tempered softmax.  Done on the host it needs all
// vocab logits (512 KB for 128000) copied back per token; here the candidates
// are selected where the logits are and only k (id, logit) pairs leave the
// device.  Order: logit descending, equal logits by smaller index first (the
// reference's order of equal logits is unspecified); NaN logits are never
// selected ahead of a number.
//
// Each CTA sorts its slice of the vector in chunks of kChunk keys in shared
// memory (bitonic sort), carrying its best kpad keys from chunk to chunk, and
// publishes them; the last CTA to finish (a self-resetting counter) merges all
// CTAs' candidates the same way and writes the k winners.  A key is
// (order-preserving bits of the logit) << 32 | ~index, so a descending sort of
// the 64-bit keys orders by logit and then by index.
#include "common.cuh"
#include "launch.h"

namespace nedo_gpu {
namespace {

constexpr uint32_t kChunk = 2048;   // keys sorted at once
constexpr uint32_t kThreadsTk = 1024;

__device__ __forceinline__ uint64_t topk_key(float f, uint32_t idx) {
    if (f == 0.f) f = 0.f;  // -0 and +0 compare equal: one key
    uint32_t u = __float_as_uint(f);
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);  // ascending floats -> ascending unsigned
    if (f != f) u = 0u;                                // NaN below every number
    return (static_cast<uint64_t>(u) << 32) | static_cast<uint64_t>(~idx);
}

// Bitonic sort of kChunk keys in shared memory, descending, by all threads.
__device__ __forceinline__ void sort_desc(uint64_t* key) {
    for (uint32_t size = 2; size <= kChunk; size <<= 1) {
        for (uint32_t stride = size >> 1; stride > 0; stride >>= 1) {
            __syncthreads();
            for (uint32_t t = threadIdx.x; t < kChunk / 2; t += blockDim.x) {
                const uint32_t i = 2u * t - (t & (stride - 1u));  // first of the pair
                const uint32_t j = i + stride;
                const bool desc = (i & size) == 0u;               // direction of this bitonic run
                const uint64_t a = key[i], b = key[j];
                if ((a < b) == desc) {
                    key[i] = b;
                    key[j] = a;
                }
            }
        }
    }
    __syncthreads();
}

// Best kpad keys of src[0..count) (keys built by `make`) into key[0..kpad),
// keeping key[0..kpad) as the running carry: chunks of kChunk - kpad new keys.
template <typename Make>
__device__ __forceinline__ void select_best(uint64_t* key, uint32_t kpad, uint64_t count, Make make) {
    const uint32_t fresh = kChunk - kpad;
    for (uint64_t base = 0; base < count; base += fresh) {
        for (uint32_t t = threadIdx.x; t < fresh; t += blockDim.x) {
            const uint64_t i = base + t;
            key[kpad + t] = i < count ? make(i) : 0ull;
        }
        sort_desc(key);
    }
}

__global__ void __launch_bounds__(kThreadsTk) topk_kernel(const float* __restrict__ v, uint64_t n, uint32_t k,
                                                         uint32_t kpad, TopkScratch s) {
    __shared__ uint64_t key[kChunk];
    __shared__ uint32_t last;
    for (uint32_t t = threadIdx.x; t < kpad; t += blockDim.x) key[t] = 0ull;
    const uint64_t b0 = n * blockIdx.x / gridDim.x, b1 = n * (blockIdx.x + 1) / gridDim.x;
    select_best(key, kpad, b1 - b0, [&](uint64_t i) {
        const uint64_t g = b0 + i;
        return topk_key(__ldg(v + g), static_cast<uint32_t>(g));
    });
    for (uint32_t t = threadIdx.x; t < kpad; t += blockDim.x) s.cand[static_cast<uint64_t>(blockIdx.x) * kpad + t] = key[t];
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) last = atomicAdd(s.counter, 1u) == gridDim.x - 1u ? 1u : 0u;
    __syncthreads();
    if (last == 0u) return;
    // the last CTA: merge every CTA's candidates
    __threadfence();
    for (uint32_t t = threadIdx.x; t < kpad; t += blockDim.x) key[t] = 0ull;
    const volatile uint64_t* cand = s.cand;
    select_best(key, kpad, static_cast<uint64_t>(gridDim.x) * kpad, [&](uint64_t i) { return cand[i]; });
    for (uint32_t t = threadIdx.x; t < k; t += blockDim.x) {
        const uint32_t idx = ~static_cast<uint32_t>(key[t] & 0xFFFFFFFFull);
        s.ids[t] = idx;
        if (s.vals != nullptr) s.vals[t] = v[idx];
    }
    if (threadIdx.x == 0) *s.counter = 0u;  // ready for the next launch
}

}  // namespace

uint32_t topk_ctas(uint64_t n, uint32_t k, int num_sms) {
    uint32_t kpad = 32;
    while (kpad < k) kpad <<= 1;
    const uint64_t fresh = kChunk - kpad;
    uint64_t g = (n + fresh - 1) / fresh;
    if (g > static_cast<uint64_t>(num_sms)) g = static_cast<uint64_t>(num_sms);
    if (g == 0) g = 1;
    return static_cast<uint32_t>(g);
}

cudaError_t launch_topk(const float* v, uint64_t n, uint32_t k, const TopkScratch& s, int num_sms,
                        cudaStream_t stream) {
    if (n == 0 || n > 0xFFFFFFFFull || k == 0 || k > kTopkMax || k > n) return cudaErrorInvalidValue;
    uint32_t kpad = 32;
    while (kpad < k) kpad <<= 1;
    const uint32_t g = topk_ctas(n, k, num_sms);
    topk_kernel<<<g, kThreadsTk, 0, stream>>>(v, n, k, kpad, s);
    return cudaGetLastError();
}

}  // namespace nedo_gpu
