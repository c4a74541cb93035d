// gemv_stream.cu -- batch-1 dequantize-and-dot matvec over raw GGUF rows.
//
// Replaces the CPU row loop of nedo::kernels::matvec (reference src/kernels.cpp:162-169)
// and its three row kernels dot_f16 / dot_q8 / dot_q4 (src/kernels.cpp:109-160).
//
// Design (one persistent CTA per SM):
//   * The weight matrix is a contiguous stream of rows (rows x row_bytes).  A
//     producer warp moves tiles of `rows_per_tile` whole rows from HBM into a
//     ring of shared-memory stages with one bulk copy per tile (cp.async.bulk,
//     mbarrier complete_tx, L2 evict-first; no multicast).  Tiles are dealt to
//     CTAs round-robin.
//   * Consumer warps are arranged as `groups` x `chunks`.  A group takes every
//     groups-th tile of its CTA; inside a group, warp c owns a fixed slice of
//     the columns (2048 columns) and keeps the matching x values in registers
//     for the whole kernel, so x is read from global memory once per CTA.
//   * Lane l of chunk c owns one *pair* of blocks (Q8_0: 68 bytes, Q4_0: 36
//     bytes), which starts on a 4-byte boundary whatever the block parity, so
//     the lane reads its bytes with aligned 32-bit shared loads and picks the
//     quant bytes with compile-time byte selectors.  F16 lanes read 16-byte
//     vectors at a 512-byte warp stride (conflict free).
//   * Integer quants become fp32 without I2F: PRMT/LOP3 place them in the
//     mantissa of a constant and one packed fp32x2 add removes the constant
//     exactly; products accumulate with packed fp32x2 FMA in fp32.
//   * Each row's lane sums are folded with warp shuffles; the per-chunk sums
//     are folded in fixed order through shared memory (an mbarrier hands them
//     to the chunk-0 warp), so results are bit-reproducible run to run.
//   * Every wait is bounded (2 s); a kernel that gives up records the failure
//     in DeviceStatus and drains its outstanding copies before exiting.
#include <math.h>

#include "common.cuh"
#include "launch.h"

namespace nedo_gpu {
namespace {

// 16 warps of 32 threads leave 120 registers per thread; a 17-warp CTA drops
// to 96 and spills, so 16 consumer warps (rows of more than 15 chunks, i.e.
// more than 30720 columns) use a separate instantiation.
constexpr uint32_t kMaxConsumerWarps = 16;
constexpr uint32_t kThreadsNormal = 16 * 32;
constexpr uint32_t kThreadsWide = 17 * 32;
constexpr uint32_t kMaxRowsPerTile = 8;
constexpr uint32_t kMaxStages = 48;

struct StreamArgs {
    const uint8_t* w;
    const float* x;
    float* y;
    uint64_t rows;
    uint64_t tiles;
    uint32_t cols;
    uint32_t row_bytes;
    uint32_t rows_per_tile;
    uint32_t chunks;
    uint32_t groups;
    uint32_t stages;
    uint32_t stage_bytes;
    uint32_t has_amax;
    DeviceStatus* status;
    ArgmaxScratch amax;
};

// ---------------------------------------------------------------------------
// bounded waits that also observe the CTA-wide abort flag
__device__ __forceinline__ bool wait_phase(uint64_t* bar, uint32_t parity, volatile uint32_t* abort_flag,
                                           DeviceStatus* st, uint32_t site) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*abort_flag) return false;
        if (global_timer_ns() - t0 > kWaitLimitNs) {
            *abort_flag = 1u;
            if (atomicOr(&st->flags, kErrWaitTimeout) == 0u) st->where = site;
            return false;
        }
    }
}

// ---------------------------------------------------------------------------
// Q8_0: a pair of blocks = 68 bytes = 17 aligned words.
//   block 0: scale bytes 0-1, quant i at pair byte 2+i
//   block 1: scale bytes 34-35, quant i at pair byte 36+i
// int8 q -> fp32: u = q ^ 0x80 (offset binary); bits 0x4B0000uu = 2^23 + u;
// subtracting 2^23 + 128 gives q exactly.
struct XQ8 {
    float2 v[32];
};

__device__ __forceinline__ float q8_float(uint32_t word_xor, uint32_t byte) {
    return __uint_as_float(prmt(word_xor, 0x4B000000u, 0x7440u | byte));
}

__device__ __forceinline__ float dot_pair_q8(const uint32_t* __restrict__ wp, const XQ8& x) {
    uint32_t w[17];
#pragma unroll
    for (int i = 0; i < 17; ++i) w[i] = wp[i];
    const float d0 = half_bits_to_float(w[0]);
    const float d1 = half_bits_to_float(w[8] >> 16);
#pragma unroll
    for (int i = 0; i < 17; ++i) w[i] ^= 0x80808080u;
    const float2 bias = make_float2(-8388736.0f, -8388736.0f);
    float2 a0 = make_float2(0.f, 0.f), a1 = a0, b0 = a0, b1 = a0;
#pragma unroll
    for (int k = 0; k < 32; k += 2) {
        const int p0 = 2 + k, p1 = 3 + k;  // block 0 bytes
        float2 q = make_float2(q8_float(w[p0 >> 2], p0 & 3), q8_float(w[p1 >> 2], p1 & 3));
        q = fadd2(q, bias);
        if ((k & 2) == 0) a0 = ffma2(q, x.v[k >> 1], a0); else a1 = ffma2(q, x.v[k >> 1], a1);
        const int r0 = 36 + k, r1 = 37 + k;  // block 1 bytes
        float2 s = make_float2(q8_float(w[r0 >> 2], r0 & 3), q8_float(w[r1 >> 2], r1 & 3));
        s = fadd2(s, bias);
        if ((k & 2) == 0) b0 = ffma2(s, x.v[16 + (k >> 1)], b0); else b1 = ffma2(s, x.v[16 + (k >> 1)], b1);
    }
    const float s0 = (a0.x + a0.y) + (a1.x + a1.y);
    const float s1 = (b0.x + b0.y) + (b1.x + b1.y);
    return fmaf(d0, s0, d1 * s1);
}

// ---------------------------------------------------------------------------
// Q4_0: a pair of blocks = 36 bytes = 9 aligned words.
//   block 0: scale bytes 0-1, quant byte j at pair byte 2+j
//   block 1: scale bytes 18-19, quant byte j at pair byte 20+j
// Nibble n -> fp32 without I2F: shift the word so that the nibble lands on
// mantissa bits 15-18 (low nibbles, f = 1 + n/256) or 19-22 (high nibbles,
// f = 1 + n/16) and OR in the exponent of 1.0.  With x' = 256x (low) and
// x' = 16x (high):  sum (n-8) x = sum f x' - C,  C = sum x' + 8 sum x,
// and C depends on x only (computed once per kernel).
struct XQ4 {
    float2 v[32];  // x' for the pair's 64 elements
    float c0, c1;  // per-block constants
};

template <int M>
__device__ __forceinline__ uint32_t q4_align(uint32_t w) {
    // byte M of the word: bring bits 8M..8M+7 to 15..22
    if constexpr (M == 0) return w << 15;
    else if constexpr (M == 1) return w << 7;
    else if constexpr (M == 2) return w >> 1;
    else return w >> 9;
}

template <int M>
__device__ __forceinline__ float2 q4_lo_hi(uint32_t w) {
    const uint32_t a = q4_align<M>(w);
    return make_float2(__uint_as_float((a & 0x00078000u) | 0x3F800000u),   // low nibble
                       __uint_as_float((a & 0x00780000u) | 0x3F800000u));  // high nibble
}

// quant bytes j, j+1 (j even) of one block: low nibbles are elements j, j+1;
// high nibbles are elements j+16, j+17.
template <int BYTE0>
__device__ __forceinline__ void q4_two_bytes(const uint32_t* w, const float2* xs, float2& acc_lo, float2& acc_hi,
                                             int elem0) {
    constexpr int B1 = BYTE0 + 1;
    const float2 f0 = q4_lo_hi<BYTE0 & 3>(w[BYTE0 >> 2]);
    const float2 f1 = q4_lo_hi<B1 & 3>(w[B1 >> 2]);
    acc_lo = ffma2(make_float2(f0.x, f1.x), xs[elem0 >> 1], acc_lo);
    acc_hi = ffma2(make_float2(f0.y, f1.y), xs[(elem0 + 16) >> 1], acc_hi);
}

template <int BASE_BYTE, int BASE_ELEM>
__device__ __forceinline__ float q4_block(const uint32_t* w, const float2* xs) {
    float2 lo0 = make_float2(0.f, 0.f), lo1 = lo0, hi0 = lo0, hi1 = lo0;
    q4_two_bytes<BASE_BYTE + 0>(w, xs, lo0, hi0, BASE_ELEM + 0);
    q4_two_bytes<BASE_BYTE + 2>(w, xs, lo1, hi1, BASE_ELEM + 2);
    q4_two_bytes<BASE_BYTE + 4>(w, xs, lo0, hi0, BASE_ELEM + 4);
    q4_two_bytes<BASE_BYTE + 6>(w, xs, lo1, hi1, BASE_ELEM + 6);
    q4_two_bytes<BASE_BYTE + 8>(w, xs, lo0, hi0, BASE_ELEM + 8);
    q4_two_bytes<BASE_BYTE + 10>(w, xs, lo1, hi1, BASE_ELEM + 10);
    q4_two_bytes<BASE_BYTE + 12>(w, xs, lo0, hi0, BASE_ELEM + 12);
    q4_two_bytes<BASE_BYTE + 14>(w, xs, lo1, hi1, BASE_ELEM + 14);
    return ((lo0.x + lo0.y) + (lo1.x + lo1.y)) + ((hi0.x + hi0.y) + (hi1.x + hi1.y));
}

__device__ __forceinline__ float dot_pair_q4(const uint32_t* __restrict__ wp, const XQ4& x) {
    uint32_t w[9];
#pragma unroll
    for (int i = 0; i < 9; ++i) w[i] = wp[i];
    const float d0 = half_bits_to_float(w[0]);
    const float d1 = half_bits_to_float(w[4] >> 16);
    const float s0 = q4_block<2, 0>(w, x.v) - x.c0;
    const float s1 = q4_block<20, 32>(w, x.v) - x.c1;
    return fmaf(d0, s0, d1 * s1);
}

// ---------------------------------------------------------------------------
// F16: lane l of chunk c owns elements 2048c + 256i + 8l + j (i, j < 8).
struct XF16 {
    float2 v[32];
};

__device__ __forceinline__ float dot_chunk_f16(const uint8_t* __restrict__ row, const XF16& x, uint32_t chunk,
                                               uint32_t lane, uint32_t cols) {
    float2 a0 = make_float2(0.f, 0.f), a1 = a0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const uint32_t e0 = chunk * 2048u + 256u * i + 8u * lane;
        if (e0 < cols) {
            const uint4 v = *reinterpret_cast<const uint4*>(row + 2u * e0);
            const uint32_t h[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&h[k]));
                if (k & 1) a1 = ffma2(f, x.v[4 * i + k], a1); else a0 = ffma2(f, x.v[4 * i + k], a0);
            }
        }
    }
    return (a0.x + a0.y) + (a1.x + a1.y);
}

// ---------------------------------------------------------------------------
template <uint32_t TYPE>
struct XRegs;
template <>
struct XRegs<kQ8_0> {
    using T = XQ8;
};
template <>
struct XRegs<kQ4_0> {
    using T = XQ4;
};
template <>
struct XRegs<kF16> {
    using T = XF16;
};

template <uint32_t TYPE>
__device__ __forceinline__ void load_x(const StreamArgs& a, uint32_t chunk, uint32_t lane, typename XRegs<TYPE>::T& xr,
                                       bool& valid) {
    if constexpr (TYPE == kF16) {
        valid = true;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t e0 = chunk * 2048u + 256u * i + 8u * lane;
            float4 u = make_float4(0.f, 0.f, 0.f, 0.f), v = u;
            if (e0 < a.cols) {
                u = __ldg(reinterpret_cast<const float4*>(a.x + e0));
                v = __ldg(reinterpret_cast<const float4*>(a.x + e0 + 4));
            }
            xr.v[4 * i + 0] = make_float2(u.x, u.y);
            xr.v[4 * i + 1] = make_float2(u.z, u.w);
            xr.v[4 * i + 2] = make_float2(v.x, v.y);
            xr.v[4 * i + 3] = make_float2(v.z, v.w);
        }
    } else {
        const uint32_t pairs = a.cols / 64u;
        const uint32_t p = chunk * 32u + lane;
        valid = p < pairs;
        const float* xp = a.x + static_cast<size_t>(p) * 64u;
        if constexpr (TYPE == kQ8_0) {
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
                if (valid) t = __ldg(reinterpret_cast<const float4*>(xp) + i);
                xr.v[2 * i] = make_float2(t.x, t.y);
                xr.v[2 * i + 1] = make_float2(t.z, t.w);
            }
        } else {
            float sx0 = 0.f, sx1 = 0.f, sp0 = 0.f, sp1 = 0.f;
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
                if (valid) t = __ldg(reinterpret_cast<const float4*>(xp) + i);
                // element e = 4i .. 4i+3 of the pair; block-local index e & 31
                const float sc = (((4 * i) & 31) < 16) ? 256.0f : 16.0f;
                const float2 lo = make_float2(t.x * sc, t.y * sc), hi = make_float2(t.z * sc, t.w * sc);
                xr.v[2 * i] = lo;
                xr.v[2 * i + 1] = hi;
                if (i < 8) {
                    sx0 += (t.x + t.y) + (t.z + t.w);
                    sp0 += (lo.x + lo.y) + (hi.x + hi.y);
                } else {
                    sx1 += (t.x + t.y) + (t.z + t.w);
                    sp1 += (lo.x + lo.y) + (hi.x + hi.y);
                }
            }
            xr.c0 = fmaf(8.0f, sx0, sp0);
            xr.c1 = fmaf(8.0f, sx1, sp1);
        }
    }
}

template <uint32_t TYPE>
__device__ __forceinline__ float row_partial(const uint8_t* row, const typename XRegs<TYPE>::T& xr, bool valid,
                                             uint32_t chunk, uint32_t lane, uint32_t cols) {
    if constexpr (TYPE == kF16) {
        return dot_chunk_f16(row, xr, chunk, lane, cols);
    } else if constexpr (TYPE == kQ8_0) {
        if (!valid) return 0.f;
        return dot_pair_q8(reinterpret_cast<const uint32_t*>(row + 68u * (chunk * 32u + lane)), xr);
    } else {
        if (!valid) return 0.f;
        return dot_pair_q4(reinterpret_cast<const uint32_t*>(row + 36u * (chunk * 32u + lane)), xr);
    }
}

__device__ __forceinline__ bool amax_better(float v, uint32_t i, float bv, uint32_t bi) {
    return v > bv || (v == bv && i < bi);
}

__device__ __forceinline__ void warp_argmax(float& v, uint32_t& i) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xFFFFFFFFu, v, o);
        const uint32_t oi = __shfl_xor_sync(0xFFFFFFFFu, i, o);
        if (amax_better(ov, oi, v, i)) {
            v = ov;
            i = oi;
        }
    }
}

// ---------------------------------------------------------------------------
template <uint32_t TYPE, uint32_t MAX_THREADS>
__global__ void __launch_bounds__(MAX_THREADS, 1) gemv_stream_kernel(const StreamArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const uint32_t S = a.stages, R = a.rows_per_tile, C = a.chunks, G = a.groups;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + static_cast<size_t>(S) * a.stage_bytes);
    uint64_t* empty = full + S;
    uint64_t* redbar = empty + S;
    float* red = reinterpret_cast<float*>(redbar + S);
    uint32_t* misc = reinterpret_cast<uint32_t*>(red + static_cast<size_t>(S) * R * C);
    volatile uint32_t* abort_flag = misc;
    float* am_val = reinterpret_cast<float*>(misc + 2);
    uint32_t* am_idx = misc + 2 + kMaxConsumerWarps;

    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t consumers = C * G;

    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], C);
            mbar_init(&redbar[s], C);
        }
        *abort_flag = 0u;
        fence_barrier_init();
    }
    __syncthreads();

    if (warp == consumers) {
        // ---------------- producer ----------------
        if (lane == 0) {
            const uint64_t policy = l2_policy_evict_first();
            uint64_t j = 0;
            for (;; ++j) {
                const uint64_t tile = blockIdx.x + j * gridDim.x;
                if (tile >= a.tiles) break;
                const uint32_t slot = static_cast<uint32_t>(j % S);
                const uint32_t use = static_cast<uint32_t>(j / S);
                if (use > 0 && !wait_phase(&empty[slot], (use - 1u) & 1u, abort_flag, a.status, 1u)) break;
                const uint64_t row0 = tile * R;
                const uint64_t left = a.rows - row0;
                const uint32_t nrows = left < R ? static_cast<uint32_t>(left) : R;
                const uint32_t bytes = nrows * a.row_bytes;
                mbar_arrive_expect_tx(&full[slot], bytes);
                bulk_copy_g2s(smem + static_cast<size_t>(slot) * a.stage_bytes, a.w + row0 * a.row_bytes, bytes,
                              &full[slot], policy);
            }
            // No copy may be in flight when the CTA exits: wait for the last
            // use of every slot that was filled.
            const uint64_t first = j > S ? j - S : 0;
            for (uint64_t k = first; k < j; ++k) {
                const uint32_t slot = static_cast<uint32_t>(k % S);
                const uint32_t use = static_cast<uint32_t>(k / S);
                mbar_wait_bounded(&full[slot], use & 1u, a.status, 2u);
            }
        }
        return;
    }

    // ---------------- consumers ----------------
    const uint32_t g = warp / C, c = warp % C;
    typename XRegs<TYPE>::T xr;
    bool valid;
    load_x<TYPE>(a, c, lane, xr, valid);

    float best_v = -INFINITY;
    uint32_t best_i = 0xFFFFFFFFu;

    for (uint64_t j = g;; j += G) {
        const uint64_t tile = blockIdx.x + j * gridDim.x;
        if (tile >= a.tiles) break;
        const uint32_t slot = static_cast<uint32_t>(j % S);
        const uint32_t use = static_cast<uint32_t>(j / S);
        if (!wait_phase(&full[slot], use & 1u, abort_flag, a.status, 3u)) break;
        const uint8_t* stage = smem + static_cast<size_t>(slot) * a.stage_bytes;
        const uint64_t row0 = tile * R;
        const uint64_t left = a.rows - row0;
        const uint32_t nrows = left < R ? static_cast<uint32_t>(left) : R;
        for (uint32_t r = 0; r < nrows; ++r) {
            float part = row_partial<TYPE>(stage + static_cast<size_t>(r) * a.row_bytes, xr, valid, c, lane, a.cols);
            part = warp_sum(part);
            if (C == 1) {
                if (lane == 0) {
                    a.y[row0 + r] = part;
                    const uint32_t idx = static_cast<uint32_t>(row0 + r);
                    if (amax_better(part, idx, best_v, best_i)) {
                        best_v = part;
                        best_i = idx;
                    }
                }
            } else if (lane == 0) {
                red[(static_cast<size_t>(slot) * R + r) * C + c] = part;
            }
        }
        __syncwarp();
        if (C == 1) {
            if (lane == 0) mbar_arrive(&empty[slot]);
            continue;
        }
        if (lane == 0) mbar_arrive(&redbar[slot]);
        if (c != 0) {
            if (lane == 0) mbar_arrive(&empty[slot]);
            continue;
        }
        // chunk-0 warp: fold the chunk sums of every row in fixed order
        if (!wait_phase(&redbar[slot], use & 1u, abort_flag, a.status, 4u)) break;
        if (lane < nrows) {
            const float* rp = red + (static_cast<size_t>(slot) * R + lane) * C;
            float v = 0.f;
            for (uint32_t cc = 0; cc < C; ++cc) v += rp[cc];
            a.y[row0 + lane] = v;
            const uint32_t idx = static_cast<uint32_t>(row0 + lane);
            if (amax_better(v, idx, best_v, best_i)) {
                best_v = v;
                best_i = idx;
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
    }

    if (!a.has_amax) return;
    // ---------------- fused argmax (F16 LM head) ----------------
    warp_argmax(best_v, best_i);
    if (lane == 0) {
        am_val[warp] = best_v;
        am_idx[warp] = best_i;
    }
    named_barrier_sync(1, consumers * 32u);
    if (threadIdx.x == 0) {
        float v = am_val[0];
        uint32_t i = am_idx[0];
        for (uint32_t k = 1; k < consumers; ++k)
            if (amax_better(am_val[k], am_idx[k], v, i)) {
                v = am_val[k];
                i = am_idx[k];
            }
        a.amax.cand_val[blockIdx.x] = v;
        a.amax.cand_idx[blockIdx.x] = i;
        __threadfence();
        const uint32_t done = atomicAdd(a.amax.counter, 1u);
        if (done == gridDim.x - 1u) {
            __threadfence();
            const volatile float* cv = a.amax.cand_val;
            const volatile uint32_t* ci = a.amax.cand_idx;
            float bv = cv[0];
            uint32_t bi = ci[0];
            for (uint32_t k = 1; k < gridDim.x; ++k)
                if (amax_better(cv[k], ci[k], bv, bi)) {
                    bv = cv[k];
                    bi = ci[k];
                }
            *a.amax.out_index = static_cast<int64_t>(bi);
            if (a.amax.out_value != nullptr) *a.amax.out_value = bv;
            *a.amax.counter = 0u;  // ready for the next launch
        }
    }
}

uint32_t ceil_div_u32(uint64_t a, uint64_t b) { return static_cast<uint32_t>((a + b - 1) / b); }

template <uint32_t TYPE, uint32_t MAX_THREADS>
cudaError_t launch_typed(const StreamPlan& plan, const StreamArgs& args, cudaStream_t stream) {
    static bool configured[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(gemv_stream_kernel<TYPE, MAX_THREADS>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
        if (e != cudaSuccess) return e;
        configured[dev] = true;
    }
    gemv_stream_kernel<TYPE, MAX_THREADS><<<plan.grid, plan.threads, plan.smem_bytes, stream>>>(args);
    return cudaGetLastError();
}

template <uint32_t TYPE>
cudaError_t launch_width(const StreamPlan& plan, const StreamArgs& args, cudaStream_t stream) {
    if (plan.threads <= kThreadsNormal) return launch_typed<TYPE, kThreadsNormal>(plan, args, stream);
    return launch_typed<TYPE, kThreadsWide>(plan, args, stream);
}

}  // namespace

uint64_t row_bytes_of(uint32_t type, uint64_t cols) {
    switch (type) {
        case kF16: return cols * 2u;
        case kQ4_0: return (cols % 32u) ? 0 : cols / 32u * 18u;
        case kQ8_0: return (cols % 32u) ? 0 : cols / 32u * 34u;
        default: return 0;
    }
}

StreamPlan plan_stream(uint32_t type, uint64_t rows, uint64_t cols, int num_sms, int max_smem_optin) {
    StreamPlan p;
    const uint64_t rb = row_bytes_of(type, cols);
    if (rb == 0 || rb % 16u || rows == 0 || cols > (1u << 20)) return p;
    uint32_t chunks;
    if (type == kF16) {
        if (cols % 8u) return p;
        chunks = ceil_div_u32(cols, 2048);
    } else {
        if ((cols / 32u) % 2u) return p;
        chunks = ceil_div_u32(cols / 64u, 32);
    }
    if (chunks == 0 || chunks > kMaxConsumerWarps) return p;
    // 15 consumer warps fit the 512-thread CTA; only 16-chunk rows take 16.
    uint32_t groups = chunks == kMaxConsumerWarps ? 1u : (kMaxConsumerWarps - 1u) / chunks;
    const uint32_t misc = 8u + 8u * kMaxConsumerWarps + 128u;
    const uint64_t budget = static_cast<uint64_t>(max_smem_optin) - misc;
    // Aim for at least two stages per group so each group always has its next
    // tile in flight.
    uint64_t r = budget / ((2ull * groups + 2ull) * rb);
    if (r < 1) r = 1;
    if (r > kMaxRowsPerTile) r = kMaxRowsPerTile;
    uint32_t rows_per_tile = static_cast<uint32_t>(r);
    if (rows_per_tile > rows) rows_per_tile = static_cast<uint32_t>(rows);
    const uint64_t stage_bytes = (rows_per_tile * rb + 127u) / 128u * 128u;
    const uint64_t per_stage = stage_bytes + 24u + 4ull * rows_per_tile * chunks;
    uint64_t stages = budget / per_stage;
    if (stages > kMaxStages) stages = kMaxStages;
    if (stages < 2) return p;
    if (stages < groups + 1u) groups = static_cast<uint32_t>(stages - 1u);
    if (groups == 0) return p;
    p.tiles = (rows + rows_per_tile - 1) / rows_per_tile;
    // Do not start more groups than a CTA has tiles.
    const uint64_t tiles_per_cta = (p.tiles + num_sms - 1) / num_sms;
    if (groups > tiles_per_cta) groups = static_cast<uint32_t>(tiles_per_cta);
    p.chunks = chunks;
    p.groups = groups;
    p.rows_per_tile = rows_per_tile;
    p.stages = static_cast<uint32_t>(stages);
    p.stage_bytes = static_cast<uint32_t>(stage_bytes);
    p.threads = (chunks * groups + 1u) * 32u;
    p.smem_bytes = static_cast<uint32_t>(stages * per_stage + misc);
    p.grid = static_cast<uint32_t>(p.tiles < static_cast<uint64_t>(num_sms) ? p.tiles : num_sms);
    p.ok = true;
    return p;
}

cudaError_t launch_stream(uint32_t type, const StreamPlan& plan, const void* w, const float* x, float* y,
                          uint64_t rows, uint64_t cols, DeviceStatus* status, const ArgmaxScratch* amax,
                          cudaStream_t stream) {
    StreamArgs a{};
    a.w = static_cast<const uint8_t*>(w);
    a.x = x;
    a.y = y;
    a.rows = rows;
    a.tiles = plan.tiles;
    a.cols = static_cast<uint32_t>(cols);
    a.row_bytes = static_cast<uint32_t>(row_bytes_of(type, cols));
    a.rows_per_tile = plan.rows_per_tile;
    a.chunks = plan.chunks;
    a.groups = plan.groups;
    a.stages = plan.stages;
    a.stage_bytes = plan.stage_bytes;
    a.status = status;
    a.has_amax = amax != nullptr ? 1u : 0u;
    if (amax != nullptr) a.amax = *amax;
    switch (type) {
        case kQ8_0: return launch_width<kQ8_0>(plan, a, stream);
        case kQ4_0: return launch_width<kQ4_0>(plan, a, stream);
        case kF16: return launch_width<kF16>(plan, a, stream);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace nedo_gpu
