// gemv_stream.cu -- batch-1 dequantize-and-dot matvec over raw GGUF rows.
//
// Replaces the CPU row loop of nedo::kernels::matvec (reference src/kernels.cpp:162-169)
// and its row kernels dot_f16 / dot_q8 / dot_q4 (src/kernels.cpp:109-160).
//
// Design:
//   * Rows are split evenly over every warp of the grid (a contiguous row range
//     per warp), so each SM streams the same number of bytes.
//   * Each warp is its own producer: lane 0 moves tiles of `rows_per_tile`
//     whole rows (one contiguous byte range) from HBM into the warp's private
//     ring of shared-memory slots with cp.async.bulk (mbarrier complete_tx,
//     L2 evict-first, no multicast), and the warp consumes its ring strictly in
//     order.  A slot is refilled by the warp that has just read it, so no
//     empty barrier exists and a wait never targets a slot whose previous use
//     is still pending.
//   * The first copies are issued before griddepcontrol.wait: with programmatic
//     dependent launch the weight stream of this kernel overlaps the tail of
//     the previous one; only x (written by earlier kernels) is read after it.
//   * x is staged once per CTA in shared memory in a lane-interleaved layout
//     (lane l reads consecutive 16-byte chunks), conflict free.  Each x load is
//     reused for the `rows_per_tile` rows of the tile.
//   * Lane l owns block pairs l, l+32, ... (Q8_0: 68 bytes, Q4_0: 36 bytes,
//     both 4-byte aligned whatever the block parity) or 8-element groups
//     (F16).  Quant bytes are picked with compile-time selectors.
//   * Integer quants become fp32 without I2F: PRMT/LOP3 place them in the
//     mantissa of a constant, a packed fp32x2 add removes it exactly (Q8_0) or
//     a per-block constant folds it out (Q4_0); products accumulate in fp32
//     with packed fp32x2 FMA.
//   * Lane sums are folded with warp shuffles in a fixed order, so results are
//     bit-reproducible run to run.
//   * Every wait is bounded (2 s); a warp that gives up records the failure in
//     DeviceStatus and waits (bounded) for its own copies before exiting.
#include <math.h>

#include "common.cuh"
#include "launch.h"

namespace nedo_gpu {
namespace {

constexpr uint32_t kMaxRowsPerTile = 8;
constexpr uint32_t kMaxSlots = 4;  // per warp

struct StreamArgs {
    const uint8_t* w;
    const float* x;
    float* y;
    uint64_t rows;
    uint32_t cols;
    uint32_t row_bytes;
    uint32_t rows_per_tile;
    uint32_t slots;       // per warp
    uint32_t slot_bytes;  // multiple of 128
    uint32_t warps;       // per CTA
    uint32_t x_bytes;     // staged x (plus Q4_0 block constants), multiple of 128
    uint32_t piece_bytes; // size of one bulk copy
    uint32_t has_amax;
    DeviceStatus* status;
    ArgmaxScratch amax;
};

__device__ __forceinline__ uint32_t align_up_dev(uint32_t v, uint32_t a) { return (v + a - 1u) / a * a; }
__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;"); }
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// ---------------------------------------------------------------------------
// x staging: 16-byte chunk k of unit u (u = 32c + l) lives at chunk index
// (c * CPU + k) * 32 + l, CPU = chunks per unit, so lane l of a warp reading
// chunk k of its unit touches consecutive 16-byte words (conflict free).
template <uint32_t TYPE>
struct Unit;
template <>
struct Unit<kQ8_0> {  // a pair of blocks: 64 elements
    static constexpr uint32_t kBytes = 68, kChunks = 16;
};
template <>
struct Unit<kQ4_0> {  // a pair of blocks: 64 elements
    static constexpr uint32_t kBytes = 36, kChunks = 16;
};
template <>
struct Unit<kF16> {  // 8 elements
    static constexpr uint32_t kBytes = 16, kChunks = 2;
};

// Units per 32-lane group are padded: the staged area holds
// ceil(units / 32) * 32 * CPU chunks, zero where the unit does not exist.
template <uint32_t TYPE>
__host__ __device__ __forceinline__ uint32_t x_stage_chunks(uint32_t cols) {
    constexpr uint32_t EPU = TYPE == kF16 ? 8u : 64u;  // elements per unit
    const uint32_t units = cols / EPU;
    return ((units + 31u) / 32u) * 32u * Unit<TYPE>::kChunks;
}

// Stage x (all threads of the CTA) from x_lin, a linear copy of x already in
// shared memory, iterating in staged order.  For Q4_0 the values are
// pre-scaled (x' = 256x for the low-nibble half of a block, 16x for the high
// half) and the per-block constants C_b = sum x' + 8 sum x are stored after
// the chunks.
template <uint32_t TYPE>
__device__ __forceinline__ void stage_x(const float4* __restrict__ x_lin, uint32_t cols, float4* xs, float* cb) {
    constexpr uint32_t CPU = Unit<TYPE>::kChunks;
    constexpr uint32_t EPU = TYPE == kF16 ? 8u : 64u;
    const uint32_t units = cols / EPU;
    const uint32_t n_slots = x_stage_chunks<TYPE>(cols);
    for (uint32_t i = threadIdx.x; i < n_slots; i += blockDim.x) {
        const uint32_t l = i & 31u, rest = i >> 5, k = rest % CPU, c = rest / CPU;
        const uint32_t u = 32u * c + l;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (u < units) {
            const uint32_t f = u * CPU + k;  // float4 index in x (< cols / 4)
            v = x_lin[f];
            if constexpr (TYPE == kQ4_0) {
                const float sc = (((4u * f) & 31u) < 16u) ? 256.0f : 16.0f;
                v = make_float4(v.x * sc, v.y * sc, v.z * sc, v.w * sc);
            }
        }
        xs[i] = v;
    }
    if constexpr (TYPE == kQ4_0) {
        for (uint32_t b = threadIdx.x; b < cols / 32u; b += blockDim.x) {
            float sx = 0.f, sp = 0.f;
#pragma unroll
            for (uint32_t j = 0; j < 8; ++j) {
                const float4 v = x_lin[8u * b + j];
                const float sc = j < 4 ? 256.0f : 16.0f;
                sx += (v.x + v.y) + (v.z + v.w);
                sp += ((v.x * sc + v.y * sc) + (v.z * sc + v.w * sc));
            }
            cb[b] = fmaf(8.0f, sx, sp);
        }
    }
}

// ---------------------------------------------------------------------------
// Q8_0 pair: 68 bytes = 17 aligned words; block 0 quants at pair bytes 2..33,
// block 1 at 36..67.  int8 q -> fp32: bits 0x4B0000uu (u = q ^ 0x80) is
// 2^23 + u; subtracting 2^23 + 128 gives q exactly.
__device__ __forceinline__ float q8_float(uint32_t word_xor, uint32_t byte) {
    return __uint_as_float(prmt(word_xor, 0x4B000000u, 0x7440u | byte));
}

__device__ __forceinline__ void dot_pair_q8(const uint32_t* __restrict__ wp, const float2* xv, float2& acc) {
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
        const int p0 = 2 + k, p1 = 3 + k;
        float2 q = fadd2(make_float2(q8_float(w[p0 >> 2], p0 & 3), q8_float(w[p1 >> 2], p1 & 3)), bias);
        if ((k & 2) == 0) a0 = ffma2(q, xv[k >> 1], a0); else a1 = ffma2(q, xv[k >> 1], a1);
        const int r0 = 36 + k, r1 = 37 + k;
        float2 s = fadd2(make_float2(q8_float(w[r0 >> 2], r0 & 3), q8_float(w[r1 >> 2], r1 & 3)), bias);
        if ((k & 2) == 0) b0 = ffma2(s, xv[16 + (k >> 1)], b0); else b1 = ffma2(s, xv[16 + (k >> 1)], b1);
    }
    acc = ffma2(fadd2(a0, a1), make_float2(d0, d0), acc);
    acc = ffma2(fadd2(b0, b1), make_float2(d1, d1), acc);
}

// ---------------------------------------------------------------------------
// Q4_0 pair: 36 bytes = 9 aligned words; block 0 quant byte j at pair byte
// 2+j, block 1 at 20+j.  A nibble n becomes f = 1 + n/256 (low nibble, mantissa
// bits 15-18) or 1 + n/16 (high nibble, bits 19-22) with one shift shared by
// the byte's two nibbles and one LOP3 each.  With x' as staged:
// sum (n-8) x = sum f x' - C_b.
template <int M>
__device__ __forceinline__ uint32_t q4_align(uint32_t w) {
    if constexpr (M == 0) return w << 15;
    else if constexpr (M == 1) return w << 7;
    else if constexpr (M == 2) return w >> 1;
    else return w >> 9;
}

// Mask and exponent constants live in registers (set once per call chain).
struct Q4Consts {
    uint32_t mask_lo, mask_hi, one;
};

template <int M>
__device__ __forceinline__ float2 q4_lo_hi(uint32_t w, const Q4Consts& k) {
    const uint32_t a = q4_align<M>(w);
    return make_float2(__uint_as_float(lop_and_or(a, k.mask_lo, k.one)),   // 1 + n_lo / 256
                       __uint_as_float(lop_and_or(a, k.mask_hi, k.one)));  // 1 + n_hi / 16
}

template <int BYTE0>
__device__ __forceinline__ void q4_two_bytes(const uint32_t* w, const float2* xs, float2& acc_lo, float2& acc_hi,
                                             int elem0, const Q4Consts& k) {
    constexpr int B1 = BYTE0 + 1;
    const float2 f0 = q4_lo_hi<BYTE0 & 3>(w[BYTE0 >> 2], k);
    const float2 f1 = q4_lo_hi<B1 & 3>(w[B1 >> 2], k);
    acc_lo = ffma2(make_float2(f0.x, f1.x), xs[elem0 >> 1], acc_lo);
    acc_hi = ffma2(make_float2(f0.y, f1.y), xs[(elem0 + 16) >> 1], acc_hi);
}

// sum f x' over one block as a float2 (two partial lanes)
template <int BASE_BYTE, int BASE_ELEM>
__device__ __forceinline__ float2 q4_block(const uint32_t* w, const float2* xs, const Q4Consts& k) {
    float2 lo0 = make_float2(0.f, 0.f), lo1 = lo0, hi0 = lo0, hi1 = lo0;
    q4_two_bytes<BASE_BYTE + 0>(w, xs, lo0, hi0, BASE_ELEM + 0, k);
    q4_two_bytes<BASE_BYTE + 2>(w, xs, lo1, hi1, BASE_ELEM + 2, k);
    q4_two_bytes<BASE_BYTE + 4>(w, xs, lo0, hi0, BASE_ELEM + 4, k);
    q4_two_bytes<BASE_BYTE + 6>(w, xs, lo1, hi1, BASE_ELEM + 6, k);
    q4_two_bytes<BASE_BYTE + 8>(w, xs, lo0, hi0, BASE_ELEM + 8, k);
    q4_two_bytes<BASE_BYTE + 10>(w, xs, lo1, hi1, BASE_ELEM + 10, k);
    q4_two_bytes<BASE_BYTE + 12>(w, xs, lo0, hi0, BASE_ELEM + 12, k);
    q4_two_bytes<BASE_BYTE + 14>(w, xs, lo1, hi1, BASE_ELEM + 14, k);
    return fadd2(fadd2(lo0, lo1), fadd2(hi0, hi1));
}

// acc (float2, two partial lanes) += d0 * (S0 - c0) + d1 * (S1 - c1)
__device__ __forceinline__ void dot_pair_q4(const uint32_t* __restrict__ wp, const float2* xs, float c0, float c1,
                                            const Q4Consts& k, float2& acc) {
    uint32_t w[9];
#pragma unroll
    for (int i = 0; i < 9; ++i) w[i] = wp[i];
    const float d0 = half_bits_to_float(w[0]);
    const float d1 = half_bits_to_float(w[4] >> 16);
    const float2 s0 = q4_block<2, 0>(w, xs, k);
    const float2 s1 = q4_block<20, 32>(w, xs, k);
    // (s.x + s.y - c) * d, split over the two lanes of acc: lane x takes s.x - c.
    acc = ffma2(make_float2(s0.x - c0, s0.y), make_float2(d0, d0), acc);
    acc = ffma2(make_float2(s1.x - c1, s1.y), make_float2(d1, d1), acc);
}

// ---------------------------------------------------------------------------
// F16 unit: 8 consecutive elements = one 16-byte chunk of the row.
__device__ __forceinline__ void dot_unit_f16(const uint8_t* __restrict__ p, const float2* xv, float2& acc) {
    const uint4 v = *reinterpret_cast<const uint4*>(p);
    const uint32_t h[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) acc = ffma2(__half22float2(*reinterpret_cast<const __half2*>(&h[k])), xv[k], acc);
}

// ---------------------------------------------------------------------------
// One tile: R rows x all columns from shared memory; lane l covers units
// l, l+32, ...  acc[r] gets the lane's partial sum of row r.  Each x load is
// used for all R rows.
template <uint32_t TYPE, uint32_t R>
__device__ __forceinline__ void tile_dot(const uint8_t* __restrict__ tile, uint32_t row_bytes, uint32_t units,
                                         const float4* __restrict__ xs, const float* __restrict__ cb, uint32_t lane,
                                         float2 (&acc)[R]) {
    constexpr uint32_t CPU = Unit<TYPE>::kChunks;
    const float4* xp = xs + lane;
    Q4Consts q4k;
    q4k.mask_lo = 0x00078000u;
    q4k.mask_hi = 0x00780000u;
    q4k.one = 0x3F800000u;
    for (uint32_t u = lane; u < units; u += 32u, xp += CPU * 32u) {
        float2 xv[CPU * 2];
#pragma unroll
        for (uint32_t k = 0; k < CPU; ++k) {
            const float4 t = xp[k * 32u];
            xv[2 * k] = make_float2(t.x, t.y);
            xv[2 * k + 1] = make_float2(t.z, t.w);
        }
        float c0 = 0.f, c1 = 0.f;
        if constexpr (TYPE == kQ4_0) {
            const float2 cc = *reinterpret_cast<const float2*>(cb + 2u * u);
            c0 = cc.x;
            c1 = cc.y;
        }
        const uint8_t* up = tile + u * Unit<TYPE>::kBytes;
#pragma unroll
        for (uint32_t r = 0; r < R; ++r) {
            const uint8_t* rp = up + r * row_bytes;
            if constexpr (TYPE == kQ8_0) dot_pair_q8(reinterpret_cast<const uint32_t*>(rp), xv, acc[r]);
            else if constexpr (TYPE == kQ4_0) dot_pair_q4(reinterpret_cast<const uint32_t*>(rp), xv, c0, c1, q4k, acc[r]);
            else dot_unit_f16(rp, xv, acc[r]);
        }
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

// Issue the bulk copies of one tile (rows [row0, row0+nrows)) into `dst`.
__device__ __forceinline__ void issue_tile(const StreamArgs& a, uint8_t* dst, uint64_t row0, uint32_t nrows,
                                           uint64_t* bar, uint64_t policy) {
    const uint32_t bytes = nrows * a.row_bytes;
    mbar_arrive_expect_tx(bar, bytes);
    const uint8_t* src = a.w + row0 * a.row_bytes;
    for (uint32_t o = 0; o < bytes; o += a.piece_bytes) {
        const uint32_t n = bytes - o < a.piece_bytes ? bytes - o : a.piece_bytes;
        bulk_copy_g2s(dst + o, src + o, n, bar, policy);
    }
}

template <uint32_t TYPE, uint32_t R>
__global__ void __launch_bounds__(512, 1) gemv_stream_kernel(const StreamArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    // [x staged | Q4_0 block constants][x linear][warp rings][barriers][argmax]
    float4* xs = reinterpret_cast<float4*>(smem);
    float* cb = reinterpret_cast<float*>(smem + static_cast<size_t>(x_stage_chunks<TYPE>(a.cols)) * 16u);
    float4* x_lin = reinterpret_cast<float4*>(smem + a.x_bytes);
    uint8_t* ring_base = smem + a.x_bytes + align_up_dev(a.cols * 4u, 128u);
    uint8_t* ring = ring_base + static_cast<size_t>(warp) * a.slots * a.slot_bytes;
    uint64_t* all_bars = reinterpret_cast<uint64_t*>(ring_base + static_cast<size_t>(a.warps) * a.slots * a.slot_bytes);
    uint64_t* bars = all_bars + warp * kMaxSlots;
    uint64_t* xbar = all_bars + a.warps * kMaxSlots;
    float* am_val = reinterpret_cast<float*>(xbar + 1);
    uint32_t* am_idx = reinterpret_cast<uint32_t*>(am_val + 32);
    uint32_t* am_last = am_idx + 32;  // set by thread 0: this CTA finished last

    // this warp's rows: an even split over all warps of the grid
    const uint64_t gw = static_cast<uint64_t>(blockIdx.x) * a.warps + warp;
    const uint64_t nw = static_cast<uint64_t>(gridDim.x) * a.warps;
    const uint64_t row_begin = a.rows * gw / nw, row_end = a.rows * (gw + 1) / nw;
    const uint64_t my_rows = row_end - row_begin;
    const uint32_t ntiles = static_cast<uint32_t>((my_rows + R - 1) / R);

    uint64_t policy = 0;
    if (threadIdx.x == 0) {
        mbar_init(xbar, 1);
        fence_barrier_init();
    }
    if (lane == 0) {
        for (uint32_t s = 0; s < a.slots; ++s) mbar_init(&bars[s], 1);
        fence_barrier_init();
        policy = l2_policy_evict_first();
        // Weights do not depend on earlier kernels: start streaming before the
        // grid dependency wait.
        const uint32_t first = ntiles < a.slots ? ntiles : a.slots;
        for (uint32_t t = 0; t < first; ++t) {
            const uint64_t r0 = row_begin + static_cast<uint64_t>(t) * R;
            const uint64_t left = row_end - r0;
            issue_tile(a, ring + static_cast<size_t>(t) * a.slot_bytes, r0, left < R ? static_cast<uint32_t>(left) : R,
                       &bars[t], policy);
        }
    }
    __syncwarp();     // warp 0 converged (lane 0 issued the first tiles)
    __syncthreads();  // barrier initialisation visible to every warp

    grid_dependency_wait();  // x and y may be produced / consumed by earlier kernels
    // x: one bulk copy into shared memory, then a reshuffle into the staged layout
    if (threadIdx.x == 0) {
        mbar_arrive_expect_tx(xbar, a.cols * 4u);
        bulk_copy_g2s(x_lin, a.x, a.cols * 4u, xbar, l2_policy_evict_last());
    }
    bool ok = mbar_wait_bounded(xbar, 0, a.status, 5u);
    if (ok) stage_x<TYPE>(x_lin, a.cols, xs, cb);
    __syncthreads();
    grid_launch_dependents();

    const uint32_t units = TYPE == kF16 ? a.cols / 8u : a.cols / 64u;
    float best_v = -INFINITY;
    uint32_t best_i = 0xFFFFFFFFu;
    uint32_t slot = 0, parity = 0, t = 0;
    for (; ok && t < ntiles; ++t) {
        if (!mbar_wait_bounded(&bars[slot], parity, a.status, 1u)) {
            ok = false;
            break;
        }
        const uint64_t r0 = row_begin + static_cast<uint64_t>(t) * R;
        const uint64_t left = row_end - r0;
        const uint32_t nrows = left < R ? static_cast<uint32_t>(left) : R;
        const uint8_t* tile = ring + static_cast<size_t>(slot) * a.slot_bytes;
        // A short last tile computes all R rows (the rows past `nrows` read
        // stale shared memory) and stores only the valid ones.
        float2 acc[R];
#pragma unroll
        for (uint32_t r = 0; r < R; ++r) acc[r] = make_float2(0.f, 0.f);
        tile_dot<TYPE, R>(tile, a.row_bytes, units, xs, cb, lane, acc);
#pragma unroll
        for (uint32_t r = 0; r < R; ++r) {
            const float v = warp_sum(acc[r].x + acc[r].y);
            if (r < nrows) {
                if (lane == r) {
                    a.y[r0 + r] = v;
                    if (amax_better(v, static_cast<uint32_t>(r0 + r), best_v, best_i)) {
                        best_v = v;
                        best_i = static_cast<uint32_t>(r0 + r);
                    }
                }
            }
        }
        // Refill the slot just read with the tile `slots` ahead.
        __syncwarp();
        if (lane == 0 && t + a.slots < ntiles) {
            fence_proxy_async_smem();
            const uint64_t n0 = row_begin + static_cast<uint64_t>(t + a.slots) * R;
            const uint64_t nleft = row_end - n0;
            issue_tile(a, ring + static_cast<size_t>(slot) * a.slot_bytes, n0,
                       nleft < R ? static_cast<uint32_t>(nleft) : R, &bars[slot], policy);
        }
        if (++slot == a.slots) {
            slot = 0;
            parity ^= 1u;
        }
    }
    if (!ok && lane == 0) {
        // Wind down: no copy of this warp may still be in flight at exit.
        for (uint32_t k = t; k < ntiles && k < t + a.slots; ++k) {
            const uint32_t s = k % a.slots;
            mbar_wait_bounded(&bars[s], (k / a.slots) & 1u, a.status, 2u);
        }
    }

    if (!a.has_amax) return;
    // ---------------- fused argmax (LM head) ----------------
    warp_argmax(best_v, best_i);
    if (lane == 0) {
        am_val[warp] = best_v;
        am_idx[warp] = best_i;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        float v = am_val[0];
        uint32_t i = am_idx[0];
        for (uint32_t k = 1; k < a.warps; ++k)
            if (amax_better(am_val[k], am_idx[k], v, i)) {
                v = am_val[k];
                i = am_idx[k];
            }
        a.amax.cand_val[blockIdx.x] = v;
        a.amax.cand_idx[blockIdx.x] = i;
        __threadfence();
        const uint32_t done = atomicAdd(a.amax.counter, 1u);
        *am_last = done == gridDim.x - 1u ? 1u : 0u;
    }
    __syncthreads();
    if (*am_last == 0u || warp != 0) return;
    // The last CTA to finish: warp 0 folds the per-CTA candidates, each lane a
    // strided subset (L2 loads, independent), then across the warp.
    __threadfence();
    float bv = -INFINITY;
    uint32_t bi = 0xFFFFFFFFu;
    for (uint32_t k = lane; k < gridDim.x; k += 32u) {
        const float v = __ldcg(a.amax.cand_val + k);
        const uint32_t i = __ldcg(a.amax.cand_idx + k);
        if (amax_better(v, i, bv, bi)) {
            bv = v;
            bi = i;
        }
    }
    warp_argmax(bv, bi);
    if (lane == 0) {
        // std::max_element keeps element 0 when it is NaN (no value compares
        // greater than NaN); otherwise NaNs never win, as in amax_better.
        const float y0 = __ldcg(a.y);
        if (y0 != y0) {
            bv = y0;
            bi = 0u;
        }
        *a.amax.out_index = static_cast<int64_t>(bi);
        if (a.amax.out_value != nullptr) *a.amax.out_value = bv;
        *a.amax.counter = 0u;  // ready for the next launch
    }
}

template <uint32_t TYPE, uint32_t R>
cudaError_t launch_typed(const StreamPlan& plan, const StreamArgs& args, cudaStream_t stream, bool pdl) {
    static bool configured[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(gemv_stream_kernel<TYPE, R>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             227 * 1024);
        if (e != cudaSuccess) return e;
        configured[dev] = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(plan.grid);
    cfg.blockDim = dim3(plan.threads);
    cfg.dynamicSmemBytes = plan.smem_bytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, gemv_stream_kernel<TYPE, R>, args);
}

template <uint32_t TYPE>
cudaError_t launch_rows(const StreamPlan& plan, const StreamArgs& args, cudaStream_t stream, bool pdl) {
    switch (plan.rows_per_tile) {
        case 1: return launch_typed<TYPE, 1>(plan, args, stream, pdl);
        case 2: return launch_typed<TYPE, 2>(plan, args, stream, pdl);
        case 3: return launch_typed<TYPE, 3>(plan, args, stream, pdl);
        case 4: return launch_typed<TYPE, 4>(plan, args, stream, pdl);
        case 5: return launch_typed<TYPE, 5>(plan, args, stream, pdl);
        case 6: return launch_typed<TYPE, 6>(plan, args, stream, pdl);
        case 7: return launch_typed<TYPE, 7>(plan, args, stream, pdl);
        case 8: return launch_typed<TYPE, 8>(plan, args, stream, pdl);
        default: return cudaErrorInvalidValue;
    }
}

uint64_t align_up(uint64_t v, uint64_t a) { return (v + a - 1) / a * a; }

}  // namespace

uint64_t row_bytes_of(uint32_t type, uint64_t cols) {
    switch (type) {
        case kF16: return cols * 2u;
        case kQ4_0: return (cols % 32u) ? 0 : cols / 32u * 18u;
        case kQ8_0: return (cols % 32u) ? 0 : cols / 32u * 34u;
        default: return 0;
    }
}

// Shared memory of the fused argmax: am_val[32], am_idx[32], am_last, padding.
constexpr uint64_t kArgmaxSmemBytes = 272;

StreamPlan plan_stream(uint32_t type, uint64_t rows, uint64_t cols, int num_sms, int max_smem_optin,
                       const StreamTuning* tune) {
    StreamPlan best;
    const uint64_t rb = row_bytes_of(type, cols);
    if (rb == 0 || rb % 16u || rows == 0 || rows > 0xFFFFFFFFull || num_sms <= 0) return best;
    if (type == kF16) {
        if (cols % 8u) return best;
    } else if ((cols / 32u) % 2u) {
        return best;
    }
    const uint64_t chunks = type == kF16 ? x_stage_chunks<kF16>(static_cast<uint32_t>(cols))
                            : type == kQ8_0 ? x_stage_chunks<kQ8_0>(static_cast<uint32_t>(cols))
                                            : x_stage_chunks<kQ4_0>(static_cast<uint32_t>(cols));
    const uint64_t x_bytes = align_up(chunks * 16u + (type == kQ4_0 ? cols / 32u * 4u : 0u), 128);
    const StreamTuning t = tune ? *tune : StreamTuning{};
    uint64_t budget = t.smem_budget ? t.smem_budget : static_cast<uint64_t>(max_smem_optin);
    if (budget > static_cast<uint64_t>(max_smem_optin)) budget = max_smem_optin;
    const uint64_t misc = align_up(cols * 4u, 128) + 8u * kMaxSlots * 16u + 8u + kArgmaxSmemBytes;
    if (x_bytes + misc >= budget) return best;

    auto make = [&](uint32_t warps, uint32_t r, uint32_t slots, uint32_t grid) {
        StreamPlan p;
        p.warps = warps;
        p.rows_per_tile = r;
        p.slots = slots;
        p.slot_bytes = static_cast<uint32_t>(align_up(r * rb, 128));
        p.x_bytes = static_cast<uint32_t>(x_bytes);
        p.piece_bytes = t.piece_bytes ? t.piece_bytes : 16384u;
        p.threads = warps * 32u;
        p.grid = grid;
        const uint64_t smem = x_bytes + align_up(cols * 4u, 128) + static_cast<uint64_t>(warps) * slots * p.slot_bytes +
                              8u * kMaxSlots * warps + 8u + kArgmaxSmemBytes;
        p.smem_bytes = static_cast<uint32_t>(smem);
        p.ok = smem <= budget;
        return p;
    };
    // F16 is HBM bound: what matters is the size of each bulk copy (>= 8 KB) and
    // enough of them in flight; 8 warps with 2 slots each measured best on
    // 128000x2048 and 32000x4096 heads.
    if (type == kF16 && !tune) {
        uint32_t grid = static_cast<uint32_t>(num_sms);
        if (static_cast<uint64_t>(grid) * 8u > rows) grid = static_cast<uint32_t>((rows + 7u) / 8u);
        const uint64_t rpw = (rows + static_cast<uint64_t>(grid) * 8u - 1) / (static_cast<uint64_t>(grid) * 8u);
        uint64_t r = (8192u + rb - 1) / rb;
        if (r > kMaxRowsPerTile) r = kMaxRowsPerTile;
        if (r > rpw) r = rpw;
        const StreamPlan p = make(8u, static_cast<uint32_t>(r), r >= rpw ? 1u : 2u, grid);
        if (p.ok) return p;
    }
    // Score: expected time ~ (rows actually computed per warp) with a penalty
    // for streaming tiles (x re-read per tile).  Lower is better.
    double best_score = 1e300;
    const uint32_t w_lo = t.warps ? t.warps : 4u, w_hi = t.warps ? t.warps : 16u;
    for (uint32_t warps = w_hi; warps >= w_lo && warps >= 1; --warps) {
        uint32_t grid = static_cast<uint32_t>(num_sms);
        if (static_cast<uint64_t>(grid) * warps > rows) grid = static_cast<uint32_t>((rows + warps - 1) / warps);
        const uint64_t nw = static_cast<uint64_t>(grid) * warps;
        const uint64_t rpw = (rows + nw - 1) / nw;  // rows of the busiest warp
        // single shot: the warp's whole row range in one tile
        if (rpw <= kMaxRowsPerTile && t.slots <= 1 && !t.tile_bytes) {
            StreamPlan p = make(warps, static_cast<uint32_t>(rpw), 1, grid);
            const double score = static_cast<double>(rpw) / warps * 16.0;
            if (p.ok && score < best_score) {
                best = p;
                best_score = score;
            }
        }
        // streaming tiles of ~tile_bytes, 2..kMaxSlots slots
        const uint64_t target = t.tile_bytes ? t.tile_bytes : 16384u;
        uint64_t r = target / rb;
        if (r < 1) r = 1;
        if (r > kMaxRowsPerTile) r = kMaxRowsPerTile;
        if (r > rpw) r = rpw;
        for (; r >= 1; --r) {
            if (t.slots == 1) break;  // single shot requested
            const uint32_t s_lo = t.slots ? t.slots : 2u, s_hi = t.slots ? t.slots : 3u;
            bool placed = false;
            for (uint32_t slots = s_hi; slots >= s_lo; --slots) {
                StreamPlan p = make(warps, static_cast<uint32_t>(r), slots, grid);
                if (!p.ok) continue;
                const uint64_t tiles = (rpw + r - 1) / r;
                // computed rows, plus the x re-read cost of every extra tile
                const double score = (static_cast<double>(tiles * r) + 0.35 * (tiles - 1)) / warps * 16.0 + 0.01 * (3 - slots);
                if (score < best_score) {
                    best = p;
                    best_score = score;
                }
                placed = true;
                break;
            }
            if (placed) break;
        }
        if (t.warps) break;
    }
    return best;
}

cudaError_t launch_stream(uint32_t type, const StreamPlan& plan, const void* w, const float* x, float* y,
                          uint64_t rows, uint64_t cols, DeviceStatus* status, const ArgmaxScratch* amax,
                          cudaStream_t stream, bool pdl) {
    StreamArgs a{};
    a.w = static_cast<const uint8_t*>(w);
    a.x = x;
    a.y = y;
    a.rows = rows;
    a.cols = static_cast<uint32_t>(cols);
    a.row_bytes = static_cast<uint32_t>(row_bytes_of(type, cols));
    a.rows_per_tile = plan.rows_per_tile;
    a.slots = plan.slots;
    a.slot_bytes = plan.slot_bytes;
    a.warps = plan.warps;
    a.x_bytes = plan.x_bytes;
    a.piece_bytes = plan.piece_bytes;
    a.status = status;
    a.has_amax = amax != nullptr ? 1u : 0u;
    if (amax != nullptr) a.amax = *amax;
    switch (type) {
        case kQ8_0: return launch_rows<kQ8_0>(plan, a, stream, pdl);
        case kQ4_0: return launch_rows<kQ4_0>(plan, a, stream, pdl);
        case kF16: return launch_rows<kF16>(plan, a, stream, pdl);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace nedo_gpu
