// gemv_imma.cu -- batch-1 Q8_0 / Q4_0 matvec on the int8 tensor pipe.
//
// Same contract as the reference row kernels dot_q8 / dot_q4
// (src/kernels.cpp:124-160): y[r] = sum_b d[r][b] * sum_i q[r][b][i] * x[32b+i],
// x consumed in fp32 precision, fp32 output.
//
// Arithmetic.  Each 32-element block of x gets a power-of-two exponent e_b
// (max |x_b| * 2^e_b in [2^26, 2^27)), x_b is rounded to the integer
// X = rint(x * 2^e_b) (28 significant bits relative to the block maximum) and X is
// split into four base-128 int8 limbs, X = L0*2^21 + L1*2^14 + L2*2^7 + L3
// (L0 signed in [-64, 63], L1..L3 in [0, 127]).
// The block dot of each limb with the int8 quants (Q8_0) or the 0..15 nibbles
// (Q4_0, minus 8 * sum L afterwards) is computed EXACTLY in int32 by
// mma.sync m16n8k32 (IMMA); only the per-block recombination
//   y += d * 2^-e_b * (L-dots combined)
// is floating point.
//
// Operand layout of one IMMA (k = 32 = 2 blocks x 16 positions):
//   A (16 x 32, row-major)  = weights: rows g, g+8 of the tile; k < 16 is the
//                             even block of a block pair, k >= 16 the odd one.
//                             Q8_0: the raw quant bytes.  Q4_0: the nibbles of
//                             the 16 quant bytes (low nibbles = positions 0..15,
//                             high = 16..31), one IMMA per nibble half.
//   B (32 x 8, col-major)   = x limbs, block-diagonal: column n = 4*block + limb.
//   D (16 x 8, s32)         = per row, per block, per limb integer dots.
// The x side of every IMMA (the B registers of each lane, the per-column
// scale 2^(7*(2-l)-e) and, for Q4_0, the "-8 * sum L" start value of the
// accumulators) is precomputed once per launch into a shared-memory table in
// fragment order, so a lane fetches its B operand of a block pair with one
// 8-byte load.
//
// Streaming.  A CTA owns a contiguous run of 16-row tiles.  A unit of work is
// one segment of seg_pairs block pairs of one tile: a single 2D tensor-map
// copy (cp.async.bulk.tensor, no multicast) of 16 rows x seg_pairs pairs into
// one slot of a shared-memory ring, with the box row padded to an odd multiple
// of 16 bytes so the eight fragment rows of an operand load sit in distinct
// banks.  Boxes overhanging the row end or the last row read zeros (no memory
// traffic).  Consumer warps are independent: warp w owns tiles w, w+W, ... of
// the CTA and runs every segment of such a tile, accumulating its rows in
// registers, then stores them.  Rows longer than the table holds are cut into
// column groups processed one after the other (the table is rebuilt between
// groups and y accumulates in group order; the same warp owns a tile in every
// group).
//
// CTA shape: one CTA per SM with up to 16 consumer warps and one producer
// warp (96 registers; 8 consumer warps within 128 registers when several
// token vectors share a launch) and a ring of up to 32 units in the whole
// shared memory.  With programmatic dependent launch a CTA starts streaming its
// weight as soon as the previous kernel's CTA on its SM exits, and reads x only
// after that kernel has completed.  Every wait is bounded; a CTA-wide abort
// flag stops every warp after the first timed-out wait.
//
// One token vector whose CTA share fits in shared memory (the 25 MB-class
// matrices and smaller) runs gemv_imma_slice_kernel instead (see there): no
// ring, wide copy units, and finer work items that share each x-side read
// among all of a CTA's tiles.
#include <math.h>
#include <stdlib.h>

#include "common.cuh"
#include "launch.h"

namespace nedo_gpu {
namespace {

constexpr uint32_t kMaxWarps = 16;               // consumer warps (+1 producer warp)
constexpr uint32_t kNarrowSmem = 113u * 1024u;   // (228 KB - 2 x 1 KB reserved) / 2, rounded down
constexpr uint32_t kMaxBoxBytes = 2048;          // 256 elements of 8 bytes
constexpr uint32_t kTileRows = 16;               // rows per tile: the M of one IMMA
constexpr uint32_t kMaxSlots = 32;

// Table entry of one block pair: 32 lanes x (w_lo, w_hi), then for each of the
// four t (a lane's D columns 2t, 2t+1) the column scale and the two start values.
constexpr uint32_t kPairTableBytes = 32u * 8u + 4u * 16u;

struct ImmaArgs {
    const float* x;
    float* y;
    uint64_t rows;
    uint32_t tiles;        // ceil(rows / 16)
    uint32_t pairs_total;  // cols / 64
    uint32_t group_pairs;  // block pairs per column group (a multiple of seg_pairs)
    uint32_t groups;
    uint32_t box_bytes;    // bytes per box row = its shared-memory pitch (an odd multiple of 16)
    uint32_t warps;        // consumer warps
    uint32_t team;         // warps sharing a tile (a power of two dividing warps)
    uint32_t slots;
    uint32_t unit_bytes;   // 16 * box_bytes
    uint32_t early_chunks; // slice: chunks copied before x is requested
    uint32_t token_groups; // multi-vector slice: groups of CTAs, each computing its own vectors
    uint64_t ldx;          // floats between token vectors of x
    uint64_t ldy;          // floats between token vectors of y
    DeviceStatus* status;
    // Fused all-gather (npeers > 0): each finished y row is also stored at
    // peer_y[k][peer_row_offset + row] on every peer (NVLink peer stores), and
    // every CTA adds 1 to each peer's counter peer_signal[k] once its rows are
    // visible system-wide.
    uint32_t npeers;
    uint64_t peer_row_offset;
    float* peer_y[kMaxPeers];
    uint32_t* peer_signal[kMaxPeers];
    XPrologue pro;  // slice kernel only
};

__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;"); }

// 2D tensor-map copy global -> this CTA's shared memory with an L2 cache hint,
// completing on `bar`.  No multicast.
__device__ __forceinline__ void tma_load_2d_hint(uint32_t dst, const CUtensorMap* map, int32_t c0, int32_t c1,
                                                 uint64_t* bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_addr(bar)), "l"(policy)
        : "memory");
}

// Bounded wait until the producer has started unit `want` in a slot (false on
// timeout, recorded in `st`, or when another warp has aborted).
__device__ __forceinline__ bool wait_issued(volatile uint32_t* issued, uint32_t want, volatile uint32_t* abort_flag,
                                            DeviceStatus* st, uint32_t site) {
    if (*issued == want) return true;
    const uint64_t t0 = global_timer_ns();
    const uint64_t limit = wait_limit_ns(st);
    while (*issued != want) {
        if (*abort_flag != 0u) return false;
        if (global_timer_ns() - t0 > limit) {
            if (atomicOr(&st->flags, kErrWaitTimeout) == 0u) st->where = site;
            return false;
        }
        __nanosleep(32);
    }
    return true;
}

template <uint32_t TYPE>
struct Pair;
template <>
struct Pair<kQ8_0> {
    static constexpr uint32_t kBytes = 68, kBlock = 34;
};
template <>
struct Pair<kQ4_0> {
    static constexpr uint32_t kBytes = 36, kBlock = 18;
};

// Q4_0: the start value of each lane's low-limb D column carries 1.5 * 2^23 as
// float bits (0x4B400000), so the combined integer 128 * d_hi + d_lo of a
// block (|value| < 2^22) is directly the bit pattern of 1.5 * 2^23 + value and
// one FADD turns it into the exact float (no integer-to-float conversion).
constexpr int kQ4Magic = 0x4B400000;
constexpr float kQ4MagicF = 12582912.0f;  // 1.5 * 2^23

// d = A * B + c (int8 inputs, exact int32 accumulation); A unsigned for Q4_0 nibbles.
template <bool A_UNSIGNED>
__device__ __forceinline__ void imma_c(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                       uint32_t b1, int c0, int c1, int c2, int c3) {
    if (A_UNSIGNED)
        asm volatile(
            "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%12,%13};"
            : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(c0), "r"(c1), "r"(c2), "r"(c3));
    else
        asm volatile(
            "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%12,%13};"
            : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(c0), "r"(c1), "r"(c2), "r"(c3));
}

// The float value of a combined block dot (for Q4_0 exact, through the offset
// carried in the start value; for Q8_0 the conversion's rounding).
template <uint32_t TYPE>
__device__ __forceinline__ float dot_value(int v) {
    if constexpr (TYPE == kQ4_0) return __int_as_float(v) - kQ4MagicF;
    else return static_cast<float>(v);
}

// d += A * B (int8 inputs, exact int32 accumulation); A unsigned for Q4_0 nibbles.
template <bool A_UNSIGNED>
__device__ __forceinline__ void imma(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                     uint32_t b1) {
    if (A_UNSIGNED)
        asm volatile(
            "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
            : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
    else
        asm volatile(
            "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
            : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// N 32-element blocks of x per thread group, 8 threads per block (4 positions
// each): the four limb words of this thread's positions, the block exponent and
// the limb sums, all written into the fragment-ordered pair table.  The N
// blocks are processed in lockstep so that their shuffles overlap.  e_b makes
// max |x_b| * 2^e_b fall in [2^26, 2^27).
// A block holding a NaN or an infinity gets all-zero limbs and a NaN column
// scale, so every row's result is NaN, as the reference's fp32 sums are for a
// NaN (and, but for the sign of the infinities, for an infinite) element.
template <bool SUMS, uint32_t N>
__device__ __forceinline__ void limb_blocks(const float4 (&vin)[N], const uint32_t (&b)[N], uint32_t q,
                                            const bool (&in)[N], uint8_t* table) {
    // |v| as bits: the order of finite magnitudes, NaN and infinity at 0x7F800000 and above
    uint32_t mb[N];
#pragma unroll
    for (uint32_t n = 0; n < N; ++n)
        mb[n] = max(max(__float_as_uint(vin[n].x) & 0x7FFFFFFFu, __float_as_uint(vin[n].y) & 0x7FFFFFFFu),
                    max(__float_as_uint(vin[n].z) & 0x7FFFFFFFu, __float_as_uint(vin[n].w) & 0x7FFFFFFFu));
#pragma unroll
    for (uint32_t k = 1; k < 8; k <<= 1)
#pragma unroll
        for (uint32_t n = 0; n < N; ++n) mb[n] = max(mb[n], __shfl_xor_sync(0xFFFFFFFFu, mb[n], k));
    uint32_t L[N][4];
    int sum[N][4];
    bool bad[N];
    int e[N];
#pragma unroll
    for (uint32_t n = 0; n < N; ++n) {
        bad[n] = mb[n] >= 0x7F800000u;
        const float4 v = bad[n] ? make_float4(0.f, 0.f, 0.f, 0.f) : vin[n];
        e[n] = 0;  // an all-zero block keeps e = 0 (all limbs 0)
        if (!bad[n] && mb[n] != 0u) {
            const int E = static_cast<int>(mb[n] >> 23) - 127;  // max |x_b| in [2^E, 2^(E+1))
            int en = 26 - E;                                     // in [-101, 153]
            if (en > 126) en = 126;
            e[n] = en;
        }
        const float sc = __uint_as_float(static_cast<uint32_t>(e[n] + 127) << 23);  // 2^e, exact
        // |X| <= 2^27 - 8 (a float below 2^27 scaled by a power of two is an integer
        // multiple of 8 there), so X = L0*2^21 + L1*2^14 + L2*2^7 + L3 with
        // L0 = X >> 21 in [-64, 63] and L1..L3 = the 7-bit floor remainders in [0, 127].
        // Limb l of element i is byte (3 - l) of X << (3 - l), masked to 7 bits for
        // l > 0; PRMT gathers that byte of the four elements into one word.
        const uint32_t X0 = static_cast<uint32_t>(__float2int_rn(v.x * sc));
        const uint32_t X1 = static_cast<uint32_t>(__float2int_rn(v.y * sc));
        const uint32_t X2 = static_cast<uint32_t>(__float2int_rn(v.z * sc));
        const uint32_t X3 = static_cast<uint32_t>(__float2int_rn(v.w * sc));
        // byte k of a and of b -> bytes 0, 1 (selector 0x33..: the upper two bytes are don't-care)
        auto gather = [](uint32_t a, uint32_t bb, uint32_t c, uint32_t d, uint32_t sel) {
            return prmt(prmt(a, bb, sel), prmt(c, d, sel), 0x5410u);
        };
        L[n][3] = gather(X0, X1, X2, X3, 0x3340u) & 0x7F7F7F7Fu;
        L[n][2] = gather(X0 << 1, X1 << 1, X2 << 1, X3 << 1, 0x3351u) & 0x7F7F7F7Fu;
        L[n][1] = gather(X0 << 2, X1 << 2, X2 << 2, X3 << 2, 0x3362u) & 0x7F7F7F7Fu;
        L[n][0] = gather(X0 << 3, X1 << 3, X2 << 3, X3 << 3, 0x3373u);
        sum[n][0] = sum[n][1] = sum[n][2] = sum[n][3] = 0;
    }
    if (SUMS) {
        // limb sums over the block (Q4_0 start values), two per word: low 16 bits a
        // non-negative sum (<= 32 * 127), high 16 bits the other
        int s32[N], s21[N];
#pragma unroll
        for (uint32_t n = 0; n < N; ++n) {
            s32[n] = __dp4a(static_cast<int>(L[n][3]), 0x01010101, 0) +
                     __dp4a(static_cast<int>(L[n][0]), 0x01010101, 0) * 65536;
            s21[n] = __dp4a(static_cast<int>(L[n][2]), 0x01010101, 0) +
                     __dp4a(static_cast<int>(L[n][1]), 0x01010101, 0) * 65536;
        }
#pragma unroll
        for (uint32_t k = 1; k < 8; k <<= 1)
#pragma unroll
            for (uint32_t n = 0; n < N; ++n) {
                s32[n] += __shfl_xor_sync(0xFFFFFFFFu, s32[n], k);
                s21[n] += __shfl_xor_sync(0xFFFFFFFFu, s21[n], k);
            }
#pragma unroll
        for (uint32_t n = 0; n < N; ++n) {
            sum[n][3] = s32[n] & 0xFFFF;
            sum[n][0] = (s32[n] - sum[n][3]) >> 16;
            sum[n][2] = s21[n] & 0xFFFF;
            sum[n][1] = (s21[n] - sum[n][2]) >> 16;
        }
    }
#pragma unroll
    for (uint32_t n = 0; n < N; ++n) {
        if (!in[n]) continue;
        // lane (g, t) of the pair's IMMAs takes limb g & 3 of block (g >= 4 ? odd : even),
        // positions 4t.. (w_lo) and 16+4t.. (w_hi): this thread's word is w_lo of
        // t = q (q < 4) or w_hi of t = q - 4
        const uint32_t odd = b[n] & 1u;
        uint8_t* pe = table + static_cast<size_t>(b[n] >> 1) * kPairTableBytes;
#pragma unroll
        for (uint32_t l = 0; l < 4; ++l) {
            const uint32_t lane = (4u * odd + l) * 4u + (q & 3u);
            reinterpret_cast<uint32_t*>(pe + lane * 8u)[q >> 2] = L[n][l];
        }
        if (q < 2) {
            // t = 2*odd + q: D columns 2t, 2t+1 = limbs la = 2q and la+1 of this block,
            // scale 2^(7*(2-la) - e) (in [2^-126, 2^115]: a normal float)
            const uint32_t la = 2u * q;
            int* te = reinterpret_cast<int*>(pe + 256u + (2u * odd + q) * 16u);
            te[0] = bad[n] ? static_cast<int>(0x7FC00000u)
                           : static_cast<int>(static_cast<uint32_t>(7 * (2 - static_cast<int>(la)) - e[n] + 127) << 23);
            te[1] = -8 * (q ? sum[n][2] : sum[n][0]);
            te[2] = -8 * (q ? sum[n][3] : sum[n][1]) + (SUMS ? kQ4Magic : 0);
        }
    }
}

template <bool SUMS>
__device__ __forceinline__ void limb_block(float4 v, uint32_t b, uint32_t q, bool in, uint8_t* table) {
    const float4 vv[1] = {v};
    const uint32_t bb[1] = {b};
    const bool ii[1] = {in};
    limb_blocks<SUMS, 1>(vv, bb, q, ii, table);
}

// All consumer threads: build the tables of blocks [0, nblocks) of `ntok`
// token vectors (x + k * ldx, table + k * tstride), 8 threads per block, all
// (token, block) pairs in one pass with every x load issued before any is used.
constexpr uint32_t kLimbPasses = 8;  // up to 8 * nthreads / 8 blocks staged in registers at once
template <bool SUMS>
__device__ __forceinline__ void build_pair_table(const float* __restrict__ x, uint64_t ldx, uint32_t ntok,
                                                 uint32_t nblocks, uint32_t tid, uint32_t nthreads, uint8_t* table,
                                                 size_t tstride) {
    const uint32_t per_pass = nthreads / 8u;
    const uint32_t q = tid & 7u;
    const uint32_t total = ntok * nblocks;
    for (uint32_t base = 0; base < total; base += per_pass * kLimbPasses) {
        float4 v[kLimbPasses];
#pragma unroll
        for (uint32_t k = 0; k < kLimbPasses; ++k) {
            const uint32_t f = base + k * per_pass + tid / 8u;
            const uint32_t tok = f / nblocks, b = f - tok * nblocks;
            v[k] = f < total ? __ldg(reinterpret_cast<const float4*>(x + tok * ldx + 32u * b + 4u * q))
                             : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (uint32_t k = 0; k < kLimbPasses; ++k) {
            const uint32_t f = base + k * per_pass + tid / 8u;
            const uint32_t tok = f / nblocks, b = f - tok * nblocks;
            // the 8 threads of a block share f, so they agree on `in` (the shuffles
            // inside span exactly those 8 lanes)
            if (base + k * per_pass < total) limb_block<SUMS>(v[k], b, q, f < total, table + tok * tstride);
        }
    }
}

// One segment of one tile for NT token vectors: `valid` block pairs starting at
// r0p / r1p (tile rows g and g+8 of the slot); token t's x side at
// pt + t * tstride (its pair table entries).  The weight fragments are loaded
// once and used for every token.  acc0[t] / acc1[t] collect rows g and g+8
// (this lane's D columns).
template <uint32_t TYPE, uint32_t SEG, bool GUARD, uint32_t NT>
__device__ __forceinline__ void segment_dot(const uint8_t* r0p, const uint8_t* r1p, const uint8_t* pt, size_t tstride,
                                            uint32_t valid, uint32_t lane, uint32_t even_mask, float (&acc0)[NT],
                                            float (&acc1)[NT]) {
    constexpr uint32_t pb = Pair<TYPE>::kBytes;
    const uint32_t t = lane & 3u;
    const uint32_t scale_blk = (t >> 1) * Pair<TYPE>::kBlock;  // this lane's D block within a pair
    // one token: every pair unrolled; several: two pairs at a time (the token loop
    // is unrolled, and its accumulators must stay in registers)
    constexpr uint32_t kUnroll = NT == 1 ? SEG : 2u;
#pragma unroll kUnroll
    for (uint32_t p = 0; p < SEG; ++p) {
        if (GUARD && p >= valid) break;
        const uint8_t* p0 = r0p + p * pb;
        const uint8_t* p1 = r1p + p * pb;
        // A fragments: Q8_0 two IMMAs (h = 0, 1), Q4_0 the low and high nibbles
        uint32_t A[2][4];
        if constexpr (TYPE == kQ8_0) {
#pragma unroll
            for (uint32_t h = 0; h < 2; ++h) {
                // even block: quant bytes 16h+4t.. at pair offset 2+16h+4t (2 mod 4)
                const uint32_t o = 16u * h + 4u * t;
                const uint32_t* e0 = reinterpret_cast<const uint32_t*>(p0 + o);
                const uint32_t* e1 = reinterpret_cast<const uint32_t*>(p1 + o);
                A[h][0] = __funnelshift_r(e0[0], e0[1], 16);
                A[h][1] = __funnelshift_r(e1[0], e1[1], 16);
                A[h][2] = *reinterpret_cast<const uint32_t*>(p0 + 36u + o);
                A[h][3] = *reinterpret_cast<const uint32_t*>(p1 + 36u + o);
            }
        } else {
            // even block quant bytes 4t.. at pair offset 2+4t; odd block at 20+4t
            const uint32_t* e0 = reinterpret_cast<const uint32_t*>(p0 + 4u * t);
            const uint32_t* e1 = reinterpret_cast<const uint32_t*>(p1 + 4u * t);
            const uint32_t w0 = __funnelshift_r(e0[0], e0[1], 16);
            const uint32_t w2 = *reinterpret_cast<const uint32_t*>(p0 + 20u + 4u * t);
            const uint32_t w1 = __funnelshift_r(e1[0], e1[1], 16);
            const uint32_t w3 = *reinterpret_cast<const uint32_t*>(p1 + 20u + 4u * t);
            const uint32_t m = 0x0F0F0F0Fu;
            A[0][0] = w0 & m;
            A[0][1] = w1 & m;
            A[0][2] = w2 & m;
            A[0][3] = w3 & m;
            A[1][0] = (w0 >> 4) & m;
            A[1][1] = (w1 >> 4) & m;
            A[1][2] = (w2 >> 4) & m;
            A[1][3] = (w3 >> 4) & m;
        }
        const float d0 = half_bits_to_float(*reinterpret_cast<const uint16_t*>(p0 + scale_blk));
        const float d1 = half_bits_to_float(*reinterpret_cast<const uint16_t*>(p1 + scale_blk));
#pragma unroll
        for (uint32_t k = 0; k < NT; ++k) {
            const uint8_t* ptk = pt + k * tstride + p * kPairTableBytes;
            const uint2 w = *reinterpret_cast<const uint2*>(ptk + lane * 8u);
            const int4 te = *reinterpret_cast<const int4*>(ptk + 256u + t * 16u);
            // B registers: column g of the block-diagonal B is in the even block (k < 16) for g < 4
            const uint32_t b0lo = w.x & even_mask, b1lo = w.x & ~even_mask;
            const uint32_t b0hi = w.y & even_mask, b1hi = w.y & ~even_mask;
            int d[4];
            if constexpr (TYPE == kQ8_0) {
                d[0] = d[1] = d[2] = d[3] = 0;
                imma<false>(d, A[0][0], A[0][1], A[0][2], A[0][3], b0lo, b1lo);
                imma<false>(d, A[1][0], A[1][1], A[1][2], A[1][3], b0hi, b1hi);
            } else {
                // accumulators start at -8 * sum L of their column (the nibble offset)
                imma_c<true>(d, A[0][0], A[0][1], A[0][2], A[0][3], b0lo, b1lo, te.y, te.z, te.y, te.z);
                imma<true>(d, A[1][0], A[1][1], A[1][2], A[1][3], b0hi, b1hi);
            }
            // d[0], d[1]: row g, limbs (2(t&1), 2(t&1)+1) of block (t>>1); d[2], d[3]: row g+8
            const float xs = __int_as_float(te.x);
            const int v0 = d[0] * 128 + d[1];
            const int v1 = d[2] * 128 + d[3];
            acc0[k] = fmaf(dot_value<TYPE>(v0), d0 * xs, acc0[k]);
            acc1[k] = fmaf(dot_value<TYPE>(v1), d1 * xs, acc1[k]);
        }
    }
}

// MULTI: the rows are cut into more than one column group.  SEG: block pairs
// per unit.  NT: token vectors per launch (x [NT][ldx], y [NT][ldy]).
template <uint32_t TYPE, uint32_t SEG, bool MULTI, uint32_t NT>
// Registers are charged per group of four warps: one token runs 16 consumer
// warps (17 warps, charged as 20) within 96 registers; several tokens run at
// most 8 (9 warps, charged as 12) within 128, room for the per-token accumulators.
__global__ void __maxnreg__(NT == 1 ? 96 : 128)
    gemv_imma_kernel(const __grid_constant__ CUtensorMap map, const ImmaArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t S = a.slots, W = a.warps;
    // [ring: S units][pair table x NT][full S][empty S][team 8][issued S][partial sums 2 x W x NT x 16][abort flag]
    uint8_t* table = smem + static_cast<size_t>(S) * a.unit_bytes;
    const size_t tstride = static_cast<size_t>(a.group_pairs) * kPairTableBytes;  // one token's table
    uint64_t* full = reinterpret_cast<uint64_t*>(table + NT * tstride);
    uint64_t* empty = full + S;
    // issued[s]: the unit whose copy into slot s was last started.  A warp skips
    // the units of other warps, so it may reach a slot two or more uses ahead of
    // its barrier's phase, which a parity wait cannot tell apart; it first waits
    // for its own unit to be issued into the slot (then the barrier's phase is
    // that unit's).
    uint64_t* teambar = empty + S;  // [8]: a team's partial sums are complete (K arrivals)
    volatile uint32_t* issued = reinterpret_cast<volatile uint32_t*>(teambar + 8);
    float* red = reinterpret_cast<float*>(const_cast<uint32_t*>(issued) + S);
    volatile uint32_t* abort_flag = reinterpret_cast<volatile uint32_t*>(red + 2u * W * NT * 16u);

    // this CTA's tiles: an even split of all 16-row tiles
    const uint32_t tile_begin = static_cast<uint32_t>(static_cast<uint64_t>(a.tiles) * blockIdx.x / gridDim.x);
    const uint32_t tile_end = static_cast<uint32_t>(static_cast<uint64_t>(a.tiles) * (blockIdx.x + 1) / gridDim.x);
    const uint32_t my_tiles = tile_end - tile_begin;
    const uint32_t ngroups = MULTI ? a.groups : 1u;

    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
            issued[s] = 0xFFFFFFFFu;
        }
        for (uint32_t i = 0; i < 8; ++i) mbar_init(&teambar[i], a.team);
        *abort_flag = 0u;
        fence_barrier_init();
    }
    __syncwarp();  // warp 0 converged before the CTA barrier
    __syncthreads();
    // The next kernel on the stream may be scheduled now: its CTAs only stream
    // their weights until this grid has completed.
    grid_launch_dependents();

    constexpr uint32_t pb = Pair<TYPE>::kBytes;
    const uint32_t teams = W / a.team;
    if (warp == W) {
        // ---------------- producer: one thread ----------------
        // The weights are not written by the previous kernel on the stream, so
        // they are streamed before its completion (griddepcontrol.wait is only
        // needed for x).  Units in order: group, block of `teams` tiles (one per
        // team), segment, tile -- so the ring always spans every warp's work.
        if (lane != 0) return;
        const uint64_t policy = l2_policy_evict_first();
        uint32_t slot = 0, use = 0, u = 0;
        bool ok = true;
        for (uint32_t gi = 0; gi < ngroups && ok; ++gi) {
            const uint32_t pair_g = gi * a.group_pairs;
            const uint32_t gp = a.pairs_total - pair_g < a.group_pairs ? a.pairs_total - pair_g : a.group_pairs;
            const uint32_t nseg = (gp + SEG - 1u) / SEG;
            for (uint32_t tb = 0; tb < my_tiles && ok; tb += teams)
            for (uint32_t s = 0; s < nseg && ok; ++s) {
                const uint32_t nb = my_tiles - tb < teams ? my_tiles - tb : teams;
                for (uint32_t jj = 0; jj < nb; ++jj, ++u) {
                    const int32_t row0 = static_cast<int32_t>((tile_begin + tb + jj) * kTileRows);
                    if (use > 0 && !mbar_wait_bounded(&empty[slot], (use - 1u) & 1u, a.status, 11u)) {
                        *abort_flag = 1u;
                        ok = false;
                        break;
                    }
                    // the previous use of the slot is consumed: full[slot] is in this unit's phase
                    issued[slot] = u;
                    mbar_arrive_expect_tx(&full[slot], a.unit_bytes);
                    // x in 8-byte elements: pair_g and SEG are multiples of 4, so the byte
                    // offset is a multiple of 16
                    const int32_t x0 = static_cast<int32_t>((pair_g + s * SEG) * pb / 8u);
                    tma_load_2d_hint(smem_addr(smem + static_cast<size_t>(slot) * a.unit_bytes), &map, x0, row0,
                                     &full[slot], policy);
                    if (++slot == S) {
                        slot = 0;
                        ++use;
                    }
                }
            }
        }
        // drain: every issued copy must land before the CTA may exit
        const uint32_t first = u > S ? u - S : 0;
        for (uint32_t k = first; k < u; ++k) mbar_wait_bounded(&full[k % S], (k / S) & 1u, a.status, 12u);
        return;
    }

    // ---------------- consumers ----------------
    // Teams of K warps: team i owns tiles i, i + W/K, ...; member k of a team
    // runs segments k, k + K, ... of each of them (K = 1: a warp owns whole tiles).
    constexpr bool kQ4 = TYPE == kQ4_0;
    const uint32_t K = a.team, team = warp / K, member = warp - team * K;
    const uint32_t g = lane >> 2;
    const uint32_t even_mask = g < 4 ? 0xFFFFFFFFu : 0u;
    // fragment rows g and g+8 = unit rows g and g+8
    const size_t off_a = static_cast<size_t>(g) * a.box_bytes;
    const size_t off_b = off_a + 8u * static_cast<size_t>(a.box_bytes);

    grid_dependency_wait();  // x may come from the previous kernel
    bool ok = true;
    uint32_t u = 0;      // first unit of the group, counted like the producer
    uint32_t round = 0;  // tiles this team has finished, over all groups (team barrier phase)
    for (uint32_t gi = 0; gi < ngroups; ++gi) {
        const uint32_t pair_g = gi * a.group_pairs;
        const uint32_t gp = a.pairs_total - pair_g < a.group_pairs ? a.pairs_total - pair_g : a.group_pairs;
        const uint32_t nseg = (gp + SEG - 1u) / SEG;
        if (gi > 0) named_barrier_sync(1, W * 32u);  // every warp is done with the last group's table
        build_pair_table<kQ4>(a.x + static_cast<size_t>(pair_g) * 64u, a.ldx, NT, 2u * gp, threadIdx.x, W * 32u, table,
                              tstride);
        named_barrier_sync(1, W * 32u);
        for (uint32_t tb = 0; tb < my_tiles; tb += teams) {
            const uint32_t j = tb + team;
            if (j >= my_tiles) break;  // the last block has fewer tiles than teams
            const uint32_t nb = my_tiles - tb < teams ? my_tiles - tb : teams;
            float acc0[NT], acc1[NT];
#pragma unroll
            for (uint32_t k = 0; k < NT; ++k) acc0[k] = acc1[k] = 0.f;
            for (uint32_t s = member; s < nseg; s += K) {
                const uint32_t uj = u + tb * nseg + s * nb + team;
                const uint32_t slot = uj % S, parity = (uj / S) & 1u;
                if (ok && *abort_flag != 0u) ok = false;
                if (ok && !(wait_issued(&issued[slot], uj, abort_flag, a.status, 15u) &&
                            mbar_wait_bounded(&full[slot], parity, a.status, 13u))) {
                    ok = false;
                    *abort_flag = 1u;
                }
                if (ok) {
                    const uint8_t* unit = smem + static_cast<size_t>(slot) * a.unit_bytes;
                    const uint32_t left = gp - s * SEG;
                    const uint8_t* pt = table + static_cast<size_t>(s) * SEG * kPairTableBytes;
                    if (left >= SEG)
                        segment_dot<TYPE, SEG, false, NT>(unit + off_a, unit + off_b, pt, tstride, SEG, lane, even_mask,
                                                          acc0, acc1);
                    else
                        segment_dot<TYPE, SEG, true, NT>(unit + off_a, unit + off_b, pt, tstride, left, lane, even_mask,
                                                         acc0, acc1);
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&empty[slot]);
                }
            }
            // per token: fold the four t-lanes (columns) of each row; row r of the tile is
            // acc0 (r < 8) or acc1 (r >= 8) of lane 4 (r mod 8), and lane r takes it
            const uint32_t r = lane & 15u;
            float v[NT];
#pragma unroll
            for (uint32_t k = 0; k < NT; ++k) {
                float c0 = acc0[k], c1 = acc1[k];
                c0 += __shfl_xor_sync(0xFFFFFFFFu, c0, 1);
                c0 += __shfl_xor_sync(0xFFFFFFFFu, c0, 2);
                c1 += __shfl_xor_sync(0xFFFFFFFFu, c1, 1);
                c1 += __shfl_xor_sync(0xFFFFFFFFu, c1, 2);
                const float v0 = __shfl_sync(0xFFFFFFFFu, c0, 4u * (r & 7u));
                const float v1 = __shfl_sync(0xFFFFFFFFu, c1, 4u * (r & 7u));
                v[k] = r < 8 ? v0 : v1;
            }
            if (K > 1) {
                // the team's partial sums meet in shared memory (two buffers by tile parity);
                // member 0 adds them up in member order
                float* rb = red + (static_cast<size_t>(2u * team + (round & 1u)) * K) * NT * 16u;
                if (lane < 16) {
#pragma unroll
                    for (uint32_t k = 0; k < NT; ++k) rb[(member * NT + k) * 16u + lane] = v[k];
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&teambar[team]);
                // every member waits (no member can arrive for the next round before this
                // round is complete, so the parity is unambiguous); member 0 adds up
                if (!mbar_wait_bounded(&teambar[team], round & 1u, a.status, 16u)) {
                    ok = false;
                    *abort_flag = 1u;
                }
                if (member == 0) {
#pragma unroll
                    for (uint32_t k = 0; k < NT; ++k) {
                        float sum = rb[k * 16u + r];
                        for (uint32_t mm = 1; mm < K; ++mm) sum += rb[(mm * NT + k) * 16u + r];
                        v[k] = sum;
                    }
                }
            }
            if (ok && member == 0 && lane < 16) {
                const uint64_t row = static_cast<uint64_t>(tile_begin + j) * kTileRows + lane;
                if (row < a.rows) {
#pragma unroll
                    for (uint32_t k = 0; k < NT; ++k) {
                        float* yr = a.y + k * a.ldy + row;
                        float val = v[k];
                        if (MULTI && gi > 0) val += *yr;  // groups add up in group order
                        *yr = val;
                        if (NT == 1 && a.npeers != 0u && gi + 1u == ngroups)
                            for (uint32_t q = 0; q < a.npeers; ++q) a.peer_y[q][a.peer_row_offset + row] = val;
                    }
                }
            }
            ++round;
        }
        u += my_tiles * nseg;
    }
    if (a.npeers != 0u) {
        // every warp's peer stores are visible system-wide before the CTA is
        // published on each peer with a release add
        __threadfence_system();
        named_barrier_sync(1, W * 32u);
        if (warp == 0 && lane == 0 && *abort_flag == 0u)
            for (uint32_t k = 0; k < a.npeers; ++k)
                asm volatile("red.release.sys.global.add.u32 [%0], 1;" ::"l"(a.peer_signal[k]) : "memory");
    }
}

// ---------------------------------------------------------------------------
// Resident-slice variant (one token vector, whole rows in one column group).
// A CTA's whole share of the weight fits in its shared memory, so every copy
// unit has its own slot and barrier and nothing is ever waited on for reuse.
//
// Streaming.  Copy units are wide (16 rows x UP block pairs, about 1.1 KB per
// row): the tensor-map engine's cost grows with the number of box rows, and
// units this wide stream a 25 MB matrix at the HBM rate where 0.5 KB rows do
// not.  The first copies (about as much as lands while the CTA waits for the
// previous kernel) are issued at CTA start, before griddepcontrol.wait; the
// rest only after every consumer warp has issued its loads of x, so that x
// (needed first) is not queued behind this SM's whole weight stream.  Copies
// go out chunk-major (chunk 0 of every tile first), the order the compute
// consumes them.  The next kernel on the stream is released
// (griddepcontrol.launch_dependents) once this CTA is past its dependency
// wait, so at most one kernel's CTAs wait behind a running one.
//
// Compute.  A work item is one sub-segment of kSubPairs block pairs of up to R
// consecutive tiles: the x side of each pair (B registers, column scales,
// start values) is read from the table once and applied to every tile, which
// cuts the shared-memory traffic per tile-pair by about a third.  Items are
// dealt round-robin to the consumer warps in landing order.  Every item folds
// its per-tile row sums into its own slot [tile][sub-segment]; after all warps
// are done each tile's rows are added over its sub-segments in order, so the
// result depends only on the shape, never on timing.
constexpr uint32_t kSubPairs = 4;
constexpr uint64_t kEarlyBytes = 160u * 1024u;  // weight bytes a CTA copies before requesting x

// The A fragments and the two block scales of one block pair of one 16-row
// tile (rows g, g+8 at p0 / p1).
template <uint32_t TYPE>
__device__ __forceinline__ void load_pair_a(const uint8_t* p0, const uint8_t* p1, uint32_t t, uint32_t (&A)[2][4],
                                            float& d0, float& d1) {
    const uint32_t scale_blk = (t >> 1) * Pair<TYPE>::kBlock;
    if constexpr (TYPE == kQ8_0) {
#pragma unroll
        for (uint32_t h = 0; h < 2; ++h) {
            const uint32_t o = 16u * h + 4u * t;
            const uint32_t* e0 = reinterpret_cast<const uint32_t*>(p0 + o);
            const uint32_t* e1 = reinterpret_cast<const uint32_t*>(p1 + o);
            A[h][0] = __funnelshift_r(e0[0], e0[1], 16);
            A[h][1] = __funnelshift_r(e1[0], e1[1], 16);
            A[h][2] = *reinterpret_cast<const uint32_t*>(p0 + 36u + o);
            A[h][3] = *reinterpret_cast<const uint32_t*>(p1 + 36u + o);
        }
    } else {
        const uint32_t* e0 = reinterpret_cast<const uint32_t*>(p0 + 4u * t);
        const uint32_t* e1 = reinterpret_cast<const uint32_t*>(p1 + 4u * t);
        const uint32_t w0 = __funnelshift_r(e0[0], e0[1], 16);
        const uint32_t w2 = *reinterpret_cast<const uint32_t*>(p0 + 20u + 4u * t);
        const uint32_t w1 = __funnelshift_r(e1[0], e1[1], 16);
        const uint32_t w3 = *reinterpret_cast<const uint32_t*>(p1 + 20u + 4u * t);
        const uint32_t m = 0x0F0F0F0Fu;
        A[0][0] = w0 & m;
        A[0][1] = w1 & m;
        A[0][2] = w2 & m;
        A[0][3] = w3 & m;
        A[1][0] = (w0 >> 4) & m;
        A[1][1] = (w1 >> 4) & m;
        A[1][2] = (w2 >> 4) & m;
        A[1][3] = (w3 >> 4) & m;
    }
    d0 = half_bits_to_float(*reinterpret_cast<const uint16_t*>(p0 + scale_blk));
    d1 = half_bits_to_float(*reinterpret_cast<const uint16_t*>(p1 + scale_blk));
}

// The two IMMAs of one block pair (A in registers) against one token's x side
// and the per-block recombination into the rows' sums.
template <uint32_t TYPE>
__device__ __forceinline__ void pair_mma(const uint32_t (&A)[2][4], float d0, float d1, uint32_t b0lo, uint32_t b1lo,
                                         uint32_t b0hi, uint32_t b1hi, const int4& te, float& acc0, float& acc1) {
    int d[4];
    if constexpr (TYPE == kQ8_0) {
        imma_c<false>(d, A[0][0], A[0][1], A[0][2], A[0][3], b0lo, b1lo, 0, 0, 0, 0);
        imma<false>(d, A[1][0], A[1][1], A[1][2], A[1][3], b0hi, b1hi);
    } else {
        imma_c<true>(d, A[0][0], A[0][1], A[0][2], A[0][3], b0lo, b1lo, te.y, te.z, te.y, te.z);
        imma<true>(d, A[1][0], A[1][1], A[1][2], A[1][3], b0hi, b1hi);
    }
    const float xs = __int_as_float(te.x);
    const int v0 = d[0] * 128 + d[1];
    const int v1 = d[2] * 128 + d[3];
    acc0 = fmaf(dot_value<TYPE>(v0), d0 * xs, acc0);
    acc1 = fmaf(dot_value<TYPE>(v1), d1 * xs, acc1);
}

// One block pair of one 16-row tile (rows g, g+8 at p0 / p1) against the x side
// already in registers: the two IMMAs and the per-block recombination.
template <uint32_t TYPE>
__device__ __forceinline__ void pair_tile_dot(const uint8_t* p0, const uint8_t* p1, uint32_t t, uint32_t b0lo,
                                              uint32_t b1lo, uint32_t b0hi, uint32_t b1hi, const int4& te, float& acc0,
                                              float& acc1) {
    uint32_t A[2][4];
    float d0, d1;
    load_pair_a<TYPE>(p0, p1, t, A, d0, d1);
    pair_mma<TYPE>(A, d0, d1, b0lo, b1lo, b0hi, b1hi, te, acc0, acc1);
}

// One work item: `valid` (<= kSubPairs) block pairs of nt <= R tiles whose rows
// g / g+8 sit at r0 / r1 + r * tstep (independent work for the schedulers).
template <uint32_t TYPE, uint32_t R>
__device__ __forceinline__ void item_dot(const uint8_t* r0, const uint8_t* r1, size_t tstep, uint32_t nt,
                                         const uint8_t* pt, uint32_t valid, uint32_t lane, uint32_t even_mask,
                                         float (&acc0)[R], float (&acc1)[R]) {
    constexpr uint32_t pb = Pair<TYPE>::kBytes;
    const uint32_t t = lane & 3u;
#pragma unroll
    for (uint32_t p = 0; p < kSubPairs; ++p) {
        if (p >= valid) break;
        const uint8_t* ptk = pt + p * kPairTableBytes;
        const uint2 w = *reinterpret_cast<const uint2*>(ptk + lane * 8u);
        const int4 te = *reinterpret_cast<const int4*>(ptk + 256u + t * 16u);
        const uint32_t b0lo = w.x & even_mask, b1lo = w.x & ~even_mask;
        const uint32_t b0hi = w.y & even_mask, b1hi = w.y & ~even_mask;
#pragma unroll
        for (uint32_t r = 0; r < R; ++r) {
            if (r < nt)
                pair_tile_dot<TYPE>(r0 + r * tstep + p * pb, r1 + r * tstep + p * pb, t, b0lo, b1lo, b0hi, b1hi, te,
                                    acc0[r], acc1[r]);
        }
    }
}

// The producer's L2 prefetch of the KV-cache rows the next attention step reads
// (XPrologue kcache): cached positions [start, pos) of the window, ring slots
// (start + j) % window, this CTA's share of them in at most two contiguous runs.
// The attention kernel's own copies of these rows, issued before its dependency
// wait, then hit L2.
__device__ __forceinline__ void prefetch_kv_rows(const XPrologue& pro) {
    const uint64_t pos = __ldcg(reinterpret_cast<const unsigned long long*>(&pro.io->pos));
    const uint64_t start = pos + 1 > pro.window ? pos + 1 - pro.window : 0;
    const uint64_t n = pos - start;  // cached rows (the current one comes from this kernel's output)
    const uint64_t j0 = n * blockIdx.x / gridDim.x, j1 = n * (blockIdx.x + 1) / gridDim.x;
    uint64_t j = j0;
    while (j < j1) {
        const uint64_t slot = (start + j) % pro.window;
        const uint64_t run = j1 - j < pro.window - slot ? j1 - j : pro.window - slot;
        const uint64_t off = slot * pro.row_bytes;
        const uint32_t bytes = static_cast<uint32_t>(run * pro.row_bytes);
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(reinterpret_cast<const uint8_t*>(pro.kcache) + off),
                     "r"(bytes)
                     : "memory");
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(reinterpret_cast<const uint8_t*>(pro.vcache) + off),
                     "r"(bytes)
                     : "memory");
        j += run;
    }
}

template <uint32_t TYPE, uint32_t UP, uint32_t R>
__global__ void __maxnreg__(96) gemv_imma_slice_kernel(const __grid_constant__ CUtensorMap map, const ImmaArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr uint32_t pb = Pair<TYPE>::kBytes;
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t W = a.warps;
    const uint32_t tile_begin = static_cast<uint32_t>(static_cast<uint64_t>(a.tiles) * blockIdx.x / gridDim.x);
    const uint32_t tile_end = static_cast<uint32_t>(static_cast<uint64_t>(a.tiles) * (blockIdx.x + 1) / gridDim.x);
    const uint32_t my_tiles = tile_end - tile_begin;
    const uint32_t nchunk = (a.pairs_total + UP - 1u) / UP;
    const uint32_t nunits = my_tiles * nchunk;
    const uint32_t nsub = (a.pairs_total + kSubPairs - 1u) / kSubPairs;  // sub-segments per tile
    const uint32_t tiles_cap = a.slots / nchunk;
    // [units: slots x unit_bytes, unit (t, c) at t * nchunk + c][pair table]
    // [partial sums: tiles_cap x nsub x 16][full: slots][x requested][abort flag]
    uint8_t* table = smem + static_cast<size_t>(a.slots) * a.unit_bytes;
    float* part = reinterpret_cast<float*>(table + static_cast<size_t>(a.group_pairs) * kPairTableBytes);
    // (at least 2 * W floats: the prologue's partial sums of squares use them first)
    const size_t part_floats = static_cast<size_t>(tiles_cap) * nsub * 16u > 2u * W ? static_cast<size_t>(tiles_cap) * nsub * 16u
                                                                                    : 2u * W;
    uint64_t* full = reinterpret_cast<uint64_t*>(part + part_floats);
    uint64_t* xbar = full + a.slots;
    volatile uint32_t* abort_flag = reinterpret_cast<volatile uint32_t*>(xbar + 1);

    if (threadIdx.x == 0) {
        for (uint32_t u = 0; u < nunits; ++u) mbar_init(&full[u], 1);
        mbar_init(xbar, W);
        *abort_flag = 0u;
        fence_barrier_init();
    }
    __syncwarp();
    __syncthreads();

    if (warp == W) {
        // producer (one thread)
        if (lane != 0) return;
        const uint64_t policy = l2_policy_evict_first();
        uint32_t issued = 0;
        bool ok = true;
        for (uint32_t c = 0; c < nchunk && ok; ++c) {
            // the first early_chunks chunks stream during griddepcontrol.wait; the rest
            // once every consumer warp has issued its x loads
            if (c == a.early_chunks) {
                ok = mbar_wait_bounded(xbar, 0u, a.status, 24u);
                // every consumer warp is past griddepcontrol.wait: the next kernel may be
                // scheduled now (not earlier, so that at most one kernel waits behind this one)
                grid_launch_dependents();
            }
            if (!ok) break;
            for (uint32_t t = 0; t < my_tiles; ++t, ++issued) {
                const uint32_t u = t * nchunk + c;
                mbar_arrive_expect_tx(&full[u], a.unit_bytes);
                // x in 8-byte elements: UP pairs are a multiple of 32 bytes
                tma_load_2d_hint(smem_addr(smem + static_cast<size_t>(u) * a.unit_bytes), &map,
                                 static_cast<int32_t>(c * UP * pb / 8u),
                                 static_cast<int32_t>((tile_begin + t) * kTileRows), &full[u], policy);
            }
        }
        if (a.early_chunks >= nchunk) {
            ok = mbar_wait_bounded(xbar, 0u, a.status, 24u) && ok;
            grid_launch_dependents();
        }
        if (!ok) *abort_flag = 1u;
        if (a.pro.kcache != nullptr) prefetch_kv_rows(a.pro);
        // every issued copy lands before the CTA may exit
        for (uint32_t c = 0, k = 0; c < nchunk; ++c)
            for (uint32_t t = 0; t < my_tiles && k < issued; ++t, ++k)
                mbar_wait_bounded(&full[t * nchunk + c], 0u, a.status, 22u);
        return;
    }

    constexpr bool kQ4 = TYPE == kQ4_0;
    const uint32_t g = lane >> 2;
    const uint32_t even_mask = g < 4 ? 0xFFFFFFFFu : 0u;
    const size_t off_a = static_cast<size_t>(g) * a.box_bytes;
    const size_t off_b = off_a + 8u * static_cast<size_t>(a.box_bytes);

    grid_dependency_wait();  // x may come from the previous kernel
    grid_launch_dependents();
    {
        // the x limb table: every x load issued, the producer released, then the limbs
        const uint32_t tid = threadIdx.x, per_pass = W * 32u / 8u, q = tid & 7u;
        const uint32_t blocks = 2u * a.pairs_total;  // at most per_pass * kLimbPasses (planned)
        const XPrologue& pro = a.pro;
        float4 v[kLimbPasses], v2[kLimbPasses];
#pragma unroll
        for (uint32_t k = 0; k < kLimbPasses; ++k) {
            const uint32_t f = k * per_pass + tid / 8u;
            const size_t e = 32u * f + 4u * q;
            v[k] = f < blocks ? __ldg(reinterpret_cast<const float4*>(a.x + e)) : make_float4(0.f, 0.f, 0.f, 0.f);
            // the second operand of the prologue: delta (norm) or up (silu)
            const float* second = pro.mode == kPrologueNorm ? pro.delta : pro.mode == kPrologueSilu ? pro.up : nullptr;
            v2[k] = (f < blocks && second) ? __ldg(reinterpret_cast<const float4*>(second + e))
                                            : make_float4(0.f, 0.f, 0.f, 0.f);
            // the norm weight is read after the sum of squares: bring its line into L1
            // now, so that read does not queue behind this SM's weight copies
            if (pro.mode == kPrologueNorm && f < blocks && q == 0) {
                const void* wl = pro.wtype == 0 ? static_cast<const void*>(static_cast<const float*>(pro.w) + 32u * f)
                                                : static_cast<const void*>(static_cast<const uint16_t*>(pro.w) + 32u * f);
                asm volatile("prefetch.global.L1 [%0];" ::"l"(wl));
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(xbar);
        if (pro.mode == kPrologueNorm) {
            // x + delta, its sum of squares in double (each CTA the same, in a fixed order)
            double ss = 0.0;
#pragma unroll
            for (uint32_t k = 0; k < kLimbPasses; ++k) {
                const uint32_t f = k * per_pass + tid / 8u;
                if (f >= blocks) continue;
                float4& x4 = v[k];
                x4.x += v2[k].x;
                x4.y += v2[k].y;
                x4.z += v2[k].z;
                x4.w += v2[k].w;
                if (pro.x_out && blockIdx.x == 0)
                    *reinterpret_cast<float4*>(pro.x_out + 32u * f + 4u * q) = x4;
                ss += static_cast<double>(x4.x) * x4.x;
                ss += static_cast<double>(x4.y) * x4.y;
                ss += static_cast<double>(x4.z) * x4.z;
                ss += static_cast<double>(x4.w) * x4.w;
            }
            for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, o);
            double* red = reinterpret_cast<double*>(part);  // free until the items write their sums
            if (lane == 0) red[warp] = ss;
            named_barrier_sync(1, W * 32u);
            double tot = 0.0;
            for (uint32_t i = 0; i < W; ++i) tot += red[i];
            const uint32_t n = 64u * a.pairs_total;
            const float inv = 1.0f / sqrtf(static_cast<float>(tot / n) + pro.eps);
#pragma unroll
            for (uint32_t k = 0; k < kLimbPasses; ++k) {
                const uint32_t f = k * per_pass + tid / 8u;
                if (f >= blocks) continue;
                const size_t e = 32u * f + 4u * q;
                float4 w4;
                if (pro.wtype == 0) {
                    w4 = __ldg(reinterpret_cast<const float4*>(static_cast<const float*>(pro.w) + e));
                } else {
                    const uint2 hb = __ldg(reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(pro.w) + e));
                    w4 = make_float4(half_bits_to_float(hb.x & 0xFFFFu), half_bits_to_float(hb.x >> 16),
                                     half_bits_to_float(hb.y & 0xFFFFu), half_bits_to_float(hb.y >> 16));
                }
                v[k].x = v[k].x * inv * w4.x;
                v[k].y = v[k].y * inv * w4.y;
                v[k].z = v[k].z * inv * w4.z;
                v[k].w = v[k].w * inv * w4.w;
            }
            named_barrier_sync(1, W * 32u);  // every warp has read the partial sums
        } else if (pro.mode == kPrologueSilu) {
            bool mask_root = false, mask_suffix = false;
            if (pro.route) {
                const uint32_t tok = pro.io->token;
                mask_root = pro.route[2u * tok] < 0.5f;
                mask_suffix = pro.route[2u * tok + 1u] < 0.5f;
            }
            const uint32_t r0 = pro.m_shared, r1 = r0 + pro.m_root, r2 = r1 + pro.m_suffix;
#pragma unroll
            for (uint32_t k = 0; k < kLimbPasses; ++k) {
                const uint32_t f = k * per_pass + tid / 8u;
                if (f >= blocks) continue;
                const uint32_t e = 32u * f + 4u * q;
                float* g = reinterpret_cast<float*>(&v[k]);
                const float* u = reinterpret_cast<const float*>(&v2[k]);
#pragma unroll
                for (uint32_t c = 0; c < 4; ++c) {
                    float o = (g[c] / (1.0f + expf(-g[c]))) * u[c];
                    const uint32_t i = e + c;
                    if (pro.route && ((mask_root && i >= r0 && i < r1) || (mask_suffix && i >= r1 && i < r2))) o = 0.f;
                    g[c] = o;
                }
            }
        }
#pragma unroll
        for (uint32_t k = 0; k < kLimbPasses; k += 2) {
            // the 8 threads of a block share f (the shuffles inside span exactly them)
            if (k * per_pass >= blocks) break;
            const uint32_t f0 = k * per_pass + tid / 8u, f1 = f0 + per_pass;
            const float4 vv[2] = {v[k], v[k + 1]};
            const uint32_t bb[2] = {f0, f1};
            const bool ii[2] = {f0 < blocks, f1 < blocks};
            limb_blocks<kQ4, 2>(vv, bb, q, ii, table);
        }
    }
    named_barrier_sync(1, W * 32u);

    const uint32_t ngroups = (my_tiles + R - 1u) / R;
    const uint32_t items = nsub * ngroups;
    const size_t tstep = static_cast<size_t>(nchunk) * a.unit_bytes;  // unit (t + 1, c) - unit (t, c)
    bool ok = true;
    for (uint32_t i = warp; i < items; i += W) {
        const uint32_t s = i / ngroups, grp = i - s * ngroups;
        const uint32_t t0 = grp * R, nt = my_tiles - t0 < R ? my_tiles - t0 : R;
        const uint32_t p0 = s * kSubPairs, c = p0 / UP;
        if (ok && *abort_flag != 0u) ok = false;
        for (uint32_t r = 0; r < nt && ok; ++r)
            if (!mbar_wait_bounded(&full[(t0 + r) * nchunk + c], 0u, a.status, 23u)) {
                ok = false;
                *abort_flag = 1u;
            }
        if (!ok) continue;
        const uint8_t* unit = smem + static_cast<size_t>(t0 * nchunk + c) * a.unit_bytes +
                              static_cast<size_t>(p0 - c * UP) * pb;
        const uint8_t* pt = table + static_cast<size_t>(p0) * kPairTableBytes;
        float acc0[R], acc1[R];
#pragma unroll
        for (uint32_t r = 0; r < R; ++r) acc0[r] = acc1[r] = 0.f;
        const uint32_t left = a.pairs_total - p0;
        item_dot<TYPE, R>(unit + off_a, unit + off_b, tstep, nt, pt, left < kSubPairs ? left : kSubPairs, lane,
                          even_mask, acc0, acc1);
        // fold the four t-lanes of each row: row r of a tile is acc0 (r < 8) or acc1
        // (r >= 8) of lane 4 (r mod 8); lane r stores it in the item's slot
#pragma unroll
        for (uint32_t r = 0; r < R; ++r) {
            float c0 = acc0[r], c1 = acc1[r];
            c0 += __shfl_xor_sync(0xFFFFFFFFu, c0, 1);
            c0 += __shfl_xor_sync(0xFFFFFFFFu, c0, 2);
            c1 += __shfl_xor_sync(0xFFFFFFFFu, c1, 1);
            c1 += __shfl_xor_sync(0xFFFFFFFFu, c1, 2);
            const uint32_t rr = lane & 15u;
            const float v0 = __shfl_sync(0xFFFFFFFFu, c0, 4u * (rr & 7u));
            const float v1 = __shfl_sync(0xFFFFFFFFu, c1, 4u * (rr & 7u));
            if (r < nt && lane < 16)
                part[(static_cast<size_t>(t0 + r) * nsub + s) * 16u + lane] = rr < 8 ? v0 : v1;
        }
    }
    named_barrier_sync(1, W * 32u);
    const bool aborted = *abort_flag != 0u;
    if (!aborted) {
        for (uint32_t t = warp; t < my_tiles; t += W) {
            if (lane < 16) {
                float sum = 0.f;
                for (uint32_t s = 0; s < nsub; ++s) sum += part[(static_cast<size_t>(t) * nsub + s) * 16u + lane];
                const uint64_t row = static_cast<uint64_t>(tile_begin + t) * kTileRows + lane;
                if (row < a.rows) {
                    a.y[row] = sum;
                    for (uint32_t q = 0; q < a.npeers; ++q) a.peer_y[q][a.peer_row_offset + row] = sum;
                }
            }
        }
    }
    if (a.npeers != 0u) {
        // every warp's peer stores are visible system-wide before the CTA is
        // published on each peer with a release add
        __threadfence_system();
        named_barrier_sync(1, W * 32u);
        if (warp == 0 && lane == 0 && !aborted)
            for (uint32_t k = 0; k < a.npeers; ++k)
                asm volatile("red.release.sys.global.add.u32 [%0], 1;" ::"l"(a.peer_signal[k]) : "memory");
    }
}

// ---------------------------------------------------------------------------
// Multi-vector resident slice (2 to 32 token vectors per launch, whole rows in
// one column group).  The grid is G token groups of C CTAs: group k computes
// the vectors [k * NT, k * NT + NT) over every tile, its C CTAs splitting the
// tiles evenly.  A CTA keeps its tiles resident as the one-vector slice does
// and builds the x tables of its own NT vectors only, so the table work per
// CTA shrinks as G grows; each weight tile is read from HBM by one group and
// from L2 by the others.
//
// Compute.  The CTA's tiles are taken R at a time (the sums of R tiles x NT
// vectors stay in registers); for each group of R tiles, warp w takes
// sub-segments w, w + W, ... (kMultiSub block pairs each) for all NT vectors:
// per block pair and tile the A fragments are loaded once and applied to
// every vector's B fragments.  Each warp's row sums of the group go to its
// own slots [warp][tile][vector][16]; once every warp is done, each
// (tile, vector) row is added over the warps in warp order, so the result
// depends only on the shape.
constexpr uint32_t kMultiSub = 2;
constexpr uint64_t kMultiCtaWeightBytes = 110u * 1024u;

// Bytes of the multi-vector kernel's tables (NT vectors) and row-sum slots
// (`warps` x `tiles` x NT x 16 floats).  With at most R tiles per CTA (one
// register group) the sums are written after the last table read and share
// the tables' memory.
__host__ __device__ constexpr uint64_t multi_table_bytes(uint64_t nt, uint64_t pairs) { return nt * pairs * kPairTableBytes; }
__host__ __device__ constexpr uint64_t multi_sums_bytes(uint64_t nt, uint64_t warps, uint64_t tiles) {
    return warps * tiles * nt * 16u * 4u;
}
__host__ __device__ constexpr uint64_t multi_region_bytes(uint64_t nt, uint64_t pairs, uint64_t warps, uint64_t tiles,
                                                          uint64_t r) {
    return tiles <= r ? (multi_table_bytes(nt, pairs) > multi_sums_bytes(nt, warps, tiles)
                             ? multi_table_bytes(nt, pairs)
                             : multi_sums_bytes(nt, warps, tiles))
                      : multi_table_bytes(nt, pairs) + multi_sums_bytes(nt, warps, tiles);
}

// One sub-segment (`valid` <= kMultiSub block pairs) of nt <= R tiles (rows g /
// g+8 at r0 / r1 + r * tstep) for NT vectors (vector k's table at pt + k * tstride).
template <uint32_t TYPE, uint32_t R, uint32_t NT>
__device__ __forceinline__ void multi_dot(const uint8_t* r0, const uint8_t* r1, size_t tstep, uint32_t nt,
                                          const uint8_t* pt, size_t tstride, uint32_t valid, uint32_t lane,
                                          uint32_t even_mask, float (&acc0)[R][NT], float (&acc1)[R][NT]) {
    constexpr uint32_t pb = Pair<TYPE>::kBytes;
    const uint32_t t = lane & 3u;
#pragma unroll
    for (uint32_t p = 0; p < kMultiSub; ++p) {
        if (p >= valid) break;
#pragma unroll
        for (uint32_t r = 0; r < R; ++r) {
            if (r >= nt) break;
            uint32_t A[2][4];
            float d0, d1;
            load_pair_a<TYPE>(r0 + r * tstep + p * pb, r1 + r * tstep + p * pb, t, A, d0, d1);
#pragma unroll
            for (uint32_t k = 0; k < NT; ++k) {
                const uint8_t* ptk = pt + k * tstride + p * kPairTableBytes;
                const uint2 w = *reinterpret_cast<const uint2*>(ptk + lane * 8u);
                const int4 te = *reinterpret_cast<const int4*>(ptk + 256u + t * 16u);
                pair_mma<TYPE>(A, d0, d1, w.x & even_mask, w.x & ~even_mask, w.y & even_mask, w.y & ~even_mask, te,
                               acc0[r][k], acc1[r][k]);
            }
        }
    }
}

// Registers: NT = 8 runs 12 consumer warps (13 warps, charged as 16) within 128,
// fewer vectors 16 consumer warps (charged as 20) within 96.  GROUPS: a CTA may
// hold more than R tiles (else one register group, its sums on the tables).
template <uint32_t TYPE, uint32_t UP, uint32_t R, uint32_t NT, bool GROUPS>
__global__ void __maxnreg__(NT >= 8 ? 128 : 96) gemv_imma_multi_kernel(const __grid_constant__ CUtensorMap map,
                                                                      const ImmaArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr uint32_t pb = Pair<TYPE>::kBytes;
    constexpr bool kQ4 = TYPE == kQ4_0;
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t W = a.warps;
    const uint32_t C = gridDim.x / a.token_groups;  // CTAs per token group
    const uint32_t grp = blockIdx.x / C, cta = blockIdx.x - grp * C;
    const uint32_t tile_begin = static_cast<uint32_t>(static_cast<uint64_t>(a.tiles) * cta / C);
    const uint32_t tile_end = static_cast<uint32_t>(static_cast<uint64_t>(a.tiles) * (cta + 1) / C);
    const uint32_t my_tiles = tile_end - tile_begin;  // at least 1, at most slots / nchunk (planned)
    const uint32_t nchunk = (a.pairs_total + UP - 1u) / UP;
    const uint32_t nunits = my_tiles * nchunk;
    const uint32_t tiles_cap = a.slots / nchunk;
    const size_t tstride = static_cast<size_t>(a.pairs_total) * kPairTableBytes;  // one vector's table
    // [units: slots x unit_bytes, unit (t, c) at t * nchunk + c][tables: NT x tstride]
    // [row sums: W x tiles_cap x NT x 16 (on the tables when tiles_cap <= R)]
    // [full: slots][x requested][abort flag]
    constexpr bool one_group = !GROUPS;
    uint8_t* table = smem + static_cast<size_t>(a.slots) * a.unit_bytes;
    float* part = reinterpret_cast<float*>(one_group ? table : table + multi_table_bytes(NT, a.pairs_total));
    uint64_t* full = reinterpret_cast<uint64_t*>(table + multi_region_bytes(NT, a.pairs_total, W, tiles_cap, R));
    uint64_t* xbar = full + a.slots;
    volatile uint32_t* abort_flag = reinterpret_cast<volatile uint32_t*>(xbar + 1);
    const float* x = a.x + static_cast<size_t>(grp) * NT * a.ldx;
    float* y = a.y + static_cast<size_t>(grp) * NT * a.ldy;

    if (threadIdx.x == 0) {
        for (uint32_t u = 0; u < nunits; ++u) mbar_init(&full[u], 1);
        mbar_init(xbar, W);
        *abort_flag = 0u;
        fence_barrier_init();
    }
    __syncwarp();
    __syncthreads();

    if (warp == W) {
        // producer (one thread), as in the one-vector slice; a tile that other
        // token groups also read keeps the normal L2 priority
        if (lane != 0) return;
        const uint64_t policy = a.token_groups > 1 ? l2_policy_evict_normal() : l2_policy_evict_first();
        uint32_t issued = 0;
        bool ok = true;
        for (uint32_t c = 0; c < nchunk && ok; ++c) {
            if (c == a.early_chunks) {
                ok = mbar_wait_bounded(xbar, 0u, a.status, 24u);
                grid_launch_dependents();
            }
            if (!ok) break;
            for (uint32_t t = 0; t < my_tiles; ++t, ++issued) {
                const uint32_t u = t * nchunk + c;
                mbar_arrive_expect_tx(&full[u], a.unit_bytes);
                tma_load_2d_hint(smem_addr(smem + static_cast<size_t>(u) * a.unit_bytes), &map,
                                 static_cast<int32_t>(c * UP * pb / 8u),
                                 static_cast<int32_t>((tile_begin + t) * kTileRows), &full[u], policy);
            }
        }
        if (a.early_chunks >= nchunk) {
            ok = mbar_wait_bounded(xbar, 0u, a.status, 24u) && ok;
            grid_launch_dependents();
        }
        if (!ok) *abort_flag = 1u;
        for (uint32_t c = 0, k = 0; c < nchunk; ++c)
            for (uint32_t t = 0; t < my_tiles && k < issued; ++t, ++k)
                mbar_wait_bounded(&full[t * nchunk + c], 0u, a.status, 22u);
        return;
    }

    const uint32_t g = lane >> 2;
    const uint32_t even_mask = g < 4 ? 0xFFFFFFFFu : 0u;
    const size_t off_a = static_cast<size_t>(g) * a.box_bytes;
    const size_t off_b = off_a + 8u * static_cast<size_t>(a.box_bytes);

    grid_dependency_wait();  // x may come from the previous kernel
    grid_launch_dependents();
    {
        // the NT vectors' tables as one table of NT * 2 * pairs blocks (vector k's
        // blocks from k * 2 * pairs): every x load issued, the producer released,
        // then the limbs
        const uint32_t tid = threadIdx.x, per_pass = W * 32u / 8u, q = tid & 7u;
        const uint32_t blocks = 2u * a.pairs_total, total = NT * blocks;  // at most per_pass * kLimbPasses (planned)
        float4 v[kLimbPasses];
#pragma unroll
        for (uint32_t k = 0; k < kLimbPasses; ++k) {
            const uint32_t f = k * per_pass + tid / 8u;
            const uint32_t tok = f / blocks, b = f - tok * blocks;
            v[k] = f < total ? __ldg(reinterpret_cast<const float4*>(x + tok * a.ldx + 32u * b + 4u * q))
                             : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(xbar);
#pragma unroll
        for (uint32_t k = 0; k < kLimbPasses; k += 2) {
            // the 8 threads of a block share f (the shuffles inside span exactly them)
            if (k * per_pass >= total) break;
            const uint32_t f0 = k * per_pass + tid / 8u, f1 = f0 + per_pass;
            const float4 vv[2] = {v[k], v[k + 1]};
            const uint32_t bb[2] = {f0, f1};
            const bool ii[2] = {f0 < total, f1 < total};
            limb_blocks<kQ4, 2>(vv, bb, q, ii, table);
        }
    }
    named_barrier_sync(1, W * 32u);

    const uint32_t nsub = (a.pairs_total + kMultiSub - 1u) / kMultiSub;
    const size_t tstep = static_cast<size_t>(nchunk) * a.unit_bytes;  // unit (t + 1, c) - unit (t, c)
    bool ok = true;
    const uint32_t ngroups = GROUPS ? (my_tiles + R - 1u) / R : 1u;
    for (uint32_t gi = 0; gi < ngroups; ++gi) {
        const uint32_t t0 = gi * R;
        const uint32_t nt = my_tiles - t0 < R ? my_tiles - t0 : R;
        float acc0[R][NT], acc1[R][NT];
#pragma unroll
        for (uint32_t r = 0; r < R; ++r)
#pragma unroll
            for (uint32_t k = 0; k < NT; ++k) acc0[r][k] = acc1[r][k] = 0.f;
        for (uint32_t s = warp; s < nsub; s += W) {
            const uint32_t p0 = s * kMultiSub, c = p0 / UP;  // kMultiSub divides UP: one chunk
            if (ok && *abort_flag != 0u) ok = false;
            for (uint32_t r = 0; r < nt && ok; ++r)
                if (!mbar_wait_bounded(&full[(t0 + r) * nchunk + c], 0u, a.status, 25u)) {
                    ok = false;
                    *abort_flag = 1u;
                }
            if (!ok) continue;
            const uint8_t* unit = smem + static_cast<size_t>(t0 * nchunk + c) * a.unit_bytes +
                                  static_cast<size_t>(p0 - c * UP) * pb;
            const uint32_t left = a.pairs_total - p0;
            multi_dot<TYPE, R, NT>(unit + off_a, unit + off_b, tstep, nt,
                                   table + static_cast<size_t>(p0) * kPairTableBytes, tstride,
                                   left < kMultiSub ? left : kMultiSub, lane, even_mask, acc0, acc1);
        }
        // this warp's row sums of the group: row r of a tile is acc0 (r < 8) or acc1
        // (r >= 8) of lane 4 (r mod 8) after folding the t-lanes
        if constexpr (one_group) named_barrier_sync(1, W * 32u);  // every warp is done with the tables
#pragma unroll
        for (uint32_t r = 0; r < R; ++r)
#pragma unroll
            for (uint32_t k = 0; k < NT; ++k) {
                float c0 = acc0[r][k], c1 = acc1[r][k];
                c0 += __shfl_xor_sync(0xFFFFFFFFu, c0, 1);
                c0 += __shfl_xor_sync(0xFFFFFFFFu, c0, 2);
                c1 += __shfl_xor_sync(0xFFFFFFFFu, c1, 1);
                c1 += __shfl_xor_sync(0xFFFFFFFFu, c1, 2);
                const uint32_t rr = lane & 15u;
                const float v0 = __shfl_sync(0xFFFFFFFFu, c0, 4u * (rr & 7u));
                const float v1 = __shfl_sync(0xFFFFFFFFu, c1, 4u * (rr & 7u));
                if (lane < 16 && r < nt)
                    part[((static_cast<size_t>(warp) * tiles_cap + t0 + r) * NT + k) * 16u + lane] = rr < 8 ? v0 : v1;
            }
    }
    named_barrier_sync(1, W * 32u);
    if (*abort_flag == 0u) {
        const uint32_t nw = nsub < W ? nsub : W;  // the warps that had sub-segments
        const uint32_t outs = my_tiles * NT * 16u;
        for (uint32_t i = threadIdx.x; i < outs; i += W * 32u) {
            const uint32_t r = i / (NT * 16u), k = (i / 16u) % NT, row16 = i & 15u;
            float sum = 0.f;
            for (uint32_t w = 0; w < nw; ++w) sum += part[((static_cast<size_t>(w) * tiles_cap + r) * NT + k) * 16u + row16];
            const uint64_t row = static_cast<uint64_t>(tile_begin + r) * kTileRows + row16;
            if (row < a.rows) y[k * a.ldy + row] = sum;
        }
    }
}

template <uint32_t TYPE, uint32_t UP, uint32_t R, uint32_t NT, bool GROUPS>
cudaError_t launch_multi_t(const ImmaPlan& plan, const CUtensorMap& map, const ImmaArgs& args, cudaStream_t stream,
                           bool pdl) {
    static bool configured[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(gemv_imma_multi_kernel<TYPE, UP, R, NT, GROUPS>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
        if (e != cudaSuccess) return e;
        configured[dev] = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(plan.grid);
    cfg.blockDim = dim3((plan.warps + 1) * 32);
    cfg.dynamicSmemBytes = plan.smem_bytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, gemv_imma_multi_kernel<TYPE, UP, R, NT, GROUPS>, map, args);
}

// Vectors per CTA: 2 (up to 8 tiles), 4 (up to 4) or 8 (up to 2): 32 row sums per lane.
template <uint32_t TYPE>
cudaError_t launch_multi_p(const ImmaPlan& plan, const CUtensorMap& map, const ImmaArgs& args, cudaStream_t stream,
                           bool pdl) {
    constexpr uint32_t UP = TYPE == kQ4_0 ? 32u : 16u;
    if (plan.seg_pairs != UP) return cudaErrorInvalidValue;
    // more tiles per CTA than one register group of 16 / NT
    const bool groups = plan.slots / ((plan.group_pairs + UP - 1u) / UP) > 16u / plan.tokens;
    switch (plan.tokens) {
        case 2: return groups ? launch_multi_t<TYPE, UP, 8, 2, true>(plan, map, args, stream, pdl)
                              : launch_multi_t<TYPE, UP, 8, 2, false>(plan, map, args, stream, pdl);
        case 4: return groups ? launch_multi_t<TYPE, UP, 4, 4, true>(plan, map, args, stream, pdl)
                              : launch_multi_t<TYPE, UP, 4, 4, false>(plan, map, args, stream, pdl);
        case 8: return groups ? launch_multi_t<TYPE, UP, 2, 8, true>(plan, map, args, stream, pdl)
                              : launch_multi_t<TYPE, UP, 2, 8, false>(plan, map, args, stream, pdl);
        default: return cudaErrorInvalidValue;
    }
}

template <uint32_t TYPE, uint32_t UP, uint32_t R>
cudaError_t launch_slice_t(const ImmaPlan& plan, const CUtensorMap& map, const ImmaArgs& args, cudaStream_t stream,
                           bool pdl) {
    static bool configured[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(gemv_imma_slice_kernel<TYPE, UP, R>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
        if (e != cudaSuccess) return e;
        configured[dev] = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(plan.grid);
    cfg.blockDim = dim3((plan.warps + 1) * 32);
    cfg.dynamicSmemBytes = plan.smem_bytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, gemv_imma_slice_kernel<TYPE, UP, R>, map, args);
}

template <uint32_t TYPE>
cudaError_t launch_slice_p(const ImmaPlan& plan, const CUtensorMap& map, const ImmaArgs& args, cudaStream_t stream,
                           bool pdl) {
    // tiles sharing one x-side read: all of a CTA's tiles up to 5, else 2
    const bool wide = plan.tile_group > 2;
    switch (plan.seg_pairs) {
        case 8: return wide ? launch_slice_t<TYPE, 8, 5>(plan, map, args, stream, pdl)
                            : launch_slice_t<TYPE, 8, 2>(plan, map, args, stream, pdl);
        case 16: return wide ? launch_slice_t<TYPE, 16, 5>(plan, map, args, stream, pdl)
                             : launch_slice_t<TYPE, 16, 2>(plan, map, args, stream, pdl);
        case 32: return wide ? launch_slice_t<TYPE, 32, 5>(plan, map, args, stream, pdl)
                             : launch_slice_t<TYPE, 32, 2>(plan, map, args, stream, pdl);
        default: return cudaErrorInvalidValue;
    }
}

template <uint32_t TYPE, uint32_t SEG, bool MULTI, uint32_t NT>
cudaError_t launch_imma_t(const ImmaPlan& plan, const CUtensorMap& map, const ImmaArgs& args, cudaStream_t stream,
                          bool pdl) {
    static bool configured[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !configured[dev]) {
        auto k = gemv_imma_kernel<TYPE, SEG, MULTI, NT>;
        cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
        // the whole unified L1 as shared memory, so two 113 KB CTAs fit on an SM
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(k, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
        if (e != cudaSuccess) return e;
        configured[dev] = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(plan.grid);
    cfg.blockDim = dim3((plan.warps + 1) * 32);
    cfg.dynamicSmemBytes = plan.smem_bytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, gemv_imma_kernel<TYPE, SEG, MULTI, NT>, map, args);
}

// One token: both group layouts; several tokens: the group-capable kernel only
// (it also serves a single group).
template <uint32_t TYPE, uint32_t SEG>
cudaError_t launch_imma_s(const ImmaPlan& plan, const CUtensorMap& map, const ImmaArgs& args, cudaStream_t stream,
                          bool pdl) {
    switch (plan.tokens) {
        case 1: return plan.groups > 1 ? launch_imma_t<TYPE, SEG, true, 1>(plan, map, args, stream, pdl)
                                       : launch_imma_t<TYPE, SEG, false, 1>(plan, map, args, stream, pdl);
        case 2: return launch_imma_t<TYPE, SEG, true, 2>(plan, map, args, stream, pdl);
        case 4: return launch_imma_t<TYPE, SEG, true, 4>(plan, map, args, stream, pdl);
        case 8: return launch_imma_t<TYPE, SEG, true, 8>(plan, map, args, stream, pdl);
        default: return cudaErrorInvalidValue;
    }
}

template <uint32_t TYPE>
cudaError_t launch_imma_p(const ImmaPlan& plan, const CUtensorMap& map, const ImmaArgs& args, cudaStream_t stream,
                          bool pdl) {
    switch (plan.seg_pairs) {
        case 4: return launch_imma_s<TYPE, 4>(plan, map, args, stream, pdl);
        case 8: return launch_imma_s<TYPE, 8>(plan, map, args, stream, pdl);
        case 16: return launch_imma_s<TYPE, 16>(plan, map, args, stream, pdl);
        default: return cudaErrorInvalidValue;
    }
}

uint64_t align_up64(uint64_t v, uint64_t a) { return (v + a - 1) / a * a; }

// NEDO_GPU_IMMA_SLICE=0 keeps one-token launches on the ring kernel (for comparisons).
bool slice_allowed() {
    static const bool allowed = [] {
        const char* e = getenv("NEDO_GPU_IMMA_SLICE");
        return !(e && e[0] == '0');
    }();
    return allowed;
}

// Bytes of one box row of `bp` block pairs: the data rounded to an odd
// multiple of 16 bytes (the eight fragment rows of a load then fall in
// distinct 16-byte bank groups).
uint64_t box_row_bytes(uint64_t bp, uint64_t pair_bytes) {
    const uint64_t b = align_up64(bp * pair_bytes, 16);
    return (b / 16u) % 2u == 0 ? b + 16u : b;
}

}  // namespace

ImmaPlan plan_imma(uint32_t type, uint64_t rows, uint64_t cols, int num_sms, int max_smem_optin,
                   const ImmaTuning* tune, uint32_t tokens) {
    ImmaPlan p;
    if (type != kQ8_0 && type != kQ4_0) return p;
    if (tokens != 1 && tokens != 2 && tokens != 4 && tokens != 8) return p;
    // tensor-map coordinates are int32: rows below 2^31
    if (cols % 64u || cols > 0xFFFFFFFFull || rows == 0 || rows >= 0x80000000ull || num_sms <= 0) return p;
    const uint64_t rb = row_bytes_of(type, cols);
    if (rb % 16u) return p;  // the tensor map's row stride
    const uint64_t pair_bytes = type == kQ8_0 ? 68u : 36u;
    const uint64_t pairs_total = cols / 64u;
    const ImmaTuning t = tune ? *tune : ImmaTuning{};
    const uint64_t tiles = (rows + kTileRows - 1) / kTileRows;
    // One CTA per SM per launch with the whole shared memory (a smaller budget on request).
    const bool wide = t.wide != 0;
    uint64_t budget = wide ? static_cast<uint64_t>(max_smem_optin) : kNarrowSmem;
    if (t.smem_budget && t.smem_budget < budget) budget = t.smem_budget;
    if (budget > static_cast<uint64_t>(max_smem_optin)) budget = max_smem_optin;
    const uint64_t per_sm = t.ctas_per_sm ? t.ctas_per_sm : 1u;
    const uint64_t grid = tiles < per_sm * num_sms ? tiles : per_sm * num_sms;
    const uint64_t tiles_per_cta = (tiles + grid - 1) / grid;
    if (tokens == 1 && t.slice != 0 && slice_allowed() && wide && per_sm == 1) {
        // resident slice: wide units (Q4_0 32 pairs = 1152 B, Q8_0 16 pairs = 1088 B
        // per row), narrower when the row is shorter
        uint64_t up = type == kQ4_0 ? 32u : 16u;
        while (up > 8u && up / 2u >= pairs_total) up /= 2u;
        const uint64_t box = box_row_bytes(up, pair_bytes);
        const uint64_t nchunk = (pairs_total + up - 1) / up;
        const uint64_t slots = tiles_per_cta * nchunk;
        const uint64_t unit = kTileRows * box;
        const uint64_t nsub = (pairs_total + kSubPairs - 1) / kSubPairs;
        const uint64_t part_floats = tiles_per_cta * nsub * 16u > 2u * kMaxWarps ? tiles_per_cta * nsub * 16u : 2u * kMaxWarps;
        const uint64_t smem = slots * unit + pairs_total * kPairTableBytes + part_floats * 4u + 8u * slots + 32u;
        // the x table's blocks in one pass of the consumer threads' registers
        if (box <= kMaxBoxBytes && smem <= budget && 2u * pairs_total <= kMaxWarps * 4u * kLimbPasses) {
            p.type = type;
            p.wide = true;
            p.slice = true;
            p.warps = kMaxWarps;
            p.team = 1;
            p.tokens = 1;
            p.seg_pairs = static_cast<uint32_t>(up);
            p.tile_rows = kTileRows;
            p.tiles = static_cast<uint32_t>(tiles);
            p.slots = static_cast<uint32_t>(slots);
            p.unit_bytes = static_cast<uint32_t>(unit);
            p.box_bytes = static_cast<uint32_t>(box);
            p.grid = static_cast<uint32_t>(grid);
            p.smem_bytes = static_cast<uint32_t>(smem);
            p.groups = 1;
            p.group_pairs = static_cast<uint32_t>(pairs_total);
            p.tile_group = tiles_per_cta > 2 && (t.max_tile_group == 0 || t.max_tile_group >= 5u) ? 5u : 2u;
            // Copies issued before x is requested: x's loads queue behind this SM's
            // earlier weight copies, so only about as much as lands while the CTA
            // waits for the previous kernel (measured: ~150 KB) goes out first.
            const uint64_t chunk_bytes = tiles_per_cta * unit;
            uint64_t early = kEarlyBytes / chunk_bytes;
            if (early < 1) early = 1;
            p.early_chunks = static_cast<uint32_t>(early < nchunk ? early : nchunk);
            p.ok = true;
            return p;
        }
    }
    // consumer warps: 16 for one token; 8 for several (each unit's MMA work grows with
    // the tokens, and 4 warps already keep the SM's int8 MMA pipe busy)
    const uint64_t max_warps = tokens == 1 ? kMaxWarps : 8u;
    // unit: 16 rows x 16 block pairs (Q4_0, 9.5 KB) or 8 (Q8_0, 9 KB), halved
    // (down to 4) while a CTA would have fewer units than warps
    uint64_t seg = t.seg_pairs ? t.seg_pairs : (type == kQ4_0 ? 16u : 8u);
    if (seg != 4u && seg != 8u && seg != 16u) return p;
    while (!t.seg_pairs && seg > 4u && (seg > pairs_total || tiles_per_cta * ((pairs_total + seg - 1) / seg) < max_warps))
        seg /= 2u;
    uint64_t box_bytes = box_row_bytes(seg, pair_bytes);
    if (box_bytes > kMaxBoxBytes) return p;
    uint64_t unit_bytes = kTileRows * box_bytes;  // a multiple of 256
    // column group: the whole row when its tables (one per token) fit the table
    // budget (24 KB for one token, 96 KB for several: their MMA work, not the ring,
    // bounds them), else a multiple of the segment
    uint64_t table_budget = t.table_budget ? t.table_budget : (tokens > 1 ? 96u : 24u) * 1024u;
    if (!t.table_budget && budget > 4u * unit_bytes + 8192u && table_budget > budget - 4u * unit_bytes - 8192u)
        table_budget = budget - 4u * unit_bytes - 8192u;  // leave room for a ring of 4 units
    const uint64_t pair_table = kPairTableBytes * tokens;
    uint64_t group = align_up64(pairs_total, seg);
    if (group * pair_table > table_budget) {
        group = (table_budget / pair_table) / seg * seg;
        if (group == 0) group = seg;
    }
    // several tokens: narrower units while a CTA's share of a group has fewer
    // units than warps (the MMA work, not the copies, bounds these)
    while (tokens > 1 && !t.seg_pairs && seg > 4u && tiles_per_cta * ((group + seg - 1) / seg) < max_warps) seg /= 2u;
    box_bytes = box_row_bytes(seg, pair_bytes);
    unit_bytes = kTileRows * box_bytes;
    const uint64_t groups = (pairs_total + group - 1) / group;
    // Teams: a CTA with fewer tiles than warps lets 2, 4 or 8 warps share a tile
    // (each a share of its segments) so that up to 8 warps stay busy.
    const uint64_t nseg = (group + seg - 1) / seg;
    // Team size K: the smallest power of two (at most the segments per tile)
    // that gives every warp a share, tiles x K >= warps.
    uint64_t team = 1;
    while (team * 2u <= nseg && team * 2u <= max_warps && tiles_per_cta * team < max_warps) team *= 2u;
    const uint64_t nteams = tiles_per_cta < max_warps / team ? tiles_per_cta : max_warps / team;
    const uint64_t warps = nteams * team;
    // tables, 8 team barriers, partial sums, abort flag
    const uint64_t fixed = group * pair_table + 64u + 2u * warps * tokens * 16u * 4u + 16u;
    auto smem_of = [&](uint64_t s) { return s * unit_bytes + fixed + 20u * s; };
    // ring: the CTA's whole work when it fits, else the most slots that fit
    const uint64_t work = tiles_per_cta * groups * nseg;
    uint64_t slots = t.slots ? t.slots : work;
    if (slots < 2) slots = 2;
    if (slots > kMaxSlots) slots = kMaxSlots;
    while (slots > 2 && smem_of(slots) > budget) --slots;
    if (smem_of(slots) > budget) return p;
    p.type = type;
    p.wide = wide;
    p.warps = static_cast<uint32_t>(warps);
    p.team = static_cast<uint32_t>(team);
    p.tokens = tokens;
    p.seg_pairs = static_cast<uint32_t>(seg);
    p.tile_rows = kTileRows;
    p.tiles = static_cast<uint32_t>(tiles);
    p.slots = static_cast<uint32_t>(slots);
    p.unit_bytes = static_cast<uint32_t>(unit_bytes);
    p.box_bytes = static_cast<uint32_t>(box_bytes);
    p.grid = static_cast<uint32_t>(grid);
    p.smem_bytes = static_cast<uint32_t>(smem_of(slots));
    p.groups = static_cast<uint32_t>(groups);
    p.group_pairs = static_cast<uint32_t>(group);
    p.ok = true;
    return p;
}

ImmaPlan plan_imma_multi(uint32_t type, uint64_t rows, uint64_t cols, int num_sms, int max_smem_optin,
                         uint32_t tokens, uint32_t vectors_per_group) {
    ImmaPlan p;
    if (type != kQ8_0 && type != kQ4_0) return p;
    if (tokens < 2 || cols % 64u || cols > 0xFFFFFFFFull || rows == 0 || rows >= 0x80000000ull || num_sms <= 0)
        return p;
    const uint64_t rb = row_bytes_of(type, cols);
    if (rb % 16u) return p;  // the tensor map's row stride
    const uint64_t pair_bytes = type == kQ8_0 ? 68u : 36u;
    const uint64_t pairs_total = cols / 64u;
    // units of 16 rows x 32 (Q4_0) or 16 (Q8_0) block pairs, as the one-vector slice
    const uint64_t up = type == kQ4_0 ? 32u : 16u;
    if (up / 2u >= pairs_total) return p;
    const uint64_t box = box_row_bytes(up, pair_bytes);
    const uint64_t unit = kTileRows * box;
    const uint64_t nchunk = (pairs_total + up - 1) / up;
    const uint64_t tiles = (rows + kTileRows - 1) / kTileRows;
    // Among the group sizes that fit: the most token groups whose CTAs hold at
    // most kMultiCtaWeightBytes of weight each, else the smallest share of
    // weight per CTA.  (Measured on 8-vector launches: the per-CTA weight
    // share sets the time above ~100 KB -- 1536 x 4096 Q8_0 at 139 KB 8.9 us,
    // 209 KB 12.4 us; 4096 x 1536 at 104 KB 6.7 us, 182 KB 10.7 us -- and below
    // it more groups win: 1536 x 1536 with 4 groups of 2 vectors 4.95 us, 2
    // groups of 4 5.3, 1 group of 8 6.1.)
    uint64_t best_bytes = 0, best_groups = 0;
    const uint32_t per_group[3] = {2u, 4u, 8u};
    for (uint32_t nt : per_group) {
        if (vectors_per_group && nt != vectors_per_group) continue;
        if (tokens % nt) continue;
        const uint64_t groups = tokens / nt;
        const uint64_t r = 16u / nt;  // tiles per register group (the kernel's R)
        uint64_t ctas = static_cast<uint64_t>(num_sms) / groups;
        if (ctas == 0) continue;
        if (ctas > tiles) ctas = tiles;
        const uint64_t tpc = (tiles + ctas - 1) / ctas;
        const uint64_t warps = nt >= 8 ? 12u : kMaxWarps;
        // every (vector, block) of the tables in one pass of the consumer threads' registers
        const uint64_t per_pass = warps * 4u;
        if (nt * 2u * pairs_total > per_pass * kLimbPasses) continue;
        const uint64_t slots = tpc * nchunk;
        const uint64_t smem = slots * unit + multi_region_bytes(nt, pairs_total, warps, tpc, r) + 8u * slots + 16u;
        if (smem > static_cast<uint64_t>(max_smem_optin)) continue;
        const uint64_t cta_bytes = tpc * kTileRows * rb;
        if (p.ok) {
            const bool small = cta_bytes <= kMultiCtaWeightBytes, best_small = best_bytes <= kMultiCtaWeightBytes;
            const bool better = small ? (!best_small || groups > best_groups) : (!best_small && cta_bytes < best_bytes);
            if (!better) continue;
        }
        best_bytes = cta_bytes;
        best_groups = groups;
        p.type = type;
        p.wide = true;
        p.slice = false;
        p.multi = true;
        p.warps = static_cast<uint32_t>(warps);
        p.team = 1;
        p.tokens = nt;
        p.token_groups = static_cast<uint32_t>(groups);
        p.seg_pairs = static_cast<uint32_t>(up);
        p.tile_rows = kTileRows;
        p.tiles = static_cast<uint32_t>(tiles);
        p.slots = static_cast<uint32_t>(slots);
        p.unit_bytes = static_cast<uint32_t>(unit);
        p.box_bytes = static_cast<uint32_t>(box);
        p.grid = static_cast<uint32_t>(groups * ctas);
        p.smem_bytes = static_cast<uint32_t>(smem);
        p.groups = 1;
        p.group_pairs = static_cast<uint32_t>(pairs_total);
        p.tile_group = static_cast<uint32_t>(r);
        const uint64_t chunk_bytes = tpc * unit;
        uint64_t early = kEarlyBytes / chunk_bytes;
        if (early < 1) early = 1;
        p.early_chunks = static_cast<uint32_t>(early < nchunk ? early : nchunk);
        p.ok = true;
    }
    return p;
}

cudaError_t launch_imma(const ImmaPlan& plan, const void* w, const float* x, float* y, uint64_t rows, uint64_t cols,
                        DeviceStatus* status, cudaStream_t stream, bool pdl, const PeerGather* gather, uint64_t ldx,
                        uint64_t ldy, const XPrologue* prologue) {
    if (prologue && prologue->mode != kPrologueNone && !plan.slice) return cudaErrorInvalidValue;
    if (plan.multi && (plan.token_groups == 0 || plan.grid % plan.token_groups != 0)) return cudaErrorInvalidValue;
    if (!plan.ok || (reinterpret_cast<uintptr_t>(w) & 15u) != 0 || (reinterpret_cast<uintptr_t>(x) & 15u) != 0)
        return cudaErrorInvalidValue;
    if (ldx == 0) ldx = cols;
    if (ldy == 0) ldy = rows;
    // x rows are read as float4: every token vector starts on a 16-byte boundary
    if ((plan.tokens > 1 || plan.multi) && (ldx % 4u != 0 || ldx < cols || ldy < rows)) return cudaErrorInvalidValue;
    if (gather != nullptr && (plan.tokens != 1 || plan.multi)) return cudaErrorInvalidValue;
    ImmaArgs a{};
    if (gather != nullptr) {
        if (gather->npeers > kMaxPeers) return cudaErrorInvalidValue;
        a.npeers = gather->npeers;
        a.peer_row_offset = gather->row_offset;
        for (uint32_t k = 0; k < gather->npeers; ++k) {
            a.peer_y[k] = gather->peer_y[k];
            a.peer_signal[k] = gather->peer_signal[k];
        }
    }
    const uint64_t rb = row_bytes_of(plan.type, cols);
    // The weight as rows of 8-byte elements; a box is 16 rows x box_bytes.
    EncodeTiled enc = encode_tiled_fn();
    if (enc == nullptr) return cudaErrorNotSupported;
    CUtensorMap map;
    const cuuint64_t dims[2] = {rb / 8u, rows}, strides[1] = {rb};
    const cuuint32_t box[2] = {plan.box_bytes / 8u, kTileRows}, es[2] = {1, 1};
    if (enc(&map, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<void*>(w), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return cudaErrorInvalidValue;
    a.x = x;
    a.y = y;
    a.rows = rows;
    a.tiles = plan.tiles;
    a.pairs_total = static_cast<uint32_t>(cols / 64u);
    a.group_pairs = plan.group_pairs;
    a.groups = plan.groups;
    a.box_bytes = plan.box_bytes;
    a.warps = plan.warps;
    a.team = plan.team;
    a.slots = plan.slots;
    a.unit_bytes = plan.unit_bytes;
    a.ldx = ldx;
    a.ldy = ldy;
    a.status = status;
    a.early_chunks = plan.early_chunks;
    a.token_groups = plan.token_groups;
    if (prologue) a.pro = *prologue;
    if (plan.multi) {
        if (plan.type == kQ8_0) return launch_multi_p<kQ8_0>(plan, map, a, stream, pdl);
        return launch_multi_p<kQ4_0>(plan, map, a, stream, pdl);
    }
    if (plan.slice) {
        if (plan.type == kQ8_0) return launch_slice_p<kQ8_0>(plan, map, a, stream, pdl);
        return launch_slice_p<kQ4_0>(plan, map, a, stream, pdl);
    }
    if (plan.type == kQ8_0) return launch_imma_p<kQ8_0>(plan, map, a, stream, pdl);
    return launch_imma_p<kQ4_0>(plan, map, a, stream, pdl);
}

}  // namespace nedo_gpu
