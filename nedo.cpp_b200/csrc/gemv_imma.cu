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
// A warp owns a fixed slice of the columns (its x limbs stay in registers while
// the CTA streams its rows) and all warps of a CTA share each 16-row tile,
// which a producer warp streams from HBM into a shared-memory ring with
// cp.async.bulk (one copy per row, 16 lanes issuing; no multicast).  Rows
// longer than 15 warps x 8 pairs are cut into column chunks processed one
// after the other (x limbs rebuilt per chunk, y accumulated in chunk order).
// Every wait is bounded; a CTA-wide abort flag stops every warp after the
// first timed-out wait.
#include <math.h>

#include "common.cuh"
#include "launch.h"

namespace nedo_gpu {
namespace {

// Consumer warps per CTA (+1 producer warp).  8 block pairs per warp keep 48
// x registers live and need the 128-register budget of 512 threads (15
// consumers); 4 or 2 pairs fit in the 120 registers of 544 threads (16).
constexpr uint32_t kImmaMaxWarps = 16;
template <uint32_t PAIRS>
constexpr uint32_t imma_max_consumers() {
    return PAIRS >= 8 ? 15u : 16u;
}

struct ImmaArgs {
    const uint8_t* w;
    const float* x;
    float* y;
    uint64_t rows;
    uint32_t row_bytes;
    uint32_t pairs_total;  // cols / 64
    uint32_t chunk_pairs;  // block pairs per column chunk (a multiple of 4 when chunks > 1)
    uint32_t chunks;       // column chunks, streamed one after the other
    uint32_t row_pitch;    // shared-memory bytes per tile row, 16 mod 32 (conflict free)
    uint32_t warps;        // consumer warps (column slices)
    uint32_t slots;
    uint32_t slot_bytes;
    DeviceStatus* status;
    // Fused all-gather (npeers > 0): each finished y row is also stored at
    // peer_y[k][peer_row_offset + row] on every peer (NVLink peer stores), and
    // every CTA adds 1 to each peer's counter peer_signal[k] once its rows are
    // visible system-wide.
    uint32_t npeers;
    uint64_t peer_row_offset;
    float* peer_y[kMaxPeers];
    uint32_t* peer_signal[kMaxPeers];
};

constexpr uint32_t kTileRows = 16;  // rows per tile: the M of one IMMA

// x limb table in shared memory: per block 144 bytes (4 limbs x 32 int8 and
// padding that keeps the lane loads conflict free), then per block the
// exponent e and the four limb sums.
constexpr uint32_t kLimbBlockBytes = 144;

__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;"); }

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

__device__ __forceinline__ void imma(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                     uint32_t b1, bool first, bool a_unsigned) {
    if (a_unsigned) {
        if (first)
            asm volatile(
                "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
                : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
                : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
        else
            asm volatile(
                "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
                : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
    } else {
        if (first)
            asm volatile(
                "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
                : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
                : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
        else
            asm volatile(
                "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
                : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
    }
}

// Per-lane x state for one block pair.
struct XPair {
    uint32_t b0[2];  // B register b0 (k < 16: even block) for the two IMMA halves; 0 unless column g is in it
    uint32_t b1[2];  // B register b1 (k >= 16: odd block)
    float scale;     // 2^(7*(3-lambda_b) - e_block) for this lane's D columns (2t, 2t+1)
    int offset;      // Q4_0: 8 * (sum L_a * 128 + sum L_b) for the same columns
};

// All consumer threads: decompose x into the limb table, 8 threads per block
// (4 positions each).  e_b makes max |x_b| * 2^e_b fall in [2^26, 2^27).
template <bool SUMS>
__device__ __forceinline__ void limb_block_group(float4 v, uint32_t b, uint32_t q, bool in, uint8_t* table, int* binfo) {
    float m = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
    m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, 1));
    m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, 2));
    m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, 4));
    int e = 0;  // an all-zero block keeps e = 0 (all limbs 0)
    if (m > 0.f) {
        const int E = static_cast<int>((__float_as_uint(m) >> 23) & 0xFFu) - 127;  // m in [2^E, 2^(E+1))
        e = 26 - E;                                                                 // in [-101, 153]
        if (e > 126) e = 126;
    }
    const float sc = __uint_as_float(static_cast<uint32_t>(e + 127) << 23);  // 2^e, exact
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
    auto gather = [](uint32_t a, uint32_t b, uint32_t c, uint32_t d, uint32_t sel) {
        return prmt(prmt(a, b, sel), prmt(c, d, sel), 0x5410u);
    };
    uint32_t L[4];
    L[3] = gather(X0, X1, X2, X3, 0x3340u) & 0x7F7F7F7Fu;
    L[2] = gather(X0 << 1, X1 << 1, X2 << 1, X3 << 1, 0x3351u) & 0x7F7F7F7Fu;
    L[1] = gather(X0 << 2, X1 << 2, X2 << 2, X3 << 2, 0x3362u) & 0x7F7F7F7Fu;
    L[0] = gather(X0 << 3, X1 << 3, X2 << 3, X3 << 3, 0x3373u);
    int sum[4] = {0, 0, 0, 0};  // limb sums over the block (Q4_0 offsets only)
    if (SUMS) {
        // two sums per word: low 16 bits a non-negative sum (<= 32 * 127), high 16 bits the other
        int s32 = __dp4a(static_cast<int>(L[3]), 0x01010101, 0) + __dp4a(static_cast<int>(L[0]), 0x01010101, 0) * 65536;
        int s21 = __dp4a(static_cast<int>(L[2]), 0x01010101, 0) + __dp4a(static_cast<int>(L[1]), 0x01010101, 0) * 65536;
        s32 += __shfl_xor_sync(0xFFFFFFFFu, s32, 1);
        s21 += __shfl_xor_sync(0xFFFFFFFFu, s21, 1);
        s32 += __shfl_xor_sync(0xFFFFFFFFu, s32, 2);
        s21 += __shfl_xor_sync(0xFFFFFFFFu, s21, 2);
        s32 += __shfl_xor_sync(0xFFFFFFFFu, s32, 4);
        s21 += __shfl_xor_sync(0xFFFFFFFFu, s21, 4);
        sum[3] = s32 & 0xFFFF;
        sum[0] = (s32 - sum[3]) >> 16;
        sum[2] = s21 & 0xFFFF;
        sum[1] = (s21 - sum[2]) >> 16;
    }
    if (in) {
        uint32_t* tb = reinterpret_cast<uint32_t*>(table + static_cast<size_t>(b) * kLimbBlockBytes);
#pragma unroll
        for (int l = 0; l < 4; ++l) tb[l * 8 + q] = L[l];
        if (q == 0) {
            int* bi = binfo + 5u * b;
            bi[0] = e;
            bi[1] = sum[0];
            bi[2] = sum[1];
            bi[3] = sum[2];
            bi[4] = sum[3];
        }
    }
}

// All consumer threads: decompose x into the limb table, 8 threads per block
// (4 positions each), every x load issued before any is used.
// e_b makes max |x_b| * 2^e_b fall in [2^26, 2^27).
constexpr uint32_t kLimbPasses = 8;  // up to 8 * nthreads / 8 blocks staged in registers at once
template <bool SUMS>
__device__ __forceinline__ void build_limb_table(const float* __restrict__ x, uint32_t nblocks, uint32_t tid,
                                                 uint32_t nthreads, uint8_t* table, int* binfo) {
    const uint32_t per_pass = nthreads / 8u;
    const uint32_t q = tid & 7u;
    for (uint32_t base = 0; base < nblocks; base += per_pass * kLimbPasses) {
        float4 v[kLimbPasses];
#pragma unroll
        for (uint32_t k = 0; k < kLimbPasses; ++k) {
            const uint32_t b = base + k * per_pass + tid / 8u;
            v[k] = b < nblocks ? __ldg(reinterpret_cast<const float4*>(x + 32u * b + 4u * q)) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (uint32_t k = 0; k < kLimbPasses; ++k) {
            const uint32_t b = base + k * per_pass + tid / 8u;
            if (base + k * per_pass < nblocks) limb_block_group<SUMS>(v[k], b, q, b < nblocks, table, binfo);
        }
    }
}

// This lane's x state for block pair `gp`, read from the limb table.
// Lane (g, t): B column n = g; g < 4 -> even block, limb g; g >= 4 -> odd block, limb g-4.
// D columns of the lane: n = 2t, 2t+1 -> block (t >> 1), limbs 2(t&1), 2(t&1)+1.
__device__ __forceinline__ XPair load_xpair(const uint8_t* table, const int* binfo, uint32_t gp, uint32_t lane,
                                            bool q4) {
    const uint32_t g = lane >> 2, t = lane & 3u;
    const uint32_t blk = 2u * gp + (g >= 4 ? 1u : 0u), lambda = g & 3u;
    const uint32_t* tb = reinterpret_cast<const uint32_t*>(table + static_cast<size_t>(blk) * kLimbBlockBytes);
    const uint32_t w_lo = tb[lambda * 8u + t], w_hi = tb[lambda * 8u + 4u + t];  // positions 4t.., 16+4t..
    const bool even = g < 4;
    XPair xp;
    xp.b0[0] = even ? w_lo : 0u;
    xp.b0[1] = even ? w_hi : 0u;
    xp.b1[0] = even ? 0u : w_lo;
    xp.b1[1] = even ? 0u : w_hi;
    const uint32_t dblk = 2u * gp + (t >> 1), la = 2u * (t & 1u);
    const int* bi = binfo + 5u * dblk;
    const int k = 7 * (3 - static_cast<int>(la + 1u)) - bi[0];  // in [-126, 115]
    xp.scale = __uint_as_float(static_cast<uint32_t>(k + 127) << 23);
    xp.offset = q4 ? 8 * (bi[1 + la] * 128 + bi[2 + la]) : 0;
    return xp;
}

// One 16-row tile against this warp's column slice: acc0 / acc1 collect the
// rows of fragment rows g and g+8 (this lane's D columns).  GUARD skips the
// pairs past `valid` (the last warp of a chunk).
template <uint32_t TYPE, uint32_t PAIRS, bool GUARD>
__device__ __forceinline__ void tile_dot(const uint8_t* r0p, const uint8_t* r1p, const XPair (&xs)[PAIRS], uint32_t valid,
                                         uint32_t t, uint32_t scale_blk, float& acc0, float& acc1) {
#pragma unroll
    for (uint32_t p = 0; p < PAIRS; ++p) {
        if (GUARD && p >= valid) break;
        const uint8_t* p0 = r0p + p * Pair<TYPE>::kBytes;
        const uint8_t* p1 = r1p + p * Pair<TYPE>::kBytes;
        int d[4];
        if constexpr (TYPE == kQ8_0) {
#pragma unroll
            for (uint32_t h = 0; h < 2; ++h) {
                // even block: quant bytes 16h+4t.. at pair offset 2+16h+4t (2 mod 4)
                const uint32_t o = 16u * h + 4u * t;
                const uint32_t* e0 = reinterpret_cast<const uint32_t*>(p0 + o);
                const uint32_t* e1 = reinterpret_cast<const uint32_t*>(p1 + o);
                const uint32_t a0 = __funnelshift_r(e0[0], e0[1], 16);
                const uint32_t a2 = *reinterpret_cast<const uint32_t*>(p0 + 36u + o);
                const uint32_t a1 = __funnelshift_r(e1[0], e1[1], 16);
                const uint32_t a3 = *reinterpret_cast<const uint32_t*>(p1 + 36u + o);
                imma(d, a0, a1, a2, a3, xs[p].b0[h], xs[p].b1[h], h == 0, false);
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
            imma(d, w0 & m, w1 & m, w2 & m, w3 & m, xs[p].b0[0], xs[p].b1[0], true, true);
            imma(d, (w0 >> 4) & m, (w1 >> 4) & m, (w2 >> 4) & m, (w3 >> 4) & m, xs[p].b0[1], xs[p].b1[1],
                 false, true);
        }
        // d[0], d[1]: row g, limbs (2(t&1), 2(t&1)+1) of block (t>>1); d[2], d[3]: row g+8
        const int v0 = d[0] * 128 + d[1] - xs[p].offset;
        const int v1 = d[2] * 128 + d[3] - xs[p].offset;
        const float s0 = half_bits_to_float(*reinterpret_cast<const uint16_t*>(p0 + scale_blk)) * xs[p].scale;
        const float s1 = half_bits_to_float(*reinterpret_cast<const uint16_t*>(p1 + scale_blk)) * xs[p].scale;
        acc0 = fmaf(static_cast<float>(v0), s0, acc0);
        acc1 = fmaf(static_cast<float>(v1), s1, acc1);
    }
}

// MULTI: the rows are cut into more than one column chunk.
template <uint32_t TYPE, uint32_t PAIRS, bool MULTI>
__global__ void __launch_bounds__((imma_max_consumers<PAIRS>() + 1) * 32, 1) gemv_imma_kernel(const ImmaArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t S = a.slots, W = a.warps;
    const uint32_t table_blocks = 2u * a.chunk_pairs;  // limb table capacity (one chunk)
    // [ring: S slots][limb table][block info][barriers][partial sums][abort flag]
    uint8_t* table = smem + static_cast<size_t>(S) * a.slot_bytes;
    int* binfo = reinterpret_cast<int*>(table + static_cast<size_t>(table_blocks) * kLimbBlockBytes);
    uint64_t* full = reinterpret_cast<uint64_t*>(
        reinterpret_cast<uint8_t*>(binfo) + ((static_cast<size_t>(table_blocks) * 20u + 7u) & ~static_cast<size_t>(7)));
    uint64_t* empty = full + S;
    uint64_t* redbar = empty + S;
    float* red = reinterpret_cast<float*>(redbar + S);  // [S][W][16]
    volatile uint32_t* abort_flag = reinterpret_cast<volatile uint32_t*>(red + static_cast<size_t>(S) * W * 16u);

    // this CTA's rows: an even split of all rows (to one row), cut into 16-row tiles;
    // the unit of work is (column chunk c, tile j), chunk-major
    const uint64_t row_begin = a.rows * blockIdx.x / gridDim.x;
    const uint64_t row_end = a.rows * (blockIdx.x + 1) / gridDim.x;
    const uint32_t my_tiles = static_cast<uint32_t>((row_end - row_begin + kTileRows - 1) / kTileRows);
    const uint32_t nchunks = MULTI ? a.chunks : 1u;
    const uint32_t units = my_tiles * nchunks;

    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], W);
            mbar_init(&redbar[s], W);
        }
        *abort_flag = 0u;
        fence_barrier_init();
    }
    __syncthreads();

    if (warp == W) {
        // ---------------- producer ----------------
        // Lane r copies row r's chunk (the whole row when there is one chunk)
        // into its padded shared-memory row: 16 copies issued in parallel.
        const uint64_t policy = l2_policy_evict_first();
        uint32_t slot = 0, use = 0, u = 0;
        for (; u < units; ++u) {
            bool ok = true;
            if (lane == 0 && use > 0) ok = mbar_wait_bounded(&empty[slot], (use - 1u) & 1u, a.status, 11u);
            if (!__shfl_sync(0xFFFFFFFFu, ok, 0)) {
                if (lane == 0) *abort_flag = 1u;
                break;
            }
            const uint32_t c = u / my_tiles, j = u - c * my_tiles;
            const uint64_t row0 = row_begin + static_cast<uint64_t>(j) * kTileRows;
            const uint64_t left = row_end - row0;
            const uint32_t nrows = left < kTileRows ? static_cast<uint32_t>(left) : kTileRows;
            uint8_t* dst = smem + static_cast<size_t>(slot) * a.slot_bytes;
            const uint32_t pair0 = c * a.chunk_pairs;
            const uint32_t cp = a.pairs_total - pair0 < a.chunk_pairs ? a.pairs_total - pair0 : a.chunk_pairs;
            const uint32_t cbytes = cp * Pair<TYPE>::kBytes, cofs = pair0 * Pair<TYPE>::kBytes;
            if (lane == 0) mbar_arrive_expect_tx(&full[slot], nrows * cbytes);
            __syncwarp();
            if (lane < nrows)
                bulk_copy_g2s(dst + static_cast<size_t>(lane) * a.row_pitch, a.w + (row0 + lane) * a.row_bytes + cofs,
                              cbytes, &full[slot], policy);
            if (++slot == S) {
                slot = 0;
                ++use;
            }
        }
        // drain: every issued copy must land before the CTA may exit
        if (lane == 0) {
            const uint32_t first = u > S ? u - S : 0;
            for (uint32_t k = first; k < u; ++k) mbar_wait_bounded(&full[k % S], (k / S) & 1u, a.status, 12u);
        }
        return;
    }

    // ---------------- consumers: warp w owns block pairs [w*PAIRS, (w+1)*PAIRS) of each chunk ----------------
    constexpr bool kQ4 = TYPE == kQ4_0;
    const uint32_t g = lane >> 2, t = lane & 3u;
    const uint32_t scale_blk = (t >> 1) * Pair<TYPE>::kBlock;  // this lane's D block within a pair
    const size_t col0 = static_cast<size_t>(warp) * PAIRS * Pair<TYPE>::kBytes;
    // fragment rows g and g+8 = tile rows g and g+8
    const size_t off_a = static_cast<size_t>(g) * a.row_pitch + col0;
    const size_t off_b = off_a + 8u * static_cast<size_t>(a.row_pitch);

    grid_dependency_wait();  // x may come from the previous kernel
    bool ok = true;
    uint32_t slot = 0, parity = 0, u = 0;
    for (uint32_t c = 0; c < nchunks; ++c) {
        const uint32_t pair0 = c * a.chunk_pairs;
        const uint32_t cp = a.pairs_total - pair0 < a.chunk_pairs ? a.pairs_total - pair0 : a.chunk_pairs;
        if (c > 0) named_barrier_sync(1, W * 32u);  // every warp has its x registers of chunk c-1
        build_limb_table<kQ4>(a.x + static_cast<size_t>(pair0) * 64u, 2u * cp, threadIdx.x, W * 32u, table, binfo);
        named_barrier_sync(1, W * 32u);
        const uint32_t pw = warp * PAIRS;
        const uint32_t valid = cp > pw ? (cp - pw < PAIRS ? cp - pw : PAIRS) : 0u;  // warp-uniform
        XPair xs[PAIRS];
#pragma unroll
        for (uint32_t p = 0; p < PAIRS; ++p) {
            if (p < valid) {
                xs[p] = load_xpair(table, binfo, pw + p, lane, kQ4);
            } else {
                xs[p].b0[0] = xs[p].b0[1] = xs[p].b1[0] = xs[p].b1[1] = 0u;
                xs[p].scale = 0.f;
                xs[p].offset = 0;
            }
        }
        if (c == 0) grid_launch_dependents();

        for (uint32_t j = 0; j < my_tiles; ++j, ++u) {
            if (ok && *abort_flag != 0u) ok = false;
            if (ok && !mbar_wait_bounded(&full[slot], parity, a.status, 13u)) {
                ok = false;
                *abort_flag = 1u;
            }
            if (ok) {
                const uint8_t* tile = smem + static_cast<size_t>(slot) * a.slot_bytes;
                const uint8_t* r0p = tile + off_a;
                const uint8_t* r1p = tile + off_b;
                float acc0 = 0.f, acc1 = 0.f;
                if (valid == PAIRS)  // every pair of the slice exists: no per-pair checks
                    tile_dot<TYPE, PAIRS, false>(r0p, r1p, xs, valid, t, scale_blk, acc0, acc1);
                else
                    tile_dot<TYPE, PAIRS, true>(r0p, r1p, xs, valid, t, scale_blk, acc0, acc1);
                // fold the four t-lanes (columns) of each row
                acc0 += __shfl_xor_sync(0xFFFFFFFFu, acc0, 1);
                acc0 += __shfl_xor_sync(0xFFFFFFFFu, acc0, 2);
                acc1 += __shfl_xor_sync(0xFFFFFFFFu, acc1, 1);
                acc1 += __shfl_xor_sync(0xFFFFFFFFu, acc1, 2);
                float* rs = red + (static_cast<size_t>(slot) * W + warp) * 16u;
                if (t == 0) {
                    rs[g] = acc0;
                    rs[g + 8] = acc1;
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&redbar[slot]);
                if (warp != 0) {
                    if (lane == 0) mbar_arrive(&empty[slot]);
                } else {
                    // warp 0 folds the column slices of every row in fixed order; chunks
                    // add up in y in chunk order (only this thread touches the row)
                    if (!mbar_wait_bounded(&redbar[slot], parity, a.status, 14u)) {
                        ok = false;
                        *abort_flag = 1u;
                    } else {
                        const uint64_t row0 = row_begin + static_cast<uint64_t>(j) * kTileRows;
                        if (lane < kTileRows && row0 + lane < row_end) {
                            const float* rr = red + static_cast<size_t>(slot) * W * 16u + lane;
                            float v = 0.f;
                            for (uint32_t k = 0; k < W; ++k) v += rr[k * 16u];
                            if (MULTI && c > 0) v += a.y[row0 + lane];
                            a.y[row0 + lane] = v;
                        }
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&empty[slot]);
                    }
                }
            }
            if (++slot == S) {
                slot = 0;
                parity ^= 1u;
            }
        }
    }
    if (a.npeers != 0u && warp == 0 && ok) {
        // This CTA's rows, all written by warp 0, go to every peer as coalesced
        // stores off the tile pipeline; then lane 0 publishes the CTA on each
        // peer with a system-scope release add (ordered after the whole warp's
        // stores by the warp barrier).
        __syncwarp();
        for (uint64_t r = row_begin + lane; r < row_end; r += 32u) {
            const float v = __ldcg(a.y + r);
            for (uint32_t k = 0; k < a.npeers; ++k) a.peer_y[k][a.peer_row_offset + r] = v;
        }
        __syncwarp();
        if (lane == 0)
            for (uint32_t k = 0; k < a.npeers; ++k)
                asm volatile("red.release.sys.global.add.u32 [%0], 1;" ::"l"(a.peer_signal[k]) : "memory");
    }
}

template <uint32_t TYPE, uint32_t PAIRS, bool MULTI>
cudaError_t launch_imma_t(const ImmaPlan& plan, const ImmaArgs& args, cudaStream_t stream, bool pdl) {
    static bool configured[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(gemv_imma_kernel<TYPE, PAIRS, MULTI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             227 * 1024);
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
    return cudaLaunchKernelEx(&cfg, gemv_imma_kernel<TYPE, PAIRS, MULTI>, args);
}

template <uint32_t TYPE>
cudaError_t launch_imma_p(const ImmaPlan& plan, const ImmaArgs& args, cudaStream_t stream, bool pdl) {
    switch (plan.pairs) {
        case 2: return plan.chunks > 1 ? launch_imma_t<TYPE, 2, true>(plan, args, stream, pdl)
                                       : launch_imma_t<TYPE, 2, false>(plan, args, stream, pdl);
        case 4: return plan.chunks > 1 ? launch_imma_t<TYPE, 4, true>(plan, args, stream, pdl)
                                       : launch_imma_t<TYPE, 4, false>(plan, args, stream, pdl);
        case 8: return plan.chunks > 1 ? launch_imma_t<TYPE, 8, true>(plan, args, stream, pdl)
                                       : launch_imma_t<TYPE, 8, false>(plan, args, stream, pdl);
        default: return cudaErrorInvalidValue;
    }
}

uint64_t align_up64(uint64_t v, uint64_t a) { return (v + a - 1) / a * a; }

}  // namespace

ImmaPlan plan_imma(uint32_t type, uint64_t rows, uint64_t cols, int num_sms, int max_smem_optin,
                   const ImmaTuning* tune) {
    ImmaPlan p;
    if (type != kQ8_0 && type != kQ4_0) return p;
    if (cols % 64u || cols > 0xFFFFFFFFull || rows == 0 || rows > 0xFFFFFFFFull || num_sms <= 0) return p;
    const uint64_t rb = row_bytes_of(type, cols);
    if (rb % 16u) return p;
    const uint64_t pair_bytes = type == kQ8_0 ? 68u : 36u;
    const uint64_t pairs_total = cols / 64u;
    const ImmaTuning t = tune ? *tune : ImmaTuning{};
    // Column chunks: at most 15 warps x 8 pairs of x limbs live in registers at a
    // time.  Longer rows are cut into chunks of a multiple of 4 pairs (so every
    // chunk starts on a 16-byte boundary), streamed one after the other; more
    // chunks than that minimum when a chunk's 16-row tile would leave fewer than
    // 3 ring slots.
    constexpr uint64_t kMaxChunkPairs = 15u * 8u;
    uint64_t budget = t.smem_budget ? t.smem_budget : static_cast<uint64_t>(max_smem_optin);
    if (budget > static_cast<uint64_t>(max_smem_optin)) budget = max_smem_optin;
    const uint32_t grid = static_cast<uint32_t>(rows < static_cast<uint64_t>(num_sms) ? rows : num_sms);
    const uint64_t rows_per_cta = (rows + grid - 1) / grid;
    const uint64_t tiles_per_cta = (rows_per_cta + kTileRows - 1) / kTileRows;

    struct Cand {
        bool ok = false;
        uint64_t chunks = 0, chunk_pairs = 0, pitch = 0, slot_bytes = 0, slots = 0, smem = 0;
        uint32_t pairs = 0, warps = 0;
    };
    auto evaluate = [&](uint64_t chunks) {
        Cand c;
        uint64_t cpairs = pairs_total;
        if (chunks > 1) {
            if (pairs_total % 4u) return c;
            cpairs = align_up64((pairs_total + chunks - 1) / chunks, 4);
            if ((pairs_total + cpairs - 1) / cpairs != chunks) return c;
        }
        if (cpairs > kMaxChunkPairs) return c;
        // pairs per warp in {8, 4, 2}: the most pairs per warp (more independent
        // IMMA chains per warp) that still leaves at least 8 consumer warps, else
        // the most warps; 8 pairs allow 15 warps, fewer pairs 16.  The last warp
        // may own fewer pairs.
        for (uint32_t pp : {8u, 4u, 2u}) {
            const uint64_t w = (cpairs + pp - 1) / pp;
            if (w > (pp >= 8 ? 15u : kImmaMaxWarps)) continue;
            if (t.warps && w != t.warps) continue;
            if (c.warps == 0 || (c.warps < 8 && w > c.warps)) {
                c.pairs = pp;
                c.warps = static_cast<uint32_t>(w);
            }
        }
        if (c.warps == 0) return c;
        // one bulk copy per tile row (its chunk) into a row of pitch 16 mod 32
        // bytes, so the eight fragment rows of a load sit in distinct banks
        // (copying two rows per copy into 2-row groups measured no faster)
        const uint64_t cbytes = cpairs * pair_bytes;
        c.pitch = (cbytes % 32u == 16u) ? cbytes : cbytes + 16u;
        c.slot_bytes = align_up64(kTileRows * c.pitch, 128);
        const uint64_t table_blocks = 2u * cpairs;
        const uint64_t fixed = table_blocks * kLimbBlockBytes + align_up64(table_blocks * 20u, 8) + 16u;
        auto smem_of = [&](uint64_t s) { return s * c.slot_bytes + fixed + 24u * s + 4ull * s * c.warps * 16u; };
        // enough slots to hold a CTA's whole work when it fits, else the most that fit (>= 2)
        uint64_t slots = t.slots ? t.slots : tiles_per_cta * chunks;
        if (slots < 2) slots = 2;
        if (slots > 8) slots = 8;
        while (slots > 2 && smem_of(slots) > budget) --slots;
        if (smem_of(slots) > budget) return c;
        c.chunks = chunks;
        c.chunk_pairs = cpairs;
        c.slots = slots;
        c.smem = smem_of(slots);
        c.ok = true;
        return c;
    };
    const uint64_t c_min = (pairs_total + kMaxChunkPairs - 1) / kMaxChunkPairs;
    Cand best;
    for (uint64_t chunks = c_min; chunks <= c_min + 8 && chunks <= pairs_total; ++chunks) {
        const Cand c = evaluate(chunks);
        if (!c.ok) continue;
        if (!best.ok || (best.slots < 3 && c.slots > best.slots)) best = c;
        if (best.slots >= 3 || best.slots >= tiles_per_cta * best.chunks) break;
    }
    if (!best.ok) return p;
    const uint64_t chunks = best.chunks, chunk_pairs = best.chunk_pairs, pitch = best.pitch;
    const uint64_t slots = best.slots, slot_bytes = best.slot_bytes;
    const uint32_t pairs = best.pairs, warps = best.warps;
    p.type = type;
    p.warps = warps;
    p.pairs = pairs;
    p.tile_rows = kTileRows;
    p.row_stride = static_cast<uint32_t>(pitch);
    p.tiles = static_cast<uint32_t>((rows + kTileRows - 1) / kTileRows);
    p.slots = static_cast<uint32_t>(slots);
    p.slot_bytes = static_cast<uint32_t>(slot_bytes);
    p.grid = grid;
    p.smem_bytes = static_cast<uint32_t>(best.smem);
    p.chunks = static_cast<uint32_t>(chunks);
    p.chunk_pairs = static_cast<uint32_t>(chunk_pairs);
    p.ok = true;
    return p;
}

cudaError_t launch_imma(const ImmaPlan& plan, const void* w, const float* x, float* y, uint64_t rows, uint64_t cols,
                        DeviceStatus* status, cudaStream_t stream, bool pdl, const PeerGather* gather) {
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
    a.w = static_cast<const uint8_t*>(w);
    a.x = x;
    a.y = y;
    a.rows = rows;
    a.row_bytes = static_cast<uint32_t>(row_bytes_of(plan.type, cols));
    a.pairs_total = static_cast<uint32_t>(cols / 64u);
    a.chunk_pairs = plan.chunk_pairs;
    a.chunks = plan.chunks;
    a.row_pitch = plan.row_stride;
    a.warps = plan.warps;
    a.slots = plan.slots;
    a.slot_bytes = plan.slot_bytes;
    a.status = status;
    if (plan.type == kQ8_0) return launch_imma_p<kQ8_0>(plan, a, stream, pdl);
    return launch_imma_p<kQ4_0>(plan, a, stream, pdl);
}

}  // namespace nedo_gpu
