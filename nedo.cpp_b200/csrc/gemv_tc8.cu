// gemv_tc8.cu -- batch-1 Q8_0 / Q4_0 matvec on the 5th-generation tensor cores
// (tcgen05.mma kind::i8, A from TMEM), sized so that two launches share an SM.
//
// Same contract as the reference row kernels dot_q8 / dot_q4
// (src/kernels.cpp:124-160): y[r] = sum_b d[r][b] * sum_i q[r][b][i] * x[32b+i],
// x consumed in fp32 precision, fp32 output.
//
// Arithmetic (as the int8 tensor-pipe kernel in gemv_imma.cu): each 32-element
// block of x gets a power-of-two exponent e_b (max |x_b| * 2^e_b in
// [2^26, 2^27)); X = rint(x * 2^e_b) is split into four base-128 int8 limbs,
// X = L0*2^21 + L1*2^14 + L2*2^7 + L3.  The integer block dots of the limbs with
// the int8 quants (Q8_0) or the 0..15 nibbles (Q4_0, minus 8 * sum L) are exact
// in int32; only the per-block recombination d * 2^-e_b * sum is floating point.
//
// One MMA = one K step of a 16-row tile: M = 128 = 16 rows x 8 blocks, K = 32.
//   A (TMEM, 128 lanes x 32 bytes): lane m = 16p + r holds row r's block 8s + p
//     of K step s (the quants, or the nibbles expanded to bytes);
//   B (shared memory, K-major, N = 32): column n = 4p' + l holds limb l of x
//     block 8s + p';
//   D (TMEM, 128 x 32 int32): D[16p + r][4p + l] is the limb-l dot of row r's
//     block 8s + p.  The other 28 columns of a lane pair a block with the limbs
//     of other blocks and are never read.
// So every lane of the MMA does useful work on exactly one (row, block) pair,
// and a tile is 16 rows: 11008 rows make 688 tiles for 148 SMs.
//
// Streaming.  A unit is 16 rows x 16 blocks (two K steps); a ring slot holds
// two units, brought in by one 2D tensor-map copy (no multicast).  Roles
// (18 warps):
//   warp 0       producer: issues every slot's copy as ring slots free up;
//   warp 1       TMEM allocation and the MMA issuer (one thread);
//   warps 2-9    loaders, one per (TMEM lane quarter, K step of a unit): read
//                their lanes' blocks from the ring (row r, block p per lane),
//                expand Q4_0 nibbles, store the A tile into TMEM (tcgen05.st)
//                and the block scales d;
//   warps 10-17  build the x limb table once x is available, then the epilogue,
//                one per (lane quarter, K step): read the K step's D
//                (tcgen05.ld), combine the limbs with d * 2^-e, accumulate per
//                (row, block phase) and, per tile, add each row's 16 partial
//                sums in a fixed order.
// The weights do not depend on earlier kernels, so the copies and the A tiles
// of the first units are prepared before griddepcontrol.wait; x is read after
// it.  A CTA takes at most ~110 KB of shared memory, 576 threads x 56
// registers and 256 TMEM columns, so under programmatic dependent launch the
// next launch's CTA streams its weight on the same SM while this one finishes.
// Every wait is bounded; a CTA-wide abort flag stops every role after the
// first timeout, and TMEM is released on every path.
#include <cuda.h>
#include <math.h>

#include "common.cuh"
#include "launch.h"

namespace nedo_gpu {
namespace {

constexpr uint32_t kTileRows = 16;
constexpr uint32_t kPhases = 8;          // blocks per K step (block phases of a tile)
constexpr uint32_t kUnitSteps = 2;       // K steps per unit
constexpr uint32_t kUnitBlocks = kPhases * kUnitSteps;
constexpr uint32_t kSlotUnits = 2;       // units per ring slot (one tensor-map copy: 32 blocks)
constexpr uint32_t kN = 32;              // MMA N: 8 blocks x 4 limbs
constexpr uint32_t kNA = 4;              // A buffers (units) in TMEM: 16 columns each
constexpr uint32_t kND = 3;              // D buffers (units) in TMEM: 64 columns each
constexpr uint32_t kTmemCols = 256;
constexpr uint32_t kACol0 = 0;
constexpr uint32_t kDCol0 = kNA * 16u;
static_assert(kDCol0 + kND * kUnitSteps * kN <= kTmemCols, "TMEM budget");
constexpr uint32_t kThreads = 576;  // 18 warps
constexpr uint32_t kMaxSlots = 48;
constexpr uint32_t kMaxSteps = 32;       // K steps per row the x table holds (8192 columns)
constexpr uint32_t kStepTableBytes = 1024;  // 8 blocks x 4 limbs x 32 bytes
constexpr uint32_t kBudget = 110u * 1024u;  // per CTA: two CTAs fit on an SM

template <uint32_t TYPE>
struct Blk;
template <>
struct Blk<kQ8_0> {
    static constexpr uint32_t kBytes = 34;
};
template <>
struct Blk<kQ4_0> {
    static constexpr uint32_t kBytes = 18;
};

struct Tc8Args {
    const float* x;
    float* y;
    uint32_t rows;
    uint32_t tiles;      // ceil(rows / 16)
    uint32_t nb;         // blocks per row
    uint32_t steps;      // K steps per row: nb / 8
    uint32_t units;      // units per tile: ceil(steps / 2)
    uint32_t slots;      // ring slots
    uint32_t off_table;  // shared-memory offsets
    uint32_t off_consts;
    uint32_t off_sd;
    uint32_t off_red;
    uint32_t off_bars;
    DeviceStatus* status;
};

__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int32_t c0, int32_t c1,
                                            uint64_t* bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_addr(bar)), "l"(policy)
        : "memory");
}

// D (TMEM) = A (TMEM) x B (shared memory), int8 in, int32 out, D overwritten.
__device__ __forceinline__ void mma_i8_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(0u)
        : "memory");
}

__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
                 : "memory");
}

// This warp's 32 TMEM lanes, 8 consecutive columns from taddr: thread i writes lane i.
__device__ __forceinline__ void tc_st_x8(uint32_t taddr, const uint32_t (&v)[8]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
                 "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
                 : "memory");
}

__device__ __forceinline__ void tc_ld_x8(uint32_t taddr, uint32_t (&v)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
                 : "r"(taddr));
}

// Shared-memory matrix descriptor, K-major without swizzle: core matrices of 8
// rows x 16 bytes, LBO = byte stride between the two 16-byte K halves, SBO =
// byte stride between 8-row groups; descriptor version 1 (sm_100).
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
    d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
    d |= static_cast<uint64_t>(1u) << 46;
    return d;  // layout type 0: no swizzle
}

// kind::i8 instruction descriptor: D s32, A u8 (Q4_0 nibbles) or s8 (Q8_0
// quants), B s8 (limbs), both K-major, M = 128, N = 32.
template <uint32_t TYPE>
__host__ __device__ constexpr uint32_t idesc_i8() {
    return (2u << 4) | ((TYPE == kQ8_0 ? 1u : 0u) << 7) | (1u << 10) | ((kN >> 3) << 17) | ((128u >> 4) << 24);
}

// Bounded wait on an mbarrier phase that also gives up when another role has
// aborted (the flag is set by the first wait that ran out).
// The waits of this kernel are short, latency-critical hand-offs between roles
// (several completed by tcgen05.commit).  A try_wait may suspend the thread for
// an implementation-defined time before it notices the completed phase (about
// 0.5 us measured here), so they poll test_wait instead.
__device__ __forceinline__ bool test_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ bool wait_phase(uint64_t* bar, uint32_t parity, volatile uint32_t* abort_flag,
                                           DeviceStatus* st, uint32_t site) {
    if (test_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    const uint64_t limit = wait_limit_ns(st);
    for (uint32_t spin = 0;; ++spin) {
        // poll back to back for the first few microseconds (a hand-off), then
        // with a short sleep (a long wait, e.g. for the previous kernel)
        if (spin >= 128u) __nanosleep(64);
        if (test_wait(bar, parity)) return true;
        if (*abort_flag != 0u) return false;
        if (global_timer_ns() - t0 > limit) {
            if (st != nullptr && atomicOr(&st->flags, kErrWaitTimeout) == 0u) st->where = site;
            *abort_flag = 1u;
            return false;
        }
    }
}

// x limb table of one 32-element block, 8 threads (4 elements each, q = 0..7):
// limb rows of the K-major B operand and the block's epilogue constants.
//   T[b/2][k/16][(b%2)*4 + l][k%16]  (bytes; k = element index in the block)
//   C[b] = {2^(14-e), 2^(-e), 8*(128*S0 + S1), 8*(128*S2 + S3)} with S_l the
//          limb sums (Q4_0 nibble offset; 0 for Q8_0); non-finite x: NaN scales.
template <bool SUMS>
__device__ __forceinline__ void limb_block(float4 v, uint32_t b, uint32_t q, bool in, uint8_t* table,
                                           float4* consts) {
    const bool bad = !(fabsf(v.x) <= 3.402823466e38f) || !(fabsf(v.y) <= 3.402823466e38f) ||
                     !(fabsf(v.z) <= 3.402823466e38f) || !(fabsf(v.w) <= 3.402823466e38f);
    float m = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
    m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, 1));
    m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, 2));
    m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, 4));
    const uint32_t badv = __reduce_or_sync(0xFFFFFFFFu, bad ? (1u << (threadIdx.x & 24u)) : 0u);
    const bool block_bad = (badv >> (threadIdx.x & 24u)) & 1u;
    int e = 0;  // an all-zero block keeps e = 0 (all limbs 0)
    if (m > 0.f && !block_bad) {
        const int E = static_cast<int>((__float_as_uint(m) >> 23) & 0xFFu) - 127;  // m in [2^E, 2^(E+1))
        e = 26 - E;
        if (e > 126) e = 126;
    }
    const float sc = __uint_as_float(static_cast<uint32_t>(e + 127) << 23);  // 2^e, exact
    uint32_t X[4] = {0u, 0u, 0u, 0u};
    if (!block_bad) {
        X[0] = static_cast<uint32_t>(__float2int_rn(v.x * sc));
        X[1] = static_cast<uint32_t>(__float2int_rn(v.y * sc));
        X[2] = static_cast<uint32_t>(__float2int_rn(v.z * sc));
        X[3] = static_cast<uint32_t>(__float2int_rn(v.w * sc));
    }
    // |X| < 2^27: X = L0*2^21 + L1*2^14 + L2*2^7 + L3 with L0 = X >> 21 in [-64, 63]
    // and L1..L3 the 7-bit floor remainders; limb l of element i is byte (3 - l)
    // of X << (3 - l), masked to 7 bits for l > 0.  PRMT gathers that byte of the
    // four elements into one word (element order = byte order).
    auto gather = [&](uint32_t s, uint32_t sel) {
        return prmt(prmt(X[0] << s, X[1] << s, sel), prmt(X[2] << s, X[3] << s, sel), 0x5410u);
    };
    uint32_t L[4];
    L[3] = gather(0, 0x3340u) & 0x7F7F7F7Fu;
    L[2] = gather(1, 0x3351u) & 0x7F7F7F7Fu;
    L[1] = gather(2, 0x3362u) & 0x7F7F7F7Fu;
    L[0] = gather(3, 0x3373u);
    uint8_t* tb = table + (b >> 1) * 256u + (q >> 2) * 128u + (b & 1u) * 64u + (q & 3u) * 4u;
    if (in) {
#pragma unroll
        for (uint32_t l = 0; l < 4; ++l) *reinterpret_cast<uint32_t*>(tb + l * 16u) = L[l];
    }
    int chi = 0, clo = 0;
    if (SUMS) {
        // limb sums over the block's 8 threads (each at most 32 * 127)
        int s0 = __dp4a(static_cast<int>(L[0]), 0x01010101, 0), s1 = __dp4a(static_cast<int>(L[1]), 0x01010101, 0);
        int s2 = __dp4a(static_cast<int>(L[2]), 0x01010101, 0), s3 = __dp4a(static_cast<int>(L[3]), 0x01010101, 0);
        int hi = 128 * s0 + s1, lo = 128 * s2 + s3;
        hi += __shfl_xor_sync(0xFFFFFFFFu, hi, 1);
        lo += __shfl_xor_sync(0xFFFFFFFFu, lo, 1);
        hi += __shfl_xor_sync(0xFFFFFFFFu, hi, 2);
        lo += __shfl_xor_sync(0xFFFFFFFFu, lo, 2);
        hi += __shfl_xor_sync(0xFFFFFFFFu, hi, 4);
        lo += __shfl_xor_sync(0xFFFFFFFFu, lo, 4);
        chi = 8 * hi;
        clo = 8 * lo;
    }
    if (in && q == 0) {
        float shi = __uint_as_float(static_cast<uint32_t>(14 - e + 127) << 23);  // 2^(14-e), a normal float
        float slo = __uint_as_float(static_cast<uint32_t>(-e + 127) << 23);      // 2^(-e)
        if (block_bad) shi = slo = __uint_as_float(0x7FC00000u);                 // NaN, as the reference's sums
        consts[b] = make_float4(shi, slo, __int_as_float(chi), __int_as_float(clo));
    }
}

template <uint32_t TYPE>
__global__ void __launch_bounds__(kThreads, 2)
    gemv_tc8_kernel(const __grid_constant__ CUtensorMap map, const Tc8Args a) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr uint32_t BB = Blk<TYPE>::kBytes;
    constexpr uint32_t kSRB = kSlotUnits * kUnitBlocks * BB;  // data bytes per slot row: 1088 or 576
    constexpr uint32_t kPitch = kSRB + 16u;                    // its shared-memory pitch: 1104 or 592
    constexpr uint32_t kSlotBytes = kTileRows * kPitch;        // 17664 or 9472
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t S = a.slots;

    uint8_t* const table = smem + a.off_table;
    float4* const consts = reinterpret_cast<float4*>(smem + a.off_consts);
    float* const sd = reinterpret_cast<float*>(smem + a.off_sd);    // [kNA][2][128] block scales d
    float* const red = reinterpret_cast<float*>(smem + a.off_red);  // [2][8][16] per-tile partial sums
    uint64_t* const ring_full = reinterpret_cast<uint64_t*>(smem + a.off_bars);
    uint64_t* const ring_empty = ring_full + S;
    uint64_t* const a_full = ring_empty + S;
    uint64_t* const a_free = a_full + kNA;
    uint64_t* const d_full = a_free + kNA;
    uint64_t* const d_free = d_full + kND;
    uint64_t* const table_full = d_free + kND;
    uint64_t* const mma_done = table_full + 1;
    uint64_t* const red_full = mma_done + 1;  // [2] a tile's per-warp partial sums are written
    uint64_t* const red_free = red_full + 2;  // [2] ... and have been added up
    uint32_t* const tmem_slot = reinterpret_cast<uint32_t*>(red_free + 2);
    volatile uint32_t* const abort_flag = tmem_slot + 1;

    // this CTA's tiles: an even split of all 16-row tiles
    const uint32_t tile_begin = static_cast<uint32_t>(static_cast<uint64_t>(a.tiles) * blockIdx.x / gridDim.x);
    const uint32_t tile_end = static_cast<uint32_t>(static_cast<uint64_t>(a.tiles) * (blockIdx.x + 1) / gridDim.x);
    const uint32_t my_tiles = tile_end - tile_begin;
    const uint32_t units = a.units;                    // compute units per tile (2 K steps each)
    const uint32_t spt = (units + kSlotUnits - 1) / kSlotUnits;  // ring slots (copies) per tile
    const uint32_t total = my_tiles * units;           // compute units of this CTA, tile-major
    const uint32_t copies = my_tiles * spt;

    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < S; ++s) {
            mbar_init(&ring_full[s], 1);
            mbar_init(&ring_empty[s], 16);  // 8 loader warps x 2 units (a lone unit arrives twice)
        }
        for (uint32_t s = 0; s < kNA; ++s) {
            mbar_init(&a_full[s], 8);  // the eight loader warps
            mbar_init(&a_free[s], 8);  // the eight epilogue warps
        }
        for (uint32_t s = 0; s < kND; ++s) {
            mbar_init(&d_full[s], 1);
            mbar_init(&d_free[s], 8);
        }
        mbar_init(table_full, 8);
        mbar_init(mma_done, 1);
        for (uint32_t s = 0; s < 2; ++s) {
            mbar_init(&red_full[s], 8);
            mbar_init(&red_free[s], 1);
        }
        *abort_flag = 0u;
        fence_barrier_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                     "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    __syncwarp();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    // the next kernel on the stream may be scheduled now: its CTAs stream their
    // weights beside this CTA and read their inputs only after this grid ends
    if (threadIdx.x == 0) asm volatile("griddepcontrol.launch_dependents;");

    if (warp == 0) {
        // ---------------- producer ----------------
        if (lane == 0) {
            const uint64_t policy = l2_policy_evict_first();
            const uint32_t sbase = smem_addr(smem);
            uint32_t issued = 0, slot = 0, use = 0, t = 0, sk = 0;
            for (uint32_t c = 0; c < copies; ++c) {
                if (use > 0 && !wait_phase(&ring_empty[slot], (use - 1u) & 1u, abort_flag, a.status, 61u)) break;
                mbar_arrive_expect_tx(&ring_full[slot], kSlotBytes);
                // x in 8-byte elements: a slot starts at sk * 32 blocks (a multiple of 16 bytes)
                tma_load_2d(sbase + slot * kSlotBytes, &map, static_cast<int32_t>(sk * (kSRB / 8u)),
                            static_cast<int32_t>((tile_begin + t) * kTileRows), &ring_full[slot], policy);
                issued = c + 1u;
                if (++sk == spt) {
                    sk = 0;
                    ++t;
                }
                if (++slot == S) {
                    slot = 0;
                    ++use;
                }
            }
            // every issued copy has landed before the CTA may exit
            const uint32_t first = issued > S ? issued - S : 0u;
            for (uint32_t k = first; k < issued; ++k) mbar_wait_bounded(&ring_full[k % S], (k / S) & 1u, a.status, 62u);
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            bool ok = wait_phase(table_full, 0, abort_flag, a.status, 63u);
            tc_fence_after();
            const uint32_t tbase = smem_addr(table);
            uint32_t ab = 0, aph = 0, db = 0, dph = 0, uk = 0;
            for (uint32_t u = 0; u < total && ok; ++u) {
                ok = wait_phase(&a_full[ab], aph, abort_flag, a.status, 64u);
                if (ok && u >= kND) ok = wait_phase(&d_free[db], dph ^ 1u, abort_flag, a.status, 65u);
                if (!ok) break;
                tc_fence_after();
#pragma unroll
                for (uint32_t sub = 0; sub < kUnitSteps; ++sub) {
                    const uint32_t s = uk * kUnitSteps + sub;
                    if (s < a.steps)
                        mma_i8_ts(tmem + kDCol0 + db * (kUnitSteps * kN) + sub * kN, tmem + kACol0 + ab * 16u + sub * 8u,
                                  kmajor_desc(tbase + s * kStepTableBytes, 128u, 256u), idesc_i8<TYPE>());
                }
                tc_commit(&d_full[db]);
                if (++uk == units) uk = 0;
                if (++ab == kNA) {
                    ab = 0;
                    aph ^= 1u;
                }
                if (++db == kND) {
                    db = 0;
                    dph ^= 1u;
                }
            }
            tc_commit(mma_done);  // arrives once every MMA issued above has completed
            mbar_wait_bounded(mma_done, 0, a.status, 66u);
        }
    } else if (warp < 10) {
        // ---------------- loaders: warp (quarter qd, K step sub) ----------------
        const uint32_t qd = warp & 3u;                  // TMEM lane quarter
        const uint32_t sub = (warp - 2u) >> 2;          // which K step of each unit
        const uint32_t m = qd * 32u + lane;             // MMA row: 16 * phase + tile row
        const uint32_t p = m >> 4, r = m & 15u;
        bool ok = true;
        uint32_t slot = 0, sph = 0, ab = 0, aph = 0, uk = 0;
        for (uint32_t u = 0; u < total && ok; ++u) {
            const uint32_t half = uk & 1u;  // which unit of the slot
            if (half == 0) ok = wait_phase(&ring_full[slot], sph, abort_flag, a.status, 67u);
            if (ok && u >= kNA) ok = wait_phase(&a_free[ab], aph ^ 1u, abort_flag, a.status, 68u);
            if (!ok) break;
            tc_fence_after();  // the MMAs that read this A buffer have completed
            if (uk * kUnitSteps + sub < a.steps) {
                const uint8_t* row = smem + slot * kSlotBytes + r * kPitch + half * (kUnitBlocks * BB);
                const uint32_t off = (sub * kPhases + p) * BB;  // this lane's block in the unit row
                const float dv = half_bits_to_float(*reinterpret_cast<const uint16_t*>(row + off));
                const uint32_t qs = off + 2u;                  // first quant byte
                const uint32_t* w = reinterpret_cast<const uint32_t*>(row + (qs & ~3u));
                const uint32_t sh = (qs & 3u) * 8u;            // 0 or 16
                uint32_t av[8];
                if constexpr (TYPE == kQ8_0) {
                    uint32_t wv[9];
#pragma unroll
                    for (uint32_t k = 0; k < 9; ++k) wv[k] = w[k];
#pragma unroll
                    for (uint32_t k = 0; k < 8; ++k) av[k] = __funnelshift_r(wv[k], wv[k + 1], sh);
                } else {
                    uint32_t wv[5];
#pragma unroll
                    for (uint32_t k = 0; k < 5; ++k) wv[k] = w[k];
#pragma unroll
                    for (uint32_t k = 0; k < 4; ++k) {
                        const uint32_t n = __funnelshift_r(wv[k], wv[k + 1], sh);
                        av[k] = n & 0x0F0F0F0Fu;              // elements 4k..4k+3: low nibbles
                        av[4u + k] = (n >> 4) & 0x0F0F0F0Fu;  // elements 16+4k..: high nibbles
                    }
                }
                tc_st_x8(tmem + kACol0 + ab * 16u + sub * 8u + ((qd * 32u) << 16), av);
                sd[(ab * kUnitSteps + sub) * 128u + m] = dv;
                asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            }
            tc_fence_before();
            __syncwarp();
            const bool slot_done = half == 1u || uk + 1u == units;
            if (lane == 0) {
                mbar_arrive(&ring_empty[slot]);
                if (slot_done && half == 0u) mbar_arrive(&ring_empty[slot]);  // a slot of one unit
                mbar_arrive(&a_full[ab]);
            }
            if (slot_done && ++slot == S) {
                slot = 0;
                sph ^= 1u;
            }
            if (++uk == units) uk = 0;
            if (++ab == kNA) {
                ab = 0;
                aph ^= 1u;
            }
        }
    } else {
        // ---------------- x table, then the epilogue: warp (quarter qd, K step sub) ----------------
        const uint32_t qd = warp & 3u;
        const uint32_t sub = (warp - 10u) >> 2;
        const uint32_t et = threadIdx.x - 320u;  // 0..255
        grid_dependency_wait();                  // x may come from the previous kernel
        {
            // 8 threads per block, 32 blocks per pass, up to 4 passes' loads in flight
            const uint32_t q = et & 7u;
            const uint32_t nbt = a.steps * kPhases;  // a.nb rounded up to whole K steps (== a.nb)
            for (uint32_t base = 0; base < nbt; base += 128u) {
                float4 v[4];
#pragma unroll
                for (uint32_t k = 0; k < 4; ++k) {
                    const uint32_t b = base + k * 32u + (et >> 3);
                    v[k] = b < a.nb ? __ldg(reinterpret_cast<const float4*>(a.x + 32u * b + 4u * q))
                                    : make_float4(0.f, 0.f, 0.f, 0.f);
                }
#pragma unroll
                for (uint32_t k = 0; k < 4; ++k) {
                    const uint32_t b = base + k * 32u + (et >> 3);
                    // every lane runs the block code (its shuffles span the warp);
                    // blocks past the row store nothing
                    if (base + k * 32u < nbt) limb_block<TYPE == kQ4_0>(v[k], b, q, b < nbt, table, consts);
                }
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // table writes -> tensor-core reads
            __syncwarp();
            if (lane == 0) mbar_arrive(table_full);
        }
        const uint32_t m = qd * 32u + lane;
        const uint32_t p = m >> 4;
        const uint32_t hi = lane >> 4;  // which 4 of the 8 loaded columns are this lane's
        bool ok = true;
        float acc = 0.f;
        // every thread of the epilogue sees the table (its own warp group wrote it)
        named_barrier_sync(1, 256);
        uint32_t ab = 0, aph = 0, db = 0, dph = 0, uk = 0, t = 0;
        for (uint32_t u = 0; u < total && ok; ++u) {
            ok = wait_phase(&d_full[db], dph, abort_flag, a.status, 69u);
            // the loaders' block scales of this unit (their arrival orders the sd stores)
            ok = ok && wait_phase(&a_full[ab], aph, abort_flag, a.status, 70u);
            if (!ok) break;
            tc_fence_after();
            const uint32_t s = uk * kUnitSteps + sub;
            uint32_t v[8];
            float dv = 0.f;
            if (s < a.steps) {
                tc_ld_x8(tmem + kDCol0 + db * (kUnitSteps * kN) + sub * kN + qd * 8u + ((qd * 32u) << 16), v);
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                dv = sd[(ab * kUnitSteps + sub) * 128u + m];
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&d_free[db]);
                mbar_arrive(&a_free[ab]);
            }
            if (s < a.steps) {
                const float4 c = consts[s * kPhases + p];
                const int d0 = static_cast<int>(hi ? v[4] : v[0]);
                const int d1 = static_cast<int>(hi ? v[5] : v[1]);
                const int d2 = static_cast<int>(hi ? v[6] : v[2]);
                const int d3 = static_cast<int>(hi ? v[7] : v[3]);
                const int vh = d0 * 128 + d1 - __float_as_int(c.z);
                const int vl = d2 * 128 + d3 - __float_as_int(c.w);
                acc = fmaf(static_cast<float>(vh), dv * c.x, acc);
                acc = fmaf(static_cast<float>(vl), dv * c.y, acc);
            }
            if (++ab == kNA) {
                ab = 0;
                aph ^= 1u;
            }
            if (++db == kND) {
                db = 0;
                dph ^= 1u;
            }
            if (++uk == units) {
                uk = 0;
                // tile done: add each row's 16 partial sums (8 block phases x 2 K-step
                // warps) in a fixed order.  Two buffers by tile parity; a buffer is
                // rewritten only after the sum of the tile two before was read from it.
                const float pair = acc + __shfl_xor_sync(0xFFFFFFFFu, acc, 16);  // phases 2qd, 2qd+1
                const uint32_t rbi = t & 1u;
                float* rb = red + rbi * 128u;
                if (t >= 2u && !wait_phase(&red_free[rbi], ((t >> 1) - 1u) & 1u, abort_flag, a.status, 71u)) {
                    ok = false;
                    break;
                }
                if (lane < 16) rb[(sub * 4u + qd) * 16u + lane] = pair;
                __syncwarp();
                if (lane == 0) mbar_arrive(&red_full[rbi]);
                if (qd == 0 && sub == 0) {
                    if (!wait_phase(&red_full[rbi], (t >> 1) & 1u, abort_flag, a.status, 72u)) {
                        ok = false;
                        break;
                    }
                    if (lane < 16) {
                        float yv = 0.f;
#pragma unroll
                        for (uint32_t k = 0; k < 8; ++k) yv += rb[k * 16u + lane];
                        const uint32_t row = (tile_begin + t) * kTileRows + lane;
                        if (row < a.rows) a.y[row] = yv;
                    }
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&red_free[rbi]);
                }
                acc = 0.f;
                ++t;
            }
        }
    }
    __syncwarp();
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
    }
}

}  // namespace

Tc8Plan plan_tc8(uint32_t type, uint64_t rows, uint64_t cols, int num_sms, int max_smem_optin) {
    Tc8Plan p;
    if (type != kQ8_0 && type != kQ4_0) return p;
    // whole K steps of 8 blocks (the tensor map's row stride is then a multiple of
    // 16 bytes), at most kMaxSteps of them (the x table), int32 coordinates
    if (cols % 256u || cols / 256u > kMaxSteps || rows == 0 || rows >= 0x7FFFFFF0ull || num_sms <= 0) return p;
    const uint32_t bb = type == kQ8_0 ? 34u : 18u;
    const uint32_t nb = static_cast<uint32_t>(cols / 32u);
    const uint32_t steps = nb / kPhases;
    const uint32_t units = (steps + kUnitSteps - 1) / kUnitSteps;
    // a ring slot (one copy) is 16 rows x 32 blocks; a row in shared memory is its
    // blocks plus 16 bytes, an odd multiple of 16 bytes, so the 16 rows of a loader
    // read fall in different bank groups (the copy reads 16 bytes of the next
    // slot's blocks, or zeros past the row end)
    const uint32_t unit_bytes = kTileRows * (kSlotUnits * kUnitBlocks * bb + 16u);
    const uint32_t spt = (units + kSlotUnits - 1) / kSlotUnits;
    const uint64_t tiles = (rows + kTileRows - 1) / kTileRows;
    const uint64_t grid = tiles < static_cast<uint64_t>(num_sms) ? tiles : static_cast<uint64_t>(num_sms);
    const uint64_t per_cta = (tiles + grid - 1) / grid * spt;  // copies of the busiest CTA
    // fixed part: x table, block constants, block scales, partial sums
    const uint32_t off_table_rel = 0;
    const uint32_t table = steps * kStepTableBytes;
    const uint32_t cbytes = steps * kPhases * 16u;
    const uint32_t sdb = kNA * kUnitSteps * 128u * 4u;
    const uint32_t redb = 2u * 128u * 4u;
    auto smem_of = [&](uint32_t s) {
        const uint32_t bars = 8u * (2u * s + 2u * kNA + 2u * kND + 6u) + 16u;
        return s * unit_bytes + table + cbytes + sdb + redb + bars + off_table_rel;
    };
    uint32_t slots = per_cta < kMaxSlots ? static_cast<uint32_t>(per_cta) : kMaxSlots;
    if (slots < 2) slots = 2;
    const uint32_t budget = kBudget < static_cast<uint32_t>(max_smem_optin) ? kBudget : max_smem_optin;
    while (slots > 2 && smem_of(slots) > budget) --slots;
    if (smem_of(slots) > budget) return p;
    p.type = type;
    p.rows = rows;
    p.cols = cols;
    p.grid = static_cast<uint32_t>(grid);
    p.threads = kThreads;
    p.slots = slots;
    p.unit_bytes = unit_bytes;
    p.tiles = static_cast<uint32_t>(tiles);
    p.steps = steps;
    p.units = units;
    p.off_table = slots * unit_bytes;
    p.off_consts = p.off_table + table;
    p.off_sd = p.off_consts + cbytes;
    p.off_red = p.off_sd + sdb;
    p.off_bars = p.off_red + redb;
    // at least 77 KB: never three CTAs on an SM (each holds 256 of its 512 TMEM columns)
    const uint32_t need = smem_of(slots);
    p.smem_bytes = need < 77u * 1024u ? 77u * 1024u : need;
    p.ok = true;
    return p;
}

cudaError_t launch_tc8(const Tc8Plan& plan, const void* w, const float* x, float* y, DeviceStatus* status,
                       cudaStream_t stream, bool pdl) {
    if (!plan.ok || (reinterpret_cast<uintptr_t>(w) & 15u) != 0 || (reinterpret_cast<uintptr_t>(x) & 15u) != 0)
        return cudaErrorInvalidValue;
    const uint64_t rb = row_bytes_of(plan.type, plan.cols);
    EncodeTiled enc = encode_tiled_fn();
    if (enc == nullptr) return cudaErrorNotSupported;
    // the weight as rows of 8-byte elements; a box is 16 rows x one unit (16 blocks)
    CUtensorMap map;
    const cuuint64_t dims[2] = {rb / 8u, plan.rows}, strides[1] = {rb};
    const cuuint32_t box[2] = {plan.unit_bytes / kTileRows / 8u, kTileRows}, es[2] = {1, 1};
    if (enc(&map, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<void*>(w), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return cudaErrorInvalidValue;
    Tc8Args a{};
    a.x = x;
    a.y = y;
    a.rows = static_cast<uint32_t>(plan.rows);
    a.tiles = plan.tiles;
    a.nb = static_cast<uint32_t>(plan.cols / 32u);
    a.steps = plan.steps;
    a.units = plan.units;
    a.slots = plan.slots;
    a.off_table = plan.off_table;
    a.off_consts = plan.off_consts;
    a.off_sd = plan.off_sd;
    a.off_red = plan.off_red;
    a.off_bars = plan.off_bars;
    a.status = status;
    static bool configured[2][64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    const int ti = plan.type == kQ8_0 ? 0 : 1;
    auto kern = plan.type == kQ8_0 ? gemv_tc8_kernel<kQ8_0> : gemv_tc8_kernel<kQ4_0>;
    if (dev < 64 && !configured[ti][dev]) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
        if (e != cudaSuccess) return e;
        configured[ti][dev] = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(plan.grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = plan.smem_bytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, map, a);
}

}  // namespace nedo_gpu
