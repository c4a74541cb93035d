// gemm_tc.cu -- batched matvec (prefill-shaped GEMM) on the 5th-generation
// tensor cores: Y[t][r] = sum_k W[r][k] * X[t][k] for a GGUF weight W
// (rows x cols) and T token vectors X (fp32).
//
// The reference has no batched product: a prompt is a loop of single-vector
// matvecs (src/model.cpp:262-266), each y[r] = dot(row r, x)
// (src/kernels.cpp:162-169).  Here the tokens become the N dimension of one
// tcgen05 contraction per 128-row weight tile:
//
//   * A CTA owns 256 weight rows x 256 tokens: two M=128 MMAs per K step share
//     the token tile, with both fp32 accumulators in TMEM (2 x 256 columns).
//     Fewer, larger tiles halve the operand bytes each SM pulls through L2 per
//     FLOP compared with 128-row tiles.
//   * W stays in GGUF block layout in HBM.  A TMA tensor map over the row bytes
//     (uint16 elements) brings 256 rows x 128 elements of raw blocks into shared
//     memory; the box starts at the 16-byte boundary at or below the chunk (8
//     bytes early for odd chunks).  Eight dequant warps, one thread per row, turn
//     each block into fp16 d*q (exact in fp32, rounded once) and write the A
//     tiles in the 64-byte-swizzled K-major layout.  F16 weights load straight
//     into that layout with a swizzled tensor map.
//   * X is converted once to fp16 (round to nearest) and loaded per stage with a
//     swizzled tensor map as the B operand (256 tokens x 32 K).
//   * One thread issues tcgen05.mma kind::f16 (M=128, N=256, K=16);
//     tcgen05.commit releases each stage.  The dequant warps then read TMEM
//     (tcgen05.ld 32x32b) and store Y.
//
//   * Quantised weights with more than 256 tokens (and no K split) run on CTA
//     pairs instead (gemm_tc_pair_kernel): tcgen05.mma.cta_group::2 with
//     M = 256 across the pair and each SM holding half of every token tile,
//     which cuts the shared-memory bytes per MMA that bound the one-SM tile.
//
// fp16 rounding of x and of d*q is the only difference from the reference's
// fp32 arithmetic (relative 2^-11 per factor); the products are summed in fp32.
// Every wait is bounded; TMEM is released on every path.
#include <cuda.h>
#include <math.h>

#include <mutex>

#include "common.cuh"
#include "launch.h"

namespace nedo_gpu {
namespace {

constexpr uint32_t kBM = 128;           // weight rows per MMA (M, TMEM lanes)
constexpr uint32_t kHalves = 2;         // MMAs per K step: a CTA covers 256 weight rows
constexpr uint32_t kRows = kBM * kHalves;
constexpr uint32_t kBN = 256;           // tokens per tile (MMA N; TMEM columns per accumulator)
constexpr uint32_t kBK = 32;            // K per stage: one 64-byte fp16 row of a swizzle atom
constexpr uint32_t kRawK = 128;         // K per raw weight chunk: 4 GGUF blocks
// A/B stages: 32 KB each; quantised weights also need two raw chunk slots
template <uint32_t TYPE>
constexpr uint32_t stages() {
    return TYPE == kF16 ? 6u : 4u;
}
// X-tile stages: one more than the A stages for quantised weights (the X tiles
// come from L2 and need the longer lead; the A tiles wait for the dequant warps
// anyway); F16 loads A and X into the same stages.
template <uint32_t TYPE>
constexpr uint32_t stages_b() {
    return TYPE == kF16 ? stages<TYPE>() : stages<TYPE>() + 1u;
}
constexpr uint32_t kRawSlots = 2;
constexpr uint32_t kDeqWarps = 8;     // warps 2..9: dequant, then epilogue
constexpr uint32_t kThreads = (2 + kDeqWarps) * 32;
constexpr uint32_t kStageA = kRows * 64;  // 16 KB: two 8 KB halves of 128 rows
constexpr uint32_t kStageB = kBN * 64;    // 16 KB

__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

template <uint32_t TYPE>
struct RawBlock;
template <>
struct RawBlock<kQ8_0> {
    static constexpr uint32_t kBytes = 34;
};
template <>
struct RawBlock<kQ4_0> {
    static constexpr uint32_t kBytes = 18;
};
template <>
struct RawBlock<kF16> {  // F16 rows load straight into the A tiles (no raw chunk)
    static constexpr uint32_t kBytes = 64;
};
// Bytes of one row of a raw chunk in shared memory: the chunk's kRawK / 32
// blocks plus 8 bytes, because the box starts at the 16-byte boundary at or
// below the chunk (4 * 34 and 4 * 18 are 8 mod 16: odd chunks start 8 bytes in).
template <uint32_t TYPE>
constexpr uint32_t raw_row_bytes() {
    return kRawK / 32u * RawBlock<TYPE>::kBytes + 8u;
}

struct GemmArgs {
    float* y;              // [tokens][ldy]; split z writes y + z * split_stride
    uint32_t rows;         // N of the weight (output features)
    uint32_t cols;         // K
    uint32_t tokens;
    uint32_t ldy;
    uint32_t ksplit;       // CTAs along K per tile (gridDim.z): each sums a range of raw chunks
    uint64_t split_stride;
    DeviceStatus* status;
};

// ---- PTX wrappers -------------------------------------------------------
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int32_t c0, int32_t c1,
                                            uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
            "r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_addr(bar))
        : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tc_mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                           uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
                 : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread i gets lane (base + i).
__device__ __forceinline__ void tc_ld_32x32b_x32(uint32_t taddr, uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
          "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
          "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor: K-major, 64-byte swizzle, 8-row atoms of
// 512 bytes (SBO), version 1 (sm_100).  Tile bases are 1024-byte aligned.
__device__ __forceinline__ uint64_t sw64_desc(uint32_t saddr) {
    uint64_t d = static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>(1u) << 16;           // LBO (unused by swizzled K-major)
    d |= static_cast<uint64_t>(512u >> 4) << 32;    // SBO: 8 rows x 64 bytes
    d |= static_cast<uint64_t>(1u) << 46;           // descriptor version for sm_100
    d |= static_cast<uint64_t>(4u) << 61;           // SWIZZLE_64B
    return d;
}

// kind::f16 instruction descriptor: A, B fp16, D fp32, both K-major, M = 128 x N
// (N a multiple of 16, 16..256).
__host__ __device__ constexpr uint32_t idesc_m128(uint32_t n) { return (1u << 4) | ((n >> 3) << 17) | ((kBM >> 4) << 24); }

// fp16 tile element (row r, 16-byte chunk c of its 64-byte row) in the
// 64-byte-swizzled K-major layout: byte-address bits 4-5 are XORed with bits
// 7-8, so chunk c of row r lands at c ^ ((r / 2) % 4).
__device__ __forceinline__ uint32_t sw64_offset(uint32_t r, uint32_t c) {
    return (r >> 3) * 512u + (r & 7u) * 64u + ((c ^ ((r >> 1) & 3u)) << 4);
}

__device__ __forceinline__ void sts128(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

__device__ __forceinline__ uint4 lds128(uint32_t addr) {
    uint4 v;
    asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
    return v;
}

// Dequantise block BLK (0..3) of row r of a raw chunk (SKEW: 0 or 8 bytes of
// the previous chunk before it) into row r of an A half-tile: the 32 elements
// of one K stage.  All offsets are compile-time; the block's bytes come from
// 16-byte aligned loads.
template <uint32_t TYPE, uint32_t SKEW, uint32_t BLK>
__device__ __forceinline__ void dequant_block(uint32_t raw_row, uint32_t a_half, uint32_t r) {
    constexpr uint32_t BB = RawBlock<TYPE>::kBytes;
    constexpr uint32_t start = SKEW + BLK * BB;    // block offset in the raw row
    constexpr uint32_t base = start & ~15u;        // 16-byte aligned window
    constexpr uint32_t off = start - base;         // 0..14, even
    constexpr uint32_t nchunks = (off + BB + 15u) / 16u;  // 2 (Q4_0) or 3 (Q8_0)
    uint32_t w[12];
#pragma unroll
    for (uint32_t c = 0; c < 3; ++c) {
        if (c < nchunks) {
            const uint4 v = lds128(raw_row + base + 16u * c);
            w[4 * c] = v.x;
            w[4 * c + 1] = v.y;
            w[4 * c + 2] = v.z;
            w[4 * c + 3] = v.w;
        } else {
            w[4 * c] = w[4 * c + 1] = w[4 * c + 2] = w[4 * c + 3] = 0u;
        }
    }
    // byte i of the block is byte (off + i) of the window.  Two quants become an
    // fp16 pair without int->float conversions: PRMT gathers their bytes into
    // the low bytes of the two halves, LOP3 puts them under the exponent of
    // 1024 (fp16 0x6400 + u = 1024 + u, exact for u < 1024), HSUB2 removes the
    // bias exactly, and HMUL2 by d rounds d*q once (as __float2half_rn(d*q)).
    // bytes i, i+1 of the block -> bytes 0 and 2 of the result (bytes 1, 3: don't care)
    auto pair_bytes = [&](uint32_t i) -> uint32_t {
        const uint32_t k = off + i, wi = k >> 2, bi = k & 3u;
        // PRMT's 8-byte window: w[wi] = bytes 0..3, w[wi+1] = bytes 4..7
        return prmt(w[wi], w[wi + 1u < 12u ? wi + 1u : 11u], bi | ((bi + 1u) << 8));
    };
    const uint32_t dbits = pair_bytes(0);
    const __half dh = __ushort_as_half(static_cast<unsigned short>((dbits & 0xFFu) | ((dbits >> 8) & 0xFF00u)));
    const __half2 d2 = __halves2half2(dh, dh);
#pragma unroll
    for (uint32_t c = 0; c < 4; ++c) {  // 8 elements per 16-byte output chunk
        uint32_t h[4];
#pragma unroll
        for (uint32_t e = 0; e < 4; ++e) {
            const uint32_t el = 8u * c + 2u * e;  // elements el, el+1 of the block
            __half2 q;
            if constexpr (TYPE == kQ8_0) {
                // int8 q: (q ^ 0x80) = q + 128 under the 1024 exponent, minus 1152
                const uint32_t v = lop_and_xor(pair_bytes(2u + el), 0x00FF00FFu, 0x64806480u);
                q = __hsub2(*reinterpret_cast<const __half2*>(&v), __float2half2_rn(1152.0f));
            } else {
                // Q4_0: elements j < 16 are the low nibbles of bytes j, elements
                // j + 16 the high nibbles; value nibble - 8
                const uint32_t j = el & 15u;
                uint32_t v = pair_bytes(2u + j);
                if (el >= 16u) v >>= 4;
                v = lop_and_or(v, 0x000F000Fu, 0x64006400u);
                q = __hsub2(*reinterpret_cast<const __half2*>(&v), __float2half2_rn(1032.0f));
            }
            const __half2 p = __hmul2(q, d2);
            h[e] = *reinterpret_cast<const uint32_t*>(&p);
        }
        sts128(a_half + sw64_offset(r, c), h[0], h[1], h[2], h[3]);
    }
}

template <uint32_t I>
struct Idx {
    static constexpr uint32_t value = I;
};

// x (fp32, tokens x cols) -> fp16 (round to nearest), same layout.
__global__ void x_to_f16_kernel(const float* __restrict__ x, __half* __restrict__ xh, uint64_t n) {
    // the GEMM that reads xh may launch now: it streams its weights until this grid completes
    asm volatile("griddepcontrol.launch_dependents;");
    // launched early itself: x may come from, and xh is read by, the kernels before
    asm volatile("griddepcontrol.wait;" ::: "memory");
    for (uint64_t i = (blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x) * 4u; i < n;
         i += static_cast<uint64_t>(gridDim.x) * blockDim.x * 4u) {
        if (i + 4u <= n) {
            const float4 v = *reinterpret_cast<const float4*>(x + i);
            *reinterpret_cast<__half2*>(xh + i) = __floats2half2_rn(v.x, v.y);
            *reinterpret_cast<__half2*>(xh + i + 2) = __floats2half2_rn(v.z, v.w);
        } else {
            for (uint64_t k = i; k < n; ++k) xh[k] = __float2half_rn(x[k]);
        }
    }
}

template <uint32_t TYPE>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_x,
                   const GemmArgs a) {
    extern __shared__ uint8_t smem_raw[];
    // 1024-byte aligned base for the swizzled tiles
    const uint32_t s0 = (smem_addr(smem_raw) + 1023u) & ~1023u;
    uint8_t* const sbase = smem_raw + (s0 - smem_addr(smem_raw));
    constexpr bool kRawW = TYPE != kF16;
    constexpr uint32_t kS = stages<TYPE>();
    constexpr uint32_t kSB = stages_b<TYPE>();
    constexpr uint32_t kRawBytes = kRawW ? kRows * raw_row_bytes<TYPE>() : 0u;
    const uint32_t sA = s0;                       // kS x 16 KB (two 128-row halves)
    const uint32_t sB = sA + kS * kStageA;        // kSB x 16 KB
    const uint32_t sRaw = sB + kSB * kStageB;     // kRawSlots x raw chunk
    uint64_t* bars = reinterpret_cast<uint64_t*>(sbase + (sRaw - s0) + kRawSlots * kRawBytes);
    uint64_t* b_full = bars;                  // [kSB] X (and F16 W) tiles landed
    uint64_t* a_full = b_full + kSB;          // [kS] A tile written by the dequant warps
    uint64_t* ab_empty = a_full + kS;         // [kS] MMAs of the A stage (F16: the stage) done
    uint64_t* b_empty = ab_empty + kS;        // [kSB] MMAs of the X stage done (quantised weights)
    uint64_t* raw_full = b_empty + kSB;       // [kRawSlots]
    uint64_t* raw_empty = raw_full + kRawSlots;
    uint64_t* done = raw_empty + kRawSlots;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);

    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t row0 = blockIdx.x * kRows;  // weight rows of this tile
    const uint32_t tok0 = blockIdx.y * kBN;   // tokens of this tile
    const uint32_t ksteps = (a.cols + kBK - 1) / kBK;
    const uint32_t chunks = (a.cols + kRawK - 1) / kRawK;
    // this CTA's share of K: raw chunks [kc_begin, kc_end), k-steps [ks_begin, ks_end)
    const uint32_t kc_begin = static_cast<uint32_t>(static_cast<uint64_t>(chunks) * blockIdx.z / a.ksplit);
    const uint32_t kc_end = static_cast<uint32_t>(static_cast<uint64_t>(chunks) * (blockIdx.z + 1) / a.ksplit);
    const uint32_t ks_begin = kc_begin * (kRawK / kBK);
    const uint32_t ks_end = kc_end * (kRawK / kBK) < ksteps ? kc_end * (kRawK / kBK) : ksteps;
    float* const y = a.y + blockIdx.z * a.split_stride;

    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < kS; ++s) {
            mbar_init(&a_full[s], kRawW ? kDeqWarps : 1u);
            mbar_init(&ab_empty[s], 1);
        }
        for (uint32_t s = 0; s < kSB; ++s) {
            mbar_init(&b_full[s], 1);
            mbar_init(&b_empty[s], 1);
        }
        for (uint32_t s = 0; s < kRawSlots; ++s) {
            mbar_init(&raw_full[s], 1);
            mbar_init(&raw_empty[s], kDeqWarps);
        }
        mbar_init(done, 1);
        fence_barrier_init();
    }
    if (warp == 1) {  // TMEM: two accumulators of kBN fp32 columns x 128 lanes
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                     "r"(kHalves * kBN));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    // every warp arrives converged: a CTA barrier counts a warp whose first
    // lanes arrive while another lane still works as arrived
    __syncwarp();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_d = *tmem_slot;
    // the kernel after this one (the split-K fold, or the next conversion of x)
    // may be scheduled now; it waits for this grid's completion before its work
    if (threadIdx.x == 0) asm volatile("griddepcontrol.launch_dependents;");

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            uint32_t issued_ks = 0, issued_kc = 0;
            bool ok = true;
            // raw weight chunk kc into its slot (the weights are not written by the
            // previous kernel, so the first slots fill before its completion)
            auto load_raw = [&](uint32_t kc) {
                const uint32_t rs = (kc - kc_begin) % kRawSlots;
                mbar_arrive_expect_tx(&raw_full[rs], kRawBytes);
                // the chunk's first byte, rounded down to 16 bytes (uint16 elements)
                const uint32_t first = kc * (kRawK / 32u) * RawBlock<TYPE>::kBytes;
                tma_load_2d(sRaw + rs * kRawBytes, &map_w, static_cast<int32_t>((first & ~15u) / 2u),
                            static_cast<int32_t>(row0), &raw_full[rs]);
                issued_kc = kc - kc_begin + 1u;  // local count
            };
            if constexpr (kRawW)
                for (uint32_t kc = kc_begin; kc < kc_begin + kRawSlots && kc < kc_end; ++kc) load_raw(kc);
            grid_dependency_wait();  // X may come from the previous kernel
            for (uint32_t kc = kc_begin; kc < kc_end && ok; ++kc) {
                if constexpr (kRawW) {
                    const uint32_t lc = kc - kc_begin;  // local chunk index: slot and phase
                    const uint32_t rs = lc % kRawSlots;
                    if (lc >= kRawSlots) {
                        if (!mbar_wait_bounded(&raw_empty[rs], ((lc / kRawSlots) - 1u) & 1u, a.status, 31u)) {
                            ok = false;
                            break;
                        }
                        load_raw(kc);
                    }
                }
                for (uint32_t j = 0; j < kRawK / kBK; ++j) {
                    const uint32_t ks = kc * (kRawK / kBK) + j;
                    if (ks >= ks_end) break;
                    const uint32_t ls = ks - ks_begin;  // local k-step: stage and phase
                    const uint32_t sb = ls % kSB;       // F16: kSB == kS, the stage of A and X
                    uint64_t* freed = kRawW ? &b_empty[sb] : &ab_empty[sb];
                    if (ls >= kSB && !mbar_wait_bounded(freed, ((ls / kSB) - 1u) & 1u, a.status, 32u)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&b_full[sb], kStageB + (kRawW ? 0u : kStageA));
                    tma_load_2d(sB + sb * kStageB, &map_x, static_cast<int32_t>(ks * kBK),
                                static_cast<int32_t>(tok0), &b_full[sb]);
                    if constexpr (!kRawW)
                        tma_load_2d(sA + sb * kStageA, &map_w, static_cast<int32_t>(ks * kBK),
                                    static_cast<int32_t>(row0), &b_full[sb]);
                    issued_ks = ls + 1u;
                }
            }
            // drain: the last copies issued into every slot have landed before exit
            for (uint32_t k = issued_ks > kSB ? issued_ks - kSB : 0u; k < issued_ks; ++k)
                mbar_wait_bounded(&b_full[k % kSB], (k / kSB) & 1u, a.status, 38u);
            for (uint32_t k = issued_kc > kRawSlots ? issued_kc - kRawSlots : 0u; k < issued_kc; ++k)
                mbar_wait_bounded(&raw_full[k % kRawSlots], (k / kRawSlots) & 1u, a.status, 39u);
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            bool ok = true;
            // MMA N: the tile's tokens rounded up to 16 (a batch of 32 computes 32
            // accumulator columns, not 256; the epilogue never reads past them)
            const uint32_t ntok = a.tokens - tok0 < kBN ? a.tokens - tok0 : kBN;
            const uint32_t idesc = idesc_m128((ntok + 15u) & ~15u);
            for (uint32_t ls = 0; ls < ks_end - ks_begin && ok; ++ls) {
                const uint32_t s = ls % kS, ph = (ls / kS) & 1u;
                const uint32_t sb = ls % kSB, phb = (ls / kSB) & 1u;
                ok = mbar_wait_bounded(&b_full[sb], phb, a.status, 33u);
                if constexpr (kRawW) ok = ok && mbar_wait_bounded(&a_full[s], ph, a.status, 34u);
                if (!ok) break;
                tc_fence_after();
                const uint64_t bd = sw64_desc(sB + sb * kStageB);
#pragma unroll
                for (uint32_t h = 0; h < kHalves; ++h) {
                    const uint64_t ad = sw64_desc(sA + s * kStageA + h * (kBM * 64u));
#pragma unroll
                    for (uint32_t kk = 0; kk < kBK / 16u; ++kk)  // K = 16 per MMA: 32 bytes along the row
                        tc_mma_f16(tmem_d + h * kBN, ad + 2u * kk, bd + 2u * kk, idesc, (ls | kk) != 0u);
                }
                tc_commit(&ab_empty[s]);
                if constexpr (kRawW) tc_commit(&b_empty[sb]);
            }
            tc_commit(done);  // every MMA issued above has completed when this arrives
        }
    } else {
        // ---------------- dequant warps, then epilogue ----------------
        const uint32_t r = threadIdx.x - 64u;    // tile row 0..255: one row per thread
        const uint32_t half = r / kBM;           // which MMA half-tile the row belongs to
        if constexpr (kRawW) {
            bool ok = true;
            for (uint32_t kc = kc_begin; kc < kc_end && ok; ++kc) {
                const uint32_t lc = kc - kc_begin;
                const uint32_t rs = lc % kRawSlots;
                if (!mbar_wait_bounded(&raw_full[rs], (lc / kRawSlots) & 1u, a.status, 35u)) {
                    ok = false;
                    break;
                }
                const uint32_t raw_row = sRaw + rs * kRawBytes + r * raw_row_bytes<TYPE>();
                // the chunk's 4 stages; stage J holds block J of every row
                auto stage = [&](auto J) {
                    constexpr uint32_t j = decltype(J)::value;
                    const uint32_t ks = kc * (kRawK / kBK) + j;
                    if (!ok || ks >= ks_end) return;
                    const uint32_t ls = ks - ks_begin;
                    const uint32_t s = ls % kS;
                    if (ls >= kS && !mbar_wait_bounded(&ab_empty[s], ((ls / kS) - 1u) & 1u, a.status, 36u)) {
                        ok = false;
                        return;
                    }
                    const uint32_t a_half = sA + s * kStageA + half * (kBM * 64u);
                    if (kc & 1u)  // odd chunks start 8 bytes into the loaded row
                        dequant_block<TYPE, 8u, j>(raw_row, a_half, r & (kBM - 1u));
                    else
                        dequant_block<TYPE, 0u, j>(raw_row, a_half, r & (kBM - 1u));
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic writes -> tensor core reads
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&a_full[s]);
                };
                stage(Idx<0>{});
                stage(Idx<1>{});
                stage(Idx<2>{});
                stage(Idx<3>{});
                __syncwarp();
                if (lane == 0) mbar_arrive(&raw_empty[rs]);
            }
        }
        // epilogue: warps 2..5 read accumulator 0 (rows 0..127), warps 6..9
        // accumulator 1 (rows 128..255), each its TMEM lane quarter, all tokens
        const uint32_t quarter = warp & 3u;
        const uint32_t acc = (warp - 2u) >> 2;
        if (mbar_wait_bounded(done, 0, a.status, 37u)) {
            tc_fence_after();
            const uint32_t wrow = row0 + acc * kBM + quarter * 32u + lane;
            for (uint32_t col = 0; col < kBN; col += 32u) {
                uint32_t v[32];
                tc_ld_32x32b_x32(tmem_d + acc * kBN + ((quarter * 32u) << 16) + col, v);
                if (wrow < a.rows) {
#pragma unroll
                    for (uint32_t i = 0; i < 32; ++i) {
                        const uint32_t t = tok0 + col + i;
                        if (t < a.tokens) y[static_cast<size_t>(t) * a.ldy + wrow] = __uint_as_float(v[i]);
                    }
                }
            }
        }
    }
    // lanes 1..31 of the producer and MMA warps wait here for lane 0, so the
    // barrier below holds until every warp (the epilogue included) is done
    __syncwarp();
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_d), "r"(kHalves * kBN));
    }
}

// Split-K fold: y[t][r] = sum over z (in z order) of ws[z][t][r].  ws is written
// by the GEMM launched just before, so the fold waits for that kernel first.
__global__ void splitk_reduce_kernel(const float* __restrict__ ws, float* __restrict__ y, uint32_t splits,
                                     uint32_t tokens, uint32_t rows, uint64_t ldy) {
    asm volatile("griddepcontrol.launch_dependents;");  // the next kernel may be scheduled
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const uint64_t n = static_cast<uint64_t>(tokens) * rows;
    const uint64_t zstride = n;
    for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        // eight splits' loads in flight at a time, added in split order
        float v = __ldg(ws + i);
        uint32_t z = 1;
        for (; z + 8u <= splits; z += 8u) {
            float p[8];
#pragma unroll
            for (uint32_t k = 0; k < 8; ++k) p[k] = __ldg(ws + (z + k) * zstride + i);
#pragma unroll
            for (uint32_t k = 0; k < 8; ++k) v += p[k];
        }
        for (; z < splits; ++z) v += __ldg(ws + z * zstride + i);
        const uint64_t t = i / rows, r = i - t * rows;
        y[t * ldy + r] = v;
    }
}

// ---- host side ----------------------------------------------------------
template <uint32_t TYPE>
cudaError_t launch_t(const void* w, const __half* xh, float* y, uint32_t rows, uint32_t cols, uint32_t tokens,
                     uint32_t ldy, uint32_t ksplit, uint64_t split_stride, DeviceStatus* status, cudaStream_t stream,
                     bool pdl) {
    EncodeTiled enc = encode_tiled_fn();
    if (enc == nullptr) return cudaErrorNotSupported;
    CUtensorMap mw, mx;
    const uint64_t rb = row_bytes_of(TYPE, cols);
    if (TYPE == kF16) {
        const cuuint64_t dims[2] = {cols, rows}, strides[1] = {rb};
        const cuuint32_t box[2] = {kBK, kRows}, es[2] = {1, 1};
        if (enc(&mw, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(w), dims, strides, box, es,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return cudaErrorInvalidValue;
    } else {
        // raw rows as uint16 elements: a 256-element chunk is raw_row_bytes/2 of them
        const cuuint64_t dims[2] = {rb / 2u, rows}, strides[1] = {rb};
        const cuuint32_t box[2] = {raw_row_bytes<TYPE>() / 2u, kRows}, es[2] = {1, 1};
        if (enc(&mw, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void*>(w), dims, strides, box, es,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return cudaErrorInvalidValue;
    }
    {
        const cuuint64_t dims[2] = {cols, tokens}, strides[1] = {static_cast<cuuint64_t>(cols) * 2u};
        const cuuint32_t box[2] = {kBK, kBN}, es[2] = {1, 1};
        if (enc(&mx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(xh), dims, strides, box, es,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return cudaErrorInvalidValue;
    }
    constexpr uint32_t raw_bytes = TYPE == kF16 ? 0u : kRows * raw_row_bytes<TYPE>();
    constexpr uint32_t kS = stages<TYPE>();
    constexpr uint32_t kSB = stages_b<TYPE>();
    const uint32_t smem = 1024u + kS * kStageA + kSB * kStageB + kRawSlots * raw_bytes +
                          8u * (2u * kS + 2u * kSB + 2u * kRawSlots + 1u) + 16u;
    static bool configured[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(gemm_tc_kernel<TYPE>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
        if (e != cudaSuccess) return e;
        configured[dev] = true;
    }
    GemmArgs a{};
    a.y = y;
    a.rows = rows;
    a.cols = cols;
    a.tokens = tokens;
    a.ldy = ldy;
    a.ksplit = ksplit;
    a.split_stride = split_stride;
    a.status = status;
    // programmatic dependent launch (when `pdl`): the CTAs start (TMEM, barriers,
    // the first weight chunks and their dequantisation) while the previous
    // kernel finishes
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((rows + kRows - 1) / kRows, (tokens + kBN - 1) / kBN, ksplit);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, gemm_tc_kernel<TYPE>, mw, mx, a);
}

// ---- 2-SM variant (quantised weights, more than 256 tokens) ---------------
// A cluster of two CTAs computes a tile of 256 weight rows x 512 tokens with
// tcgen05.mma.cta_group::2 (M = 256 across the pair, N = 256 per MMA, two token
// halves).  CTA rank r holds rows 128r..128r+127 of A and tokens
// 128r..128r+127 of each token half of B, so each SM's MMAs read half of the
// B bytes a one-SM tile of the same work would: shared-memory traffic per K
// stage drops from ~97 KB to ~65 KB per SM.  The leader (rank 0) issues the
// MMAs; the X copies of both CTAs and the dequant warps of both CTAs signal
// the leader's barriers; its commits reach both CTAs.  Raw weight chunks stay
// per CTA.  Each CTA's TMEM holds its 128 rows of both 256-token accumulators.
namespace pair {
constexpr uint32_t kRowsC = 128;             // weight rows per CTA (pair: 256)
constexpr uint32_t kTokC = 128;              // tokens per CTA per token half
constexpr uint32_t kTokPair = 512;           // tokens per pair tile (two MMA N = 256 halves)
constexpr uint32_t kS = 6;                   // A stages
constexpr uint32_t kSB = 6;                  // X stages
// raw chunk slots: every weight row is read by one CTA only (no second token
// tile hits it in L2), so the chunks are fetched four ahead
constexpr uint32_t kRawSlotsP = 4;
constexpr uint32_t kPairStageA = kRowsC * 64;    // 8 KB
constexpr uint32_t kHalfB = kTokC * 64;      // 8 KB: one token half
constexpr uint32_t kPairStageB = 2 * kHalfB;     // 16 KB
constexpr uint32_t kXBytesPair = 2 * kPairStageB;  // bytes landing on the leader's X barrier per stage
// kind::f16, fp32 D, M = 256 (pair), N = 256
constexpr uint32_t kIdesc2 = (1u << 4) | ((256u >> 3) << 17) | ((256u >> 4) << 24);

template <uint32_t TYPE>
constexpr uint32_t raw_bytes() { return kRowsC * raw_row_bytes<TYPE>(); }
template <uint32_t TYPE>
constexpr uint32_t smem_bytes() {
    return 1024u + kS * kPairStageA + kSB * kPairStageB + kRawSlotsP * raw_bytes<TYPE>() +
           8u * (2u * kS + 2u * kSB + 2u * kRawSlotsP + 1u) + 16u;
}

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// shared::cluster address of the same shared-memory offset in CTA `rank`
__device__ __forceinline__ uint32_t map_to_rank(uint32_t saddr, uint32_t rank) {
    uint32_t d;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(d) : "r"(saddr), "r"(rank));
    return d;
}
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void arrive_remote(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// X copy into this CTA's shared memory, completion on a barrier of either CTA of the pair
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map, int32_t c0, int32_t c1,
                                                 uint32_t bar_cluster_addr) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(bar_cluster_addr)
        : "memory");
}
__device__ __forceinline__ void mma_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(kIdesc2), "r"(accumulate)
        : "memory");
}
// arrive on the barrier at this offset in both CTAs once the MMAs issued so far complete
__device__ __forceinline__ void commit_both(uint64_t* bar) {
    const uint16_t mask = 3;
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::
                     "r"(smem_addr(bar)),
                 "h"(mask)
                 : "memory");
}
// bounded wait.  Most phases of this kernel's barriers are completed from the
// other SM of the pair (remote arrivals, the peer's copies, multicast
// commits), so the wait takes no suspend-time hint.
__device__ __forceinline__ bool try_wait_cluster(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ bool wait_cluster_bounded(uint64_t* bar, uint32_t parity, DeviceStatus* st, uint32_t site) {
    if (try_wait_cluster(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    const uint64_t limit = wait_limit_ns(st);
    while (true) {
        if (try_wait_cluster(bar, parity)) return true;
        if (global_timer_ns() - t0 > limit) {
            if (st != nullptr && atomicOr(&st->flags, kErrWaitTimeout) == 0u) st->where = site;
            return false;
        }
    }
}
}  // namespace pair

template <uint32_t TYPE>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    gemm_tc_pair_kernel(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_x,
                        const GemmArgs a) {
    using namespace pair;
    static_assert(TYPE != kF16, "the pair kernel dequantises GGUF blocks");
    extern __shared__ uint8_t smem_raw[];
    const uint32_t s0 = (smem_addr(smem_raw) + 1023u) & ~1023u;
    uint8_t* const sbase = smem_raw + (s0 - smem_addr(smem_raw));
    constexpr uint32_t kRawB = raw_bytes<TYPE>();
    const uint32_t sA = s0;                        // kS x 8 KB
    const uint32_t sB = sA + kS * kPairStageA;         // kSB x 16 KB (two token halves)
    const uint32_t sRaw = sB + kSB * kPairStageB;      // kRawSlotsP x raw chunk
    uint64_t* bars = reinterpret_cast<uint64_t*>(sbase + (sRaw - s0) + kRawSlotsP * kRawB);
    uint64_t* b_full = bars;                  // [kSB] leader: X of both CTAs landed
    uint64_t* a_full = b_full + kSB;          // [kS] leader: A written by both CTAs' dequant warps
    uint64_t* a_empty = a_full + kS;          // [kS] both: MMAs of the A stage done
    uint64_t* b_empty = a_empty + kS;         // [kSB] both: MMAs of the X stage done
    uint64_t* raw_full = b_empty + kSB;       // [kRawSlotsP] per CTA
    uint64_t* raw_empty = raw_full + kRawSlotsP;
    uint64_t* done = raw_empty + kRawSlotsP;   // both: every MMA complete
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);

    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t rank = cluster_rank();
    const uint32_t row0 = (blockIdx.x >> 1) * (2u * kRowsC) + rank * kRowsC;  // this CTA's weight rows
    const uint32_t tok0 = blockIdx.y * kTokPair;                             // the pair's tokens
    const uint32_t ksteps = (a.cols + kBK - 1) / kBK;
    const uint32_t chunks = (a.cols + kRawK - 1) / kRawK;

    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < kS; ++s) {
            mbar_init(&a_full[s], 2u * 4u);  // 4 dequant warps of each CTA write a stage
            mbar_init(&a_empty[s], 1);
        }
        for (uint32_t s = 0; s < kSB; ++s) {
            mbar_init(&b_full[s], 1);
            mbar_init(&b_empty[s], 1);
        }
        for (uint32_t s = 0; s < kRawSlotsP; ++s) {
            mbar_init(&raw_full[s], 1);
            mbar_init(&raw_empty[s], kDeqWarps);
        }
        mbar_init(done, 1);
        fence_barrier_init();
    }
    if (warp == 1) {  // TMEM: both token halves, 2 x 256 fp32 columns (same warp in both CTAs)
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                     "r"(2u * kBN));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
    }
    __syncwarp();
    tc_fence_before();
    // both CTAs' barriers are initialised before either signals the other's
    cluster_sync();
    tc_fence_after();
    const uint32_t tmem_d = *tmem_slot;

    if (warp == 0) {
        // ---------------- TMA producers (both CTAs) ----------------
        // lane 1 streams this CTA's raw weight chunks, gated only by free raw
        // slots (weights never come from the previous kernel), so they are
        // fetched kRawSlotsP chunks ahead; lane 0 copies the X tiles, gated by
        // the MMAs freeing X stages
        if (lane == 1) {
            uint32_t issued_kc = 0;
            for (uint32_t kc = 0; kc < chunks; ++kc) {
                const uint32_t rs = kc % kRawSlotsP;
                if (kc >= kRawSlotsP &&
                    !pair::wait_cluster_bounded(&raw_empty[rs], ((kc / kRawSlotsP) - 1u) & 1u, a.status, 51u))
                    break;
                mbar_arrive_expect_tx(&raw_full[rs], kRawB);
                // the chunk's first byte, rounded down to 16 bytes (uint16 elements)
                const uint32_t first = kc * (kRawK / 32u) * RawBlock<TYPE>::kBytes;
                tma_load_2d(sRaw + rs * kRawB, &map_w, static_cast<int32_t>((first & ~15u) / 2u),
                            static_cast<int32_t>(row0), &raw_full[rs]);
                issued_kc = kc + 1u;
            }
            // drain: the last raw copies have landed before exit
            for (uint32_t k = issued_kc > kRawSlotsP ? issued_kc - kRawSlotsP : 0u; k < issued_kc; ++k)
                pair::wait_cluster_bounded(&raw_full[k % kRawSlotsP], (k / kRawSlotsP) & 1u, a.status, 59u);
        } else if (lane == 0) {
            uint32_t issued_ks = 0;
            grid_dependency_wait();  // X may come from the previous kernel
            for (uint32_t ks = 0; ks < ksteps; ++ks) {
                const uint32_t sb = ks % kSB;
                if (ks >= kSB && !pair::wait_cluster_bounded(&b_empty[sb], ((ks / kSB) - 1u) & 1u, a.status, 52u))
                    break;
                if (rank == 0) mbar_arrive_expect_tx(&b_full[sb], kXBytesPair);
                const uint32_t bar = map_to_rank(smem_addr(&b_full[sb]), 0);
#pragma unroll
                for (uint32_t h = 0; h < 2; ++h)  // token half h: tokens 256h + 128 rank ..
                    tma_load_2d_pair(sB + sb * kPairStageB + h * kHalfB, &map_x, static_cast<int32_t>(ks * kBK),
                                     static_cast<int32_t>(tok0 + h * kBN + rank * kTokC), bar);
                issued_ks = ks + 1u;
            }
            // drain: the leader waits for the last X stages, whose barrier also
            // counts the peer's copies
            if (rank == 0)
                for (uint32_t k = issued_ks > kSB ? issued_ks - kSB : 0u; k < issued_ks; ++k)
                    pair::wait_cluster_bounded(&b_full[k % kSB], (k / kSB) & 1u, a.status, 58u);
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer (leader only) ----------------
        if (rank == 0 && lane == 0) {
            bool ok = true;
            for (uint32_t ks = 0; ks < ksteps && ok; ++ks) {
                const uint32_t s = ks % kS, sb = ks % kSB;
                ok = wait_cluster_bounded(&b_full[sb], (ks / kSB) & 1u, a.status, 53u) &&
                     wait_cluster_bounded(&a_full[s], (ks / kS) & 1u, a.status, 54u);
                if (!ok) break;
                tc_fence_after();
                const uint64_t ad = sw64_desc(sA + s * kPairStageA);
#pragma unroll
                for (uint32_t h = 0; h < 2; ++h) {
                    const uint64_t bd = sw64_desc(sB + sb * kPairStageB + h * kHalfB);
#pragma unroll
                    for (uint32_t kk = 0; kk < kBK / 16u; ++kk)  // +32 bytes = +2 in descriptor units
                        mma_pair(tmem_d + h * kBN, ad + 2u * kk, bd + 2u * kk, (ks | kk) != 0u);
                }
                commit_both(&a_empty[s]);
                commit_both(&b_empty[sb]);
            }
            commit_both(done);
        }
    } else {
        // ---------------- dequant warps (both CTAs), then the epilogue ----------------
        // warps 2..5 write the even K stages of a chunk, warps 6..9 the odd ones;
        // one thread per row of this CTA's 128
        const uint32_t t = threadIdx.x - 64u;
        const uint32_t r = t & (kRowsC - 1u);
        const uint32_t grp = t >> 7;
        bool ok = true;
        for (uint32_t kc = 0; kc < chunks && ok; ++kc) {
            const uint32_t rs = kc % kRawSlotsP;
            if (!pair::wait_cluster_bounded(&raw_full[rs], (kc / kRawSlotsP) & 1u, a.status, 55u)) {
                ok = false;
                break;
            }
            const uint32_t raw_row = sRaw + rs * kRawB + r * raw_row_bytes<TYPE>();
            auto stage = [&](auto J) {
                constexpr uint32_t j = decltype(J)::value;
                const uint32_t ks = kc * (kRawK / kBK) + j;
                if (!ok || ks >= ksteps) return;
                const uint32_t s = ks % kS;
                if (ks >= kS && !pair::wait_cluster_bounded(&a_empty[s], ((ks / kS) - 1u) & 1u, a.status, 56u)) {
                    ok = false;
                    return;
                }
                if (kc & 1u)  // odd chunks start 8 bytes into the loaded row
                    dequant_block<TYPE, 8u, j>(raw_row, sA + s * kPairStageA, r);
                else
                    dequant_block<TYPE, 0u, j>(raw_row, sA + s * kPairStageA, r);
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic writes -> tensor core reads
                __syncwarp();
                if (lane == 0) arrive_remote(map_to_rank(smem_addr(&a_full[s]), 0));
            };
            if (grp == 0) {
                stage(Idx<0>{});
                stage(Idx<2>{});
            } else {
                stage(Idx<1>{});
                stage(Idx<3>{});
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&raw_empty[rs]);
        }
        // epilogue: warp w reads TMEM lane quarter w % 4 of token half (w - 2) / 4
        const uint32_t quarter = warp & 3u;
        const uint32_t h = (warp - 2u) >> 2;
        if (pair::wait_cluster_bounded(done, 0, a.status, 57u)) {
            tc_fence_after();
            const uint32_t wrow = row0 + quarter * 32u + lane;
            for (uint32_t col = 0; col < kBN; col += 32u) {
                uint32_t v[32];
                tc_ld_32x32b_x32(tmem_d + h * kBN + ((quarter * 32u) << 16) + col, v);
                if (wrow < a.rows) {
#pragma unroll
                    for (uint32_t i = 0; i < 32; ++i) {
                        const uint32_t tk = tok0 + h * kBN + col + i;
                        if (tk < a.tokens) a.y[static_cast<size_t>(tk) * a.ldy + wrow] = __uint_as_float(v[i]);
                    }
                }
            }
        }
    }
    // every warp converged; both CTAs done with TMEM and with each other's barriers
    __syncwarp();
    tc_fence_before();
    cluster_sync();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_d), "r"(2u * kBN));
    }
}


template <uint32_t TYPE>
cudaError_t launch_pair_t(const void* w, const __half* xh, float* y, uint32_t rows, uint32_t cols, uint32_t tokens,
                          uint32_t ldy, DeviceStatus* status, cudaStream_t stream, bool pdl) {
    EncodeTiled enc = encode_tiled_fn();
    if (enc == nullptr) return cudaErrorNotSupported;
    CUtensorMap mw, mx;
    const uint64_t rb = row_bytes_of(TYPE, cols);
    {
        // raw rows as uint16 elements, 128 rows per box (one CTA's share of the pair)
        const cuuint64_t dims[2] = {rb / 2u, rows}, strides[1] = {rb};
        const cuuint32_t box[2] = {raw_row_bytes<TYPE>() / 2u, pair::kRowsC}, es[2] = {1, 1};
        if (enc(&mw, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void*>(w), dims, strides, box, es,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return cudaErrorInvalidValue;
    }
    {
        const cuuint64_t dims[2] = {cols, tokens}, strides[1] = {static_cast<cuuint64_t>(cols) * 2u};
        const cuuint32_t box[2] = {kBK, pair::kTokC}, es[2] = {1, 1};
        if (enc(&mx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(xh), dims, strides, box, es,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return cudaErrorInvalidValue;
    }
    static bool configured[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(gemm_tc_pair_kernel<TYPE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             pair::smem_bytes<TYPE>());
        if (e != cudaSuccess) return e;
        configured[dev] = true;
    }
    GemmArgs a{};
    a.y = y;
    a.rows = rows;
    a.cols = cols;
    a.tokens = tokens;
    a.ldy = ldy;
    a.ksplit = 1;
    a.split_stride = 0;
    a.status = status;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2u * ((rows + 2u * pair::kRowsC - 1) / (2u * pair::kRowsC)),
                       (tokens + pair::kTokPair - 1) / pair::kTokPair, 1);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = pair::smem_bytes<TYPE>();
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, gemm_tc_pair_kernel<TYPE>, mw, mx, a);
}

// Quantised weights with more than one 256-token tile and no K split run on
// CTA pairs.
bool use_pair(uint32_t type, uint64_t tokens, uint32_t ksplit) { return type != kF16 && tokens > kBN && ksplit == 1; }

}  // namespace

EncodeTiled encode_tiled_fn() {
    static EncodeTiled fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiled>(p);
    });
    return fn;
}

bool gemm_tc_supported(uint32_t type, uint64_t rows, uint64_t cols, uint64_t tokens) {
    if (type != kF16 && type != kQ8_0 && type != kQ4_0) return false;
    if (rows == 0 || tokens == 0 || rows > 0x7FFFFFFFull || tokens > 0x7FFFFFFFull || cols > 0x7FFFFFFFull) return false;
    if (cols % 32u) return false;
    const uint64_t rb = row_bytes_of(type, cols);
    return rb % 16u == 0 && cols % 8u == 0;
}

uint32_t gemm_tc_ctas(uint64_t rows, uint64_t tokens) {
    return static_cast<uint32_t>(((rows + kRows - 1) / kRows) * ((tokens + kBN - 1) / kBN));
}

uint32_t gemm_tc_launch_ctas(uint32_t type, uint64_t rows, uint64_t cols, uint64_t tokens, int num_sms) {
    const uint32_t splits = gemm_tc_splits(rows, cols, tokens, num_sms);
    if (use_pair(type, tokens, splits))
        return static_cast<uint32_t>(2u * ((rows + 2u * pair::kRowsC - 1) / (2u * pair::kRowsC)) *
                                     ((tokens + pair::kTokPair - 1) / pair::kTokPair));
    return gemm_tc_ctas(rows, tokens) * splits;
}

uint32_t gemm_tc_splits(uint64_t rows, uint64_t cols, uint64_t tokens, int num_sms) {
    // tiles that leave most SMs idle share each tile's K among several CTAs
    const uint64_t tiles = gemm_tc_ctas(rows, tokens);
    const uint64_t chunks = (cols + kRawK - 1) / kRawK;
    if (num_sms <= 0 || tiles * 2u >= static_cast<uint64_t>(num_sms)) return 1;
    uint64_t s = static_cast<uint64_t>(num_sms) / tiles;
    if (s > chunks) s = chunks;
    return s < 1 ? 1u : static_cast<uint32_t>(s);
}

cudaError_t launch_splitk_reduce(const float* ws, float* y, uint32_t splits, uint64_t tokens, uint64_t rows,
                                 uint64_t ldy, int num_sms, cudaStream_t stream, bool pdl) {
    const uint64_t n = tokens * rows;
    uint64_t blocks = (n + 255u) / 256u;
    if (blocks > static_cast<uint64_t>(num_sms) * 8u) blocks = static_cast<uint64_t>(num_sms) * 8u;
    if (blocks == 0) blocks = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<uint32_t>(blocks));
    cfg.blockDim = dim3(256);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, splitk_reduce_kernel, ws, y, splits, static_cast<uint32_t>(tokens),
                              static_cast<uint32_t>(rows), ldy);
}

cudaError_t launch_x_to_f16(const float* x, __half* xh, uint64_t n, int num_sms, cudaStream_t stream, bool pdl) {
    uint64_t blocks = (n / 4u + 255u) / 256u;
    if (blocks > static_cast<uint64_t>(num_sms) * 8u) blocks = static_cast<uint64_t>(num_sms) * 8u;
    if (blocks == 0) blocks = 1;
    // programmatic dependent launch (when `pdl`): scheduled while the previous
    // kernel runs, the conversion itself starts after that kernel's completion
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<uint32_t>(blocks));
    cfg.blockDim = dim3(256);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, x_to_f16_kernel, x, xh, n);
}

cudaError_t launch_gemm_tc(uint32_t type, const void* w, const __half* xh, float* y, uint64_t rows, uint64_t cols,
                           uint64_t tokens, uint64_t ldy, DeviceStatus* status, cudaStream_t stream, bool pdl,
                           uint32_t ksplit, uint64_t split_stride) {
    if (!gemm_tc_supported(type, rows, cols, tokens)) return cudaErrorInvalidValue;
    if (ksplit == 0 || ksplit > (cols + kRawK - 1) / kRawK || ksplit > 65535u) return cudaErrorInvalidValue;
    const uint32_t r = static_cast<uint32_t>(rows), c = static_cast<uint32_t>(cols), t = static_cast<uint32_t>(tokens);
    if (use_pair(type, tokens, ksplit)) {
        if (type == kQ8_0) return launch_pair_t<kQ8_0>(w, xh, y, r, c, t, static_cast<uint32_t>(ldy), status, stream, pdl);
        return launch_pair_t<kQ4_0>(w, xh, y, r, c, t, static_cast<uint32_t>(ldy), status, stream, pdl);
    }
    switch (type) {
        case kQ8_0:
            return launch_t<kQ8_0>(w, xh, y, r, c, t, static_cast<uint32_t>(ldy), ksplit, split_stride, status, stream,
                                    pdl);
        case kQ4_0:
            return launch_t<kQ4_0>(w, xh, y, r, c, t, static_cast<uint32_t>(ldy), ksplit, split_stride, status, stream,
                                    pdl);
        case kF16:
            return launch_t<kF16>(w, xh, y, r, c, t, static_cast<uint32_t>(ldy), ksplit, split_stride, status, stream,
                                    pdl);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace nedo_gpu
