// launch.h -- host-side launchers of the matvec kernels (internal to libnedo_gpu.so).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

namespace nedo_gpu {

// Argmax bookkeeping for the fused LM-head path: one candidate per CTA plus a
// self-resetting completion counter (the last CTA to finish folds the
// candidates and writes the winner).
struct ArgmaxScratch {
    float* cand_val;      // [max_ctas]
    uint32_t* cand_idx;   // [max_ctas] (row index of the candidate)
    uint32_t* counter;    // starts at 0, reset to 0 by the last CTA
    int64_t* out_index;   // result
    float* out_value;     // result (may be null)
};

struct StreamPlan {
    bool ok = false;
    uint32_t warps = 0;          // per CTA; every warp streams its own row range
    uint32_t rows_per_tile = 0;  // rows moved per tile (one contiguous byte range)
    uint32_t slots = 0;          // ring slots per warp
    uint32_t slot_bytes = 0;
    uint32_t x_bytes = 0;        // shared memory for the staged activations
    uint32_t piece_bytes = 0;    // bytes per bulk copy
    uint32_t threads = 0;
    uint32_t smem_bytes = 0;
    uint32_t grid = 0;
};

// Optional overrides of the planner's choices (0 = planner default).
struct StreamTuning {
    uint32_t warps = 0;
    uint32_t slots = 0;
    uint32_t tile_bytes = 0;
    uint32_t piece_bytes = 0;
    uint32_t smem_budget = 0;
};

StreamPlan plan_stream(uint32_t type, uint64_t rows, uint64_t cols, int num_sms, int max_smem_optin,
                       const StreamTuning* tune = nullptr);

// Batch-1 streaming GEMV over GGUF bytes.  w/x/y are device pointers on the
// current device.  When `amax` is non-null the argmax of y is also produced
// (first index on ties).  `pdl` launches with programmatic stream
// serialisation: the kernel starts streaming its weight while the previous
// kernel on the stream finishes, and reads x only after that kernel completed.
cudaError_t launch_stream(uint32_t type, const StreamPlan& plan, const void* w, const float* x, float* y,
                          uint64_t rows, uint64_t cols, DeviceStatus* status, const ArgmaxScratch* amax,
                          cudaStream_t stream, bool pdl);

// Batch-1 Q8_0 / Q4_0 on the int8 tensor pipe (mma.sync m16n8k32, x as exact
// int8 limbs).  A unit of work is 16 rows x seg_pairs block pairs, one
// tensor-map copy; each consumer warp owns whole 16-row tiles.
struct ImmaPlan {
    bool ok = false;
    bool wide = false;         // ring sized for the whole SM (else two CTAs fit on an SM)
    bool slice = false;        // resident slice: every unit of a CTA in its own slot (gemv_imma_slice_kernel)
    uint32_t tile_group = 0;   // slice: tiles sharing one read of the x side
    uint32_t early_chunks = 0; // slice: column chunks copied before x is requested
    bool multi = false;        // multi-vector resident slice (gemv_imma_multi_kernel)
    uint32_t token_groups = 0; // multi: groups of CTAs, `tokens` vectors each
    uint32_t type = 0;
    uint32_t warps = 0;        // consumer warps; one more warp streams units
    uint32_t team = 0;         // warps sharing one tile (its segments split among them)
    uint32_t tokens = 0;       // token vectors per launch (1, 2, 4 or 8)
    uint32_t seg_pairs = 0;    // block pairs per unit
    uint32_t tile_rows = 0;    // 16
    uint32_t tiles = 0;        // ceil(rows / 16)
    uint32_t slots = 0;
    uint32_t unit_bytes = 0;   // shared-memory bytes per slot
    uint32_t box_bytes = 0;    // bytes per unit row: its pitch (an odd multiple of 16)
    uint32_t smem_bytes = 0;
    uint32_t grid = 0;
    uint32_t groups = 0;       // column groups per row (the x table is rebuilt between them)
    uint32_t group_pairs = 0;  // block pairs per group
};

struct ImmaTuning {
    int wide = -1;             // 1 = ring sized for the whole SM
    int slice = -1;            // 0 = never the resident-slice kernel
    uint32_t ctas_per_sm = 0;  // grid = SMs x this (at most the tile count)
    uint32_t slots = 0;
    uint32_t seg_pairs = 0;    // 8 or 16
    uint32_t smem_budget = 0;
    uint32_t table_budget = 0; // bytes of x table built at once (0 = default)
    uint32_t max_tile_group = 0; // slice: at most this many tiles per work item (0 = up to 5)
};

ImmaPlan plan_imma(uint32_t type, uint64_t rows, uint64_t cols, int num_sms, int max_smem_optin,
                   const ImmaTuning* tune = nullptr, uint32_t tokens = 1);

// The multi-vector resident slice for exactly `tokens` (>= 2) vectors in one
// launch: token groups of 2, 4 or 8 vectors (the lowest estimated time among
// those that fit; only `vectors_per_group` when it is non-zero), or !ok when
// none fits.
ImmaPlan plan_imma_multi(uint32_t type, uint64_t rows, uint64_t cols, int num_sms, int max_smem_optin,
                         uint32_t tokens, uint32_t vectors_per_group = 0);

// Fused all-gather of a row-sharded matvec over NVLink: the kernel also stores
// its rows into every peer's gathered y and counts each finished CTA on the
// peer's signal word (see launch_gather_wait).
constexpr uint32_t kMaxPeers = 7;
struct PeerGather {
    uint32_t npeers = 0;
    uint64_t row_offset = 0;          // this rank's first row in the gathered y
    float* peer_y[kMaxPeers] = {};     // each peer's gathered y (peer device pointers)
    uint32_t* peer_signal[kMaxPeers] = {};
};
// plan.tokens token vectors: x [tokens][ldx], y [tokens][ldy] (0 = cols / rows);
// every weight unit is read once for all of them.
// The input transform a resident-slice launch (plan.slice) can apply to x as
// it builds its x table, fusing the step that precedes a projection in the
// decode pass: kPrologueNorm x_in = RMSNorm(x + delta) * w (src/kernels.cpp:50-72;
// every CTA sums the squares itself, CTA 0 also stores x + delta to x_out),
// kPrologueSilu x_in = silu(x) * up with the MorphFFN masking
// (src/kernels.cpp:88-91, src/model.cpp:196-209).
enum : uint32_t { kPrologueNone = 0, kPrologueNorm = 1, kPrologueSilu = 2 };
struct DecodeIo;
struct XPrologue {
    uint32_t mode = kPrologueNone;
    const float* delta = nullptr;  // norm: added to x first (may be null)
    const void* w = nullptr;       // norm: weight (F32 or F16)
    uint32_t wtype = 0;            // 0 F32, 1 F16
    float eps = 0.f;
    float* x_out = nullptr;        // norm: x + delta (may be null)
    const float* up = nullptr;     // silu: the up half
    const float* route = nullptr;  // silu: MorphFFN flags [vocab][2] (null: no masking)
    const DecodeIo* io = nullptr;  // silu with route: the token; cache prefetch: the position
    uint32_t m_shared = 0, m_root = 0, m_suffix = 0;
    // L2 prefetch of a layer's KV-cache rows for the attention step that follows
    // (kcache non-null): the rows of the window's cached positions before io->pos,
    // a ring of `window` rows of `row_bytes` (a multiple of 16) for keys and for
    // values, shared out among the CTAs
    const float* kcache = nullptr;
    const float* vcache = nullptr;
    uint32_t window = 0;
    uint32_t row_bytes = 0;
};
cudaError_t launch_imma(const ImmaPlan& plan, const void* w, const float* x, float* y, uint64_t rows, uint64_t cols,
                        DeviceStatus* status, cudaStream_t stream, bool pdl, const PeerGather* gather = nullptr,
                        uint64_t ldx = 0, uint64_t ldy = 0, const XPrologue* prologue = nullptr);

// Batch-1 Q8_0 / Q4_0 on tcgen05 (kind::i8, A from TMEM): 16-row tiles, one
// MMA per 8 blocks of a tile (M = 16 rows x 8 blocks), at most ~110 KB of
// shared memory and 256 TMEM columns per CTA so that two launches share an SM.
// Rows of a multiple of 256 elements, at most 8192.
struct Tc8Plan {
    bool ok = false;
    uint32_t type = 0;
    uint64_t rows = 0, cols = 0;
    uint32_t grid = 0;
    uint32_t threads = 0;
    uint32_t slots = 0;        // ring slots (units of 16 rows x 16 blocks)
    uint32_t unit_bytes = 0;
    uint32_t tiles = 0;
    uint32_t steps = 0;        // K steps (8 blocks) per row
    uint32_t units = 0;        // units per tile
    uint32_t off_table = 0, off_consts = 0, off_sd = 0, off_red = 0, off_bars = 0;
    uint32_t smem_bytes = 0;
};
Tc8Plan plan_tc8(uint32_t type, uint64_t rows, uint64_t cols, int num_sms, int max_smem_optin);
cudaError_t launch_tc8(const Tc8Plan& plan, const void* w, const float* x, float* y, DeviceStatus* status,
                       cudaStream_t stream, bool pdl);

// Top-k of an fp32 vector (k <= kTopkMax): ids[0..k) and vals[0..k) by value
// descending, equal values by smaller index first, NaN never ahead of a number.
constexpr uint32_t kTopkMax = 256;
struct TopkScratch {
    uint64_t* cand;     // [ctas x 256] candidate keys
    uint32_t* counter;  // starts at 0, reset to 0 by the last CTA
    uint32_t* ids;      // result
    float* vals;        // result (may be null)
};
uint32_t topk_ctas(uint64_t n, uint32_t k, int num_sms);
cudaError_t launch_topk(const float* v, uint64_t n, uint32_t k, const TopkScratch& s, int num_sms,
                        cudaStream_t stream);

// One thread waits (bounded, 2 s) until *signal has advanced by `increment`
// past *expected, then advances *expected: the peers' rows are visible after it.
cudaError_t launch_gather_wait(uint32_t* signal, uint32_t* expected, uint32_t increment, DeviceStatus* status,
                               cudaStream_t stream, bool pdl);

// Any shape the streaming kernel does not take (odd row sizes, unaligned
// pointers): one warp per row, byte-granular loads.  x is [batch][ldx], y [batch][ldy].
cudaError_t launch_generic(uint32_t type, const void* w, const float* x, float* y, uint64_t rows, uint64_t cols,
                           uint32_t batch, uint64_t ldx, uint64_t ldy, cudaStream_t stream);

// embedding_row: out[i] = d * q[i] for one row (bit-exact with the reference).
cudaError_t launch_dequant_rows(uint32_t type, const void* w, uint64_t rows, uint64_t cols, uint64_t row_begin,
                                uint64_t row_count, float* out, cudaStream_t stream);

// argmax over an fp32 vector already in device memory (first index on ties).
cudaError_t launch_argmax(const float* v, uint64_t n, ArgmaxScratch* scratch, int num_sms, cudaStream_t stream);

// Batched matvec (prefill-shaped GEMM) on the tcgen05 tensor cores:
// y[t][r] = sum_k W[r][k] * xh[t][k], W a GGUF tensor (dequantised to fp16 in
// shared memory), xh the token vectors in fp16 (launch_x_to_f16), y fp32 with
// row pitch ldy.  Supported: F16 / Q8_0 / Q4_0, cols % 32 == 0, 16-byte rows.
bool gemm_tc_supported(uint32_t type, uint64_t rows, uint64_t cols, uint64_t tokens);
uint32_t gemm_tc_ctas(uint64_t rows, uint64_t tokens);  // CTAs of one launch (128 rows x 256 tokens each)
cudaError_t launch_x_to_f16(const float* x, __half* xh, uint64_t n, int num_sms, cudaStream_t stream, bool pdl);
// ksplit > 1: each tile's K is shared by ksplit CTAs, split z writing its partial
// sums to y + z * split_stride (a workspace, folded by launch_splitk_reduce).
// `pdl`: programmatic dependent launch (weights streamed before the previous
// kernel on the stream completes; x read after it), for all three launches.
cudaError_t launch_gemm_tc(uint32_t type, const void* w, const __half* xh, float* y, uint64_t rows, uint64_t cols,
                           uint64_t tokens, uint64_t ldy, DeviceStatus* status, cudaStream_t stream, bool pdl,
                           uint32_t ksplit = 1, uint64_t split_stride = 0);
// CTAs along K per tile for a GEMM whose tiles would leave most SMs idle (1 otherwise).
uint32_t gemm_tc_splits(uint64_t rows, uint64_t cols, uint64_t tokens, int num_sms);
// CTAs launch_gemm_tc starts for this shape with gemm_tc_splits' K split: quantised
// weights with more than 256 tokens and no split run as CTA pairs of 256 rows x
// 512 tokens, everything else as 256-row x 256-token tiles.
uint32_t gemm_tc_launch_ctas(uint32_t type, uint64_t rows, uint64_t cols, uint64_t tokens, int num_sms);
// y[t * ldy + r] = sum_z ws[(z * tokens + t) * rows + r], z in order (deterministic).
cudaError_t launch_splitk_reduce(const float* ws, float* y, uint32_t splits, uint64_t tokens, uint64_t rows,
                                 uint64_t ldy, int num_sms, cudaStream_t stream, bool pdl);

uint64_t row_bytes_of(uint32_t type, uint64_t cols);

// ---- decode forward (decode.cu) ----
// The per-step inputs of a captured decode graph, in device memory.
struct DecodeIo {
    uint64_t pos;
    uint32_t token;
    uint32_t step;  // generation: passes run so far (index of the next pick in ids)
};
// x = embedding row io->token (F16 / Q8_0 / Q4_0 rows of `cols`; an id >= rows sets kErrArgument).
cudaError_t launch_embed(uint32_t type, const void* w, uint64_t cols, uint64_t rows, const DecodeIo* io, float* x,
                         DeviceStatus* st, cudaStream_t stream, bool pdl);
// x += delta (delta may be null), y = RMSNorm(x) * w (w F32, wtype 0, or F16, wtype 1).
cudaError_t launch_add_rmsnorm(float* x, const float* delta, const void* w, uint32_t wtype, float* y, uint32_t n,
                               float eps, cudaStream_t stream, bool pdl);
// RoPE, the KV-cache write of position io->pos and attention of the nq heads
// over the window, for qkv = [q (nq x hd) | k (nkv x hd) | v (nkv x hd)]: one
// launch of attention_splits(window) x nq CTAs; part holds nq x splits x
// (hd + 2) floats, counter nq zeros (left zero).
uint32_t attention_splits(uint32_t window);
cudaError_t launch_attention(const float* qkv, float* kcache, float* vcache, float* att, float* part,
                             uint32_t* counter, const DecodeIo* io, uint32_t nq, uint32_t nkv, uint32_t hd,
                             uint32_t window, float theta, float inv_sqrt_hd, cudaStream_t stream, bool pdl);
// io->token = pick, io->pos += 1, ids[io->step++] = pick (single thread, after the pass).
cudaError_t launch_advance(DecodeIo* io, const int64_t* pick, uint32_t* ids, uint32_t cap, cudaStream_t stream);
// gu = [gate | up] (f each): gate = silu(gate) * up, MorphFFN masks when route is non-null.
cudaError_t launch_silu_mul(float* gu, uint32_t f, const float* route, const DecodeIo* io, uint32_t shared_w,
                            uint32_t root_w, uint32_t suffix_w, cudaStream_t stream, bool pdl);

// cuTensorMapEncodeTiled reached through the runtime's driver entry point
// (null when the driver does not provide it).
using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiled encode_tiled_fn();

}  // namespace nedo_gpu
