/*
 * nedo_gpu.h -- C ABI of the B200 (sm_100a) matvec library, libnedo_gpu.so.
 *
 * This is the boundary that replaces the CPU hot path of nedo.cpp:
 *
 *   void nedo::kernels::matvec(const TensorInfo& t, std::span<const std::byte> bytes,
 *                              const float* x, float* y);                 kernels.hpp:20
 *   void nedo::kernels::embedding_row(const TensorInfo& t, std::span<const std::byte> bytes,
 *                                     uint32_t row, float* out);          kernels.hpp:21
 *
 * (paths relative to the nedo.cpp project: include/nedo/kernels.hpp,
 * src/kernels.cpp:162-176).  The C++ forwarding layer in
 * nedo.cpp_b200/cpp/nedo_kernels_cuda.cpp keeps those two signatures and calls
 * the host-pointer entry points below, so src/model.cpp and src/pybind.cpp
 * link unchanged.
 *
 * Conventions
 *   - `type` is the GGUF tensor type code (include/nedo/gguf.hpp:18-19):
 *     NEDO_GPU_F16 = 1, NEDO_GPU_Q4_0 = 2, NEDO_GPU_Q8_0 = 8.
 *   - A weight is `rows` rows of `cols` elements, rows contiguous; `cols` is
 *     the contiguous GGUF dimension (TensorInfo::shape[0]) and `rows` is
 *     TensorInfo::shape[1].  Row size follows tensor_nbytes
 *     (src/gguf.cpp:106-114): F16 2*cols, Q4_0 18*cols/32, Q8_0 34*cols/32.
 *   - Activations and outputs are fp32.  Batched calls use x[batch][cols] and
 *     y[batch][rows].
 *   - Every function returns 0 on success or an NEDO_GPU_ERR_* code, never
 *     throws, and leaves a message for nedo_gpu_last_error() (per thread).
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default
 *     stream).  Pointers named *_dev must be device memory on the current
 *     CUDA device; *_host pointers are ordinary host memory.
 */
#ifndef NEDO_GPU_H
#define NEDO_GPU_H

#include <stdint.h>

#if defined(__GNUC__)
#define NEDO_GPU_API __attribute__((visibility("default")))
#else
#define NEDO_GPU_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum {
    NEDO_GPU_F16 = 1,
    NEDO_GPU_Q4_0 = 2,
    NEDO_GPU_Q8_0 = 8
};

enum {
    NEDO_GPU_OK = 0,
    NEDO_GPU_ERR_TYPE = 1,    /* type not supported by this entry point          */
    NEDO_GPU_ERR_ALIGN = 2,   /* Q4_0/Q8_0 column count not a multiple of 32      */
    NEDO_GPU_ERR_ROW = 3,     /* embedding row out of range                        */
    NEDO_GPU_ERR_ARG = 4,     /* null pointer, size mismatch, unsupported size     */
    NEDO_GPU_ERR_CUDA = 5,    /* CUDA runtime error (message names the call)       */
    NEDO_GPU_ERR_DEVICE = 6,  /* a kernel gave up on a bounded wait                */
    NEDO_GPU_ERR_NOMEM = 7    /* device or pinned allocation failed                */
};

/* Library version: major*10000 + minor*100 + patch. */
NEDO_GPU_API int nedo_gpu_version(void);

/* Programmatic dependent launch for the device entry points (process-wide,
 * off by default).  When on, a matvec kernel starts streaming its weight
 * while the previous kernel on the same stream is still running and reads x
 * only once that kernel has completed.  Contract: the weight must not be
 * written by the kernel launched immediately before on that stream (GGUF
 * weights are immutable).  Returns the previous setting. */
NEDO_GPU_API int nedo_gpu_set_pdl(int enable);

/* Batched calls on the exact kernels only (process-wide, off by default).
 * By default a batch of 16 or more Q8_0/Q4_0 vectors (4 or more for F16) with
 * rows of at least 1024 elements -- unless it is at most 32 vectors and one
 * launch of the exact multi-vector int8 kernel takes it whole (small
 * matrices) -- runs one tcgen05 GEMM on fp16 operands: x
 * and d*q are each rounded to fp16 once (relative error <= 2^-11 per
 * factor), products and sums are fp32.  Its worst-case error is therefore
 * about 2^-10 * sum_i |w_i x_i| per output, ten times the reference
 * tolerance of 1e-4 * sum_i |w_i x_i|, reached only when the rounding errors
 * of a row share one sign (e.g. a constant positive x against same-sign
 * weights); on independent inputs they cancel and the results stay within
 * the tolerance (tested at every benchmark shape).  When enabled, batches run
 * the int8 tensor-pipe kernels (exact integer block dots, x carried with 28
 * significant bits; up to 32 vectors per weight pass) or, for F16, one
 * streaming pass per vector: within the tolerance by bound.  Returns the
 * previous setting.  No reference counterpart. */
NEDO_GPU_API int nedo_gpu_set_exact_batches(int enable);

/* Message of the last failing call on this thread ("" if none). */
NEDO_GPU_API const char* nedo_gpu_last_error(void);

/* Bound of every spin-wait of the kernels on the current device, in
 * nanoseconds (0 restores the default of 2 s).  A wait that runs out makes
 * its kernel wind down and record the failure, which the next
 * nedo_gpu_status / host call reports as NEDO_GPU_ERR_DEVICE; the device stays
 * usable.  No reference counterpart (the reference has no device waits). */
NEDO_GPU_API int nedo_gpu_set_wait_limit_ns(uint64_t ns);

/* ---------------------------------------------------------------------------
 * Host-pointer entry points: drop-in semantics of the reference.
 *
 * Synchronous: the result is in y_host/out_host on return, like the CPU
 * kernel.  The weight bytes are uploaded to the device on first use (through
 * pinned bounce buffers) and kept resident, keyed by (w_host, w_bytes) and a
 * content fingerprint (first and last 4 KB plus 64 samples, checked on every
 * call) -- the reference passes spans into a GGUF mmap that stay valid and
 * unchanged for the model's lifetime (src/gguf.cpp:139).  A buffer freed and
 * reused at the same address with other bytes is uploaded again.  A caller
 * that rewrites a weight buffer in place where the fingerprint does not look
 * must call nedo_gpu_weight_evict() first.  Calls are serialised per device.
 * ------------------------------------------------------------------------- */

/* Replaces nedo::kernels::matvec (src/kernels.cpp:162-169):
 *   y_host[r] = sum_i dequant(w)[r][i] * x_host[i], r < rows.
 * Errors mirror the reference: a Q4_0/Q8_0 column count that is not a
 * multiple of 32 ("... elements not block aligned", src/gguf.cpp:109-110),
 * an unsupported type ("matvec tensor type not supported", src/kernels.cpp:168).
 * w_bytes must be at least rows * row_bytes. */
NEDO_GPU_API int nedo_gpu_matvec(uint32_t type, uint64_t rows, uint64_t cols, const void* w_host, uint64_t w_bytes,
                    const float* x_host, float* y_host);

/* `batch` calls of nedo_gpu_matvec over one weight in one call:
 * y_host[b][r] = dot(row r, x_host[b]), b < batch (x_host [batch][cols],
 * y_host [batch][rows]).  Replaces the reference's prompt loop, one matvec per
 * token for every weight (src/model.cpp:262-266, the forward lambda at
 * :212-260), with one pass over the weight; the kernel choice is that of
 * nedo_gpu_matvec_dev with the same batch.  Errors as nedo_gpu_matvec. */
NEDO_GPU_API int nedo_gpu_matvec_batch(uint32_t type, uint64_t rows, uint64_t cols, const void* w_host,
                                       uint64_t w_bytes, const float* x_host, float* y_host, uint32_t batch);

/* Replaces nedo::kernels::embedding_row (src/kernels.cpp:170-176): writes the
 * dequantised row `row` (cols floats) to out_host, bit-identical to the
 * reference.  row >= rows -> NEDO_GPU_ERR_ROW ("bad embedding row"). */
NEDO_GPU_API int nedo_gpu_embedding_row(uint32_t type, uint64_t rows, uint64_t cols, const void* w_host, uint64_t w_bytes,
                           uint32_t row, float* out_host);

/* Upload (or find) the resident device copy of a host weight buffer.
 * *w_dev_out receives the device pointer (valid until evicted). */
NEDO_GPU_API int nedo_gpu_weight_upload(const void* w_host, uint64_t w_bytes, const void** w_dev_out);
/* Drop the resident copy of w_host (no-op if absent). */
NEDO_GPU_API int nedo_gpu_weight_evict(const void* w_host);
/* Drop every resident weight on every device this library touched, and free
 * the batched-call buffers that larger calls replaced (a CUDA graph captured
 * with one of those is invalid afterwards). */
NEDO_GPU_API int nedo_gpu_cache_clear(void);

/* ---------------------------------------------------------------------------
 * Device-pointer entry points (asynchronous on `stream`).
 * ------------------------------------------------------------------------- */

/* The matvec of nedo_gpu_matvec on device buffers, for `batch` activation
 * vectors: y_dev[b][r] = dot(row r, x_dev[b]), b < batch.  batch == 1 is the
 * decode path (src/model.cpp:217-259); batch > 1 replaces `batch` serial
 * calls over the same weight, which is how the reference processes a prompt
 * (src/model.cpp:262-266).  Q8_0/Q4_0 batches of 2 to 15 vectors, and of up
 * to 32 that one launch takes whole, run the exact multi-vector int8 kernel
 * (each weight tile read once per launch for all its vectors).  Otherwise,
 * for rows of at least 1024 elements, from 16 vectors on (4 for F16 weights)
 * the batch runs as one tensor-core GEMM with x and the dequantised weight
 * rounded to fp16 (fp32 accumulation).  The GEMM calls
 * calls use two per-device buffers (an fp16 copy of x and, for few row tiles,
 * a split-K workspace), allocated by the first call that needs them and grown
 * by a larger one.  A grown-out buffer stays allocated until
 * nedo_gpu_cache_clear, so a CUDA graph captured earlier keeps working.  To
 * capture such a call in a graph, size the buffers first, outside capture,
 * with nedo_gpu_reserve (or one eager call of the largest shape): a call that
 * has to allocate cannot be captured.  Calls on one device share the buffers:
 * serialise calls that may overlap (other streams, other threads). */
NEDO_GPU_API int nedo_gpu_matvec_dev(uint32_t type, uint64_t rows, uint64_t cols, const void* w_dev, const float* x_dev,
                        float* y_dev, uint32_t batch, void* stream);

/* Size the per-device buffers of a batched nedo_gpu_matvec_dev call of this
 * shape (no-op for shapes that need none), so that the call itself allocates
 * nothing and can be captured in a CUDA graph.  Call outside stream capture.
 * No reference counterpart. */
NEDO_GPU_API int nedo_gpu_reserve(uint32_t type, uint64_t rows, uint64_t cols, uint32_t batch);

/* matvec followed by the greedy pick of the LM head (std::max_element over
 * the logits, src/model.cpp:36: first index of the maximum), fused into the
 * matvec kernel where the shape allows.  y_dev receives the logits;
 * index_dev (int64) the argmax; value_dev (may be NULL) its value.  Uses a
 * per-device scratch area: calls that overlap on the GPU must not share a
 * device. */
NEDO_GPU_API int nedo_gpu_matvec_argmax_dev(uint32_t type, uint64_t rows, uint64_t cols, const void* w_dev, const float* x_dev,
                               float* y_dev, int64_t* index_dev, float* value_dev, void* stream);

/* argmax of an fp32 vector in device memory (first index of the maximum).
 * NaN behaves as in std::max_element: a NaN never wins, except that a NaN at
 * index 0 makes the result 0 (every comparison with it is false); this holds
 * for every argmax entry point. */
NEDO_GPU_API int nedo_gpu_argmax_dev(const float* v_dev, uint64_t n, int64_t* index_dev, float* value_dev, void* stream);

/* nedo_gpu_argmax_dev without any allocation: the same kernel and result,
 * with its per-CTA candidates and completion counter in a fixed 8448-byte
 * __device__ array of the library (room for 1024 CTAs; a launch needing more
 * returns NEDO_GPU_ERR_ARG) instead of the per-device scratch that the other
 * entry points allocate on first use.  No reference counterpart: the
 * reference picks the token on the host (std::max_element, src/model.cpp:36).
 * The first call on a device resolves the array's address; make it outside
 * stream capture.  Calls that may overlap on one device (other streams, other
 * threads) share the array and race: serialise them. */
NEDO_GPU_API int nedo_gpu_argmax_dev_noalloc(const float* v_dev, uint64_t n, int64_t* index_dev, float* value_dev,
                                void* stream);

/* The k largest elements of an fp32 vector in device memory, largest first
 * (equal values: smaller index first; NaN never ahead of a number):
 * ids_dev[0..k) (uint32) and vals_dev[0..k) (may be NULL).  1 <= k <= 256 and
 * k <= n.  This is the candidate selection of the reference's sampler
 * (sample_token, src/model.cpp:38-44: nth_element + sort by logit), done where
 * the logits are.  Uses a per-device scratch area: calls that overlap on the
 * GPU must not share a device. */
NEDO_GPU_API int nedo_gpu_topk_dev(const float* v_dev, uint64_t n, uint32_t k, uint32_t* ids_dev, float* vals_dev,
                                   void* stream);

/* Host-pointer LM head (the matvec of src/model.cpp:259, nedo_gpu_matvec's
 * residency and errors) followed by the top k logits (nedo_gpu_topk_dev), with
 * only the k (id, logit) pairs copied back instead of all `rows` logits:
 * ids_host[0..k), vals_host[0..k) (may be NULL).  1 <= k <= min(rows, 256). */
NEDO_GPU_API int nedo_gpu_lm_head_topk(uint32_t type, uint64_t rows, uint64_t cols, const void* w_host,
                                       uint64_t w_bytes, const float* x_host, uint32_t k, uint32_t* ids_host,
                                       float* vals_host);

/* Host-pointer LM head with the greedy pick (src/model.cpp:36, std::max_element
 * semantics as nedo_gpu_argmax_dev), fused into the matvec where the shape
 * allows: *index_host, *value_host (may be NULL); no logits are copied back. */
NEDO_GPU_API int nedo_gpu_lm_head_argmax(uint32_t type, uint64_t rows, uint64_t cols, const void* w_host,
                                         uint64_t w_bytes, const float* x_host, int64_t* index_host,
                                         float* value_host);

/* Row-sharded matvec with the all-gather of y fused into it (one process
 * per GPU; rows are independent, src/kernels.cpp:166-168).  Computes this
 * rank's rows into y_dev like nedo_gpu_matvec_dev and also stores each row at
 * peer_y[k] + row_offset + r on every peer k (peer device addresses, e.g. from
 * CUDA IPC or symmetric memory, reachable over NVLink), then adds 1 per CTA to
 * each peer's 32-bit word peer_signal[k].  Q8_0 / Q4_0 shapes of the int8
 * tensor-pipe kernel only (plan_info path 4); at most 7 peers.  A receiver
 * calls nedo_gpu_allgather_wait_dev before reading the gathered y.  No
 * reference counterpart: the reference runs on one CPU. */
NEDO_GPU_API int nedo_gpu_matvec_allgather_dev(uint32_t type, uint64_t rows, uint64_t cols, const void* w_dev,
                                  const float* x_dev, float* y_dev, const uint64_t* peer_y,
                                  const uint64_t* peer_signal, uint32_t npeers, uint64_t row_offset, void* stream);

/* Wait on `stream` (one GPU thread, bounded by nedo_gpu_set_wait_limit_ns, 2 s
 * by default; a timeout sets the status word read by nedo_gpu_status) until
 * *signal_dev has advanced by `increment` (peers x CTAs of their launches)
 * past *expected_dev, then advance *expected_dev by `increment` -- also after
 * a timeout, so that signals of a late step are never counted for the next
 * one.  After NEDO_GPU_ERR_DEVICE the gathered rows of that step are invalid;
 * later steps are correct once the late peer has caught up.  Both words start
 * at zero; the caller keeps them per receiving buffer. */
NEDO_GPU_API int nedo_gpu_allgather_wait_dev(uint32_t* signal_dev, uint32_t* expected_dev, uint32_t increment,
                                void* stream);

/* embedding_row for rows [row_begin, row_begin + row_count) into
 * out_dev[row_count][cols]; bit-identical to the reference. */
NEDO_GPU_API int nedo_gpu_dequant_rows_dev(uint32_t type, uint64_t rows, uint64_t cols, const void* w_dev, uint64_t row_begin,
                              uint64_t row_count, float* out_dev, void* stream);

/* Wait for `stream`, then report (and clear) device-side failures recorded
 * by kernels on the current device since the last check. */
NEDO_GPU_API int nedo_gpu_status(void* stream);

/* Describe the kernel choice for a shape: out[0] = path (1 streaming CUDA-core,
 * 2 generic, 3 batched streaming (one launch per vector), 4 int8 tensor-pipe
 * matvec, 5 tcgen05 GEMM over the batch), out[1] grid,
 * out[2] threads, out[3] dynamic shared bytes, out[4] rows per tile,
 * out[5] ring slots (path 5: K splits per tile, > 1 adding a fold kernel),
 * out[6] slot bytes, out[7] warps per CTA (compute warps for path 4),
 * out[8] (when n > 8) kernels one call launches.  Path 4 with several vectors
 * describes the first launch.  n = capacity of out (>= 8). */
NEDO_GPU_API int nedo_gpu_plan_info(uint32_t type, uint64_t rows, uint64_t cols, uint32_t batch, uint32_t* out, int n);

/* ---- Device-resident decode forward pass -------------------------------
 *
 * Replaces the `forward` step of NedoModel::generate_ids (src/model.cpp:212-260):
 * embedding row, then per layer RMSNorm, q/k/v projections, RoPE, the KV-cache
 * write, attention over the sliding window, the output projection and residual,
 * RMSNorm, gate/up projections, SiLU gate (with the MorphFFN masking of the
 * trailing layers, :196-209), the down projection and residual; then the final
 * RMSNorm and the LM-head matvec.  Weights and the fp32 KV cache stay on the
 * device; one call runs the whole pass as one CUDA graph (captured on the first
 * call, the token and position read from device memory) and returns the greedy
 * pick and, on request, the logits.
 *
 * The configuration mirrors ModelConfig (include/nedo/model.hpp:12-16). */
typedef struct {
    uint32_t vocab, dim, layers, heads, kv_heads, head_dim, ffn, context, sliding;
    uint32_t morph_layers, morph_shared, morph_root, morph_suffix;
    float rms_eps, rope_theta;
} nedo_gpu_decoder_config;

/* One GGUF tensor: TensorInfo's type and shape (contiguous dimension first)
 * and a host view of its bytes (e.g. GgufFile::bytes, src/gguf.cpp:139). */
typedef struct {
    uint32_t type;
    uint32_t ndims;
    uint64_t shape[2];
    const void* data;
    uint64_t nbytes;
} nedo_gpu_tensor_view;

/* Tensor order of nedo_gpu_decoder_create:
 *   [0] token_embd (F16 / Q8_0 / Q4_0), [1] output_norm (F32 / F16),
 *   [2] output (F16 / Q8_0 / Q4_0; data NULL: the head is token_embd),
 *   [3] blk.0.ffn_gate_tid2eid, the MorphFFN routing table (F32 [2, vocab];
 *       data NULL: none),
 *   then 9 per layer: attn_norm, attn_q, attn_k, attn_v, attn_output, ffn_norm,
 *   ffn_gate, ffn_up, ffn_down (norms F32 / F16, projections F16 / Q8_0 / Q4_0;
 *   q, k, v of one type, gate and up of one type).
 * Shape and type checks follow the reference: "invalid GQA dimensions"
 * (heads % kv_heads, dim == heads * head_dim), "context_length is zero",
 * "MorphFFN widths do not sum to feed_forward_length", and every tensor's
 * shape against the configuration.  The weights are copied to the device; the
 * host views may be released afterwards. */
typedef struct nedo_gpu_decoder nedo_gpu_decoder;
NEDO_GPU_API int nedo_gpu_decoder_create(const nedo_gpu_decoder_config* cfg, const nedo_gpu_tensor_view* tensors,
                                         uint64_t ntensors, nedo_gpu_decoder** out);

/* One forward pass for `token` at position `pos` (positions from 0, one per
 * call, as generate_ids: the KV-cache slot is pos % window with window =
 * min(sliding ? sliding : context, context)).  *argmax_out (if non-null) gets
 * the greedy pick (std::max_element semantics: first index of the maximum);
 * logits_host (if non-null) gets the vocab logits.  token >= vocab
 * ("prompt token id out of range") and pos >= context are NEDO_GPU_ERR_ARG. */
NEDO_GPU_API int nedo_gpu_decoder_forward(nedo_gpu_decoder* d, uint32_t token, uint64_t pos, float* logits_host,
                                          uint32_t* argmax_out);

/* Greedy generation with the loop on the device: n passes, the first for
 * `token` at `pos`, each next pass fed the previous pass's greedy pick; the
 * picks go to ids_host[0..n) (ids_host[k] is the pick of pass k).  Equivalent
 * to n forward calls with temperature-0 sampling between them
 * (src/model.cpp:271-279) but without a host round trip per token: the n
 * passes are launched back to back and the ids read once.  The eos id does
 * not stop the device loop (the caller truncates at it); pos + n <= context. */
NEDO_GPU_API int nedo_gpu_decoder_generate(nedo_gpu_decoder* d, uint32_t token, uint64_t pos, uint32_t n,
                                           uint32_t* ids_host);

/* Run the passes on `stream` (a cudaStream_t; NULL returns to the decoder's
 * own stream).  The captured graphs are dropped and captured again on the
 * next calls.  Every forward call still waits for its pass to finish. */
NEDO_GPU_API int nedo_gpu_decoder_set_stream(nedo_gpu_decoder* d, void* stream);

/* The logits of the last forward pass in device memory (valid until the next
 * call), for the sampler entry points (nedo_gpu_topk_dev). */
NEDO_GPU_API int nedo_gpu_decoder_logits_dev(nedo_gpu_decoder* d, const float** logits_dev);

/* Zero the KV cache (a new sequence starts at pos 0 either way). */
NEDO_GPU_API int nedo_gpu_decoder_reset(nedo_gpu_decoder* d);

/* Free the decoder's device memory and graphs (NULL is a no-op). */
NEDO_GPU_API void nedo_gpu_decoder_destroy(nedo_gpu_decoder* d);

#ifdef __cplusplus
}
#endif
#endif /* NEDO_GPU_H */
