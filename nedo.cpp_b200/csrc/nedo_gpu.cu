// nedo_gpu.cu -- the C ABI declared in include/nedo_gpu.h.
//
// Host-side responsibilities: argument checks with the reference's error
// semantics (src/kernels.cpp:162-176, src/gguf.cpp:106-114), per-device state
// (SM count, status word, argmax scratch, pinned staging), the weight
// residency cache for the host-pointer entry points, and the choice between
// the streaming kernel, the batched tensor-core kernel and the generic kernel.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <atomic>
#include <cstring>
#include <algorithm>
#include <mutex>
#include <string>
#include <unordered_map>
#include <utility>
#include <vector>

#include "../../include/nedo_gpu.h"
#include "common.cuh"
#include "launch.h"

using namespace nedo_gpu;

namespace {

thread_local std::string g_last_error;

int fail(int code, const std::string& msg) {
    g_last_error = msg;
    return code;
}

int cuda_fail(cudaError_t e, const char* what) {
    std::string m = std::string(what) + ": " + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ")";
    return fail(e == cudaErrorMemoryAllocation ? NEDO_GPU_ERR_NOMEM : NEDO_GPU_ERR_CUDA, m);
}

#define NEDO_CUDA_TRY(call)                                  \
    do {                                                     \
        cudaError_t e_ = (call);                             \
        if (e_ != cudaSuccess) return cuda_fail(e_, #call);  \
    } while (0)

// A resident weight, and the CUDA graph of the host entry point's call on it
// (x upload, matvec, y and status download) once the call has run eagerly.
struct Resident {
    void* dev = nullptr;
    uint64_t bytes = 0;
    uint64_t fingerprint = 0;  // content_fingerprint() of the host bytes at upload
    cudaGraphExec_t call = nullptr;
    uint32_t type = 0;
    uint64_t rows = 0, cols = 0;
    const void* bufs[5] = {};  // staging buffers the graph was captured with
};

void release_resident(Resident& r) {
    if (r.call) cudaGraphExecDestroy(r.call);
    r.call = nullptr;
    if (r.dev) cudaFree(r.dev);
    r.dev = nullptr;
}

struct DeviceState {
    int device = -1;
    int num_sms = 0;
    int max_smem = 0;
    DeviceStatus* status = nullptr;  // device memory
    ArgmaxScratch scratch{};
    uint64_t* topk_cand = nullptr;   // [num_sms x kTopkMax] candidate keys of the top-k kernel
    uint32_t* topk_counter = nullptr;
    uint32_t* topk_ids = nullptr;    // [kTopkMax] results of the host LM-head entry points
    float* topk_vals = nullptr;
    int64_t* amax_index = nullptr;
    float* amax_value = nullptr;
    uint32_t* topk_ids_pin = nullptr;
    float* topk_vals_pin = nullptr;
    cudaStream_t stream = nullptr;   // for the host-pointer entry points
    float* x_dev = nullptr;
    float* y_dev = nullptr;
    uint64_t x_cap = 0, y_cap = 0;
    float* x_pin = nullptr;
    float* y_pin = nullptr;
    uint64_t xp_cap = 0, yp_cap = 0;
    DeviceStatus* status_pin = nullptr;
    __half* xh = nullptr;  // fp16 copy of the token vectors for the tensor-core GEMM
    uint64_t xh_cap = 0;
    float* splitk_ws = nullptr;  // split-K partial sums of the tensor-core GEMM
    uint64_t splitk_cap = 0;
    // Buffers a larger call replaced.  A CUDA graph captured earlier may still
    // name them, so they are freed only by nedo_gpu_cache_clear.
    std::vector<void*> retired;
    uint8_t* upload_pin[2] = {nullptr, nullptr};  // pinned bounce buffers of weight uploads
    cudaEvent_t upload_done[2] = {nullptr, nullptr};
    uint64_t wait_limit_ns = 0;  // 0 = the kernels' default bound
    std::unordered_map<const void*, Resident> cache;
    std::mutex mu;
};

std::mutex g_states_mu;
std::vector<DeviceState*> g_states;
std::atomic<int> g_pdl{0};
std::atomic<int> g_exact_batches{0};

int current_device(int* dev) {
    cudaError_t e = cudaGetDevice(dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    return 0;
}

int get_state(DeviceState** out) {
    int dev = 0;
    if (int rc = current_device(&dev)) return rc;
    std::lock_guard<std::mutex> lk(g_states_mu);
    if (static_cast<int>(g_states.size()) <= dev) g_states.resize(dev + 1, nullptr);
    if (g_states[dev] != nullptr) {
        *out = g_states[dev];
        return 0;
    }
    auto* s = new DeviceState();
    s->device = dev;
    NEDO_CUDA_TRY(cudaDeviceGetAttribute(&s->num_sms, cudaDevAttrMultiProcessorCount, dev));
    NEDO_CUDA_TRY(cudaDeviceGetAttribute(&s->max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
    NEDO_CUDA_TRY(cudaMalloc(&s->status, sizeof(DeviceStatus)));
    NEDO_CUDA_TRY(cudaMemset(s->status, 0, sizeof(DeviceStatus)));
    const size_t n = static_cast<size_t>(s->num_sms) + 1;
    NEDO_CUDA_TRY(cudaMalloc(&s->scratch.cand_val, n * sizeof(float)));
    NEDO_CUDA_TRY(cudaMalloc(&s->scratch.cand_idx, n * sizeof(uint32_t)));
    NEDO_CUDA_TRY(cudaMalloc(&s->scratch.counter, sizeof(uint32_t)));
    NEDO_CUDA_TRY(cudaMemset(s->scratch.counter, 0, sizeof(uint32_t)));
    NEDO_CUDA_TRY(cudaStreamCreateWithFlags(&s->stream, cudaStreamNonBlocking));
    NEDO_CUDA_TRY(cudaHostAlloc(&s->status_pin, sizeof(DeviceStatus), cudaHostAllocDefault));
    NEDO_CUDA_TRY(cudaMalloc(&s->topk_cand, static_cast<size_t>(s->num_sms) * kTopkMax * sizeof(uint64_t)));
    NEDO_CUDA_TRY(cudaMalloc(&s->topk_counter, sizeof(uint32_t)));
    NEDO_CUDA_TRY(cudaMemset(s->topk_counter, 0, sizeof(uint32_t)));
    NEDO_CUDA_TRY(cudaMalloc(&s->topk_ids, kTopkMax * sizeof(uint32_t)));
    NEDO_CUDA_TRY(cudaMalloc(&s->topk_vals, kTopkMax * sizeof(float)));
    NEDO_CUDA_TRY(cudaMalloc(&s->amax_index, sizeof(int64_t) + sizeof(float)));
    s->amax_value = reinterpret_cast<float*>(s->amax_index + 1);
    NEDO_CUDA_TRY(cudaHostAlloc(&s->topk_ids_pin, kTopkMax * (sizeof(uint32_t) + sizeof(float)) + 16,
                                cudaHostAllocDefault));
    s->topk_vals_pin = reinterpret_cast<float*>(s->topk_ids_pin + kTopkMax);
    g_states[dev] = s;
    *out = s;
    return 0;
}

bool is_matvec_type(uint32_t t) { return t == kF16 || t == kQ4_0 || t == kQ8_0; }

// tensor_nbytes semantics (src/gguf.cpp:106-114) for the types it knows.
int tensor_row_bytes(uint32_t type, uint64_t cols, uint64_t* rb) {
    switch (type) {
        case 0: *rb = cols * 4; return 0;                      // F32
        case 1: *rb = cols * 2; return 0;                      // F16
        case 30: *rb = cols * 2; return 0;                     // BF16
        case 2:
            if (cols % 32) return fail(NEDO_GPU_ERR_ALIGN, "Q4_0 elements not block aligned");
            *rb = cols / 32 * 18;
            return 0;
        case 8:
            if (cols % 32) return fail(NEDO_GPU_ERR_ALIGN, "Q8_0 elements not block aligned");
            *rb = cols / 32 * 34;
            return 0;
        case 24: *rb = cols; return 0;      // I8
        case 25: *rb = cols * 2; return 0;  // I16
        case 26: *rb = cols * 4; return 0;  // I32
        case 27: *rb = cols * 8; return 0;  // I64
        default: return fail(NEDO_GPU_ERR_TYPE, "tensor type not implemented: " + std::to_string(type));
    }
}

int check_matvec_args(uint32_t type, uint64_t rows, uint64_t cols, uint64_t* rb) {
    if (int rc = tensor_row_bytes(type, cols, rb)) return rc;
    if (rows > 0 && !is_matvec_type(type)) return fail(NEDO_GPU_ERR_TYPE, "matvec tensor type not supported");
    if (rows > 0xFFFFFFFFull) return fail(NEDO_GPU_ERR_ARG, "matvec: more than 2^32-1 rows");
    return 0;
}

template <typename T>
int ensure_dev(T** p, uint64_t* cap, uint64_t need) {
    if (*cap >= need) return 0;
    if (*p) cudaFree(*p);
    *p = nullptr;
    *cap = 0;
    cudaError_t e = cudaMalloc(reinterpret_cast<void**>(p), need * sizeof(T));
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(staging)");
    *cap = need;
    return 0;
}

// Like ensure_dev for buffers that device entry points hand to kernels a
// caller may capture in a CUDA graph: a buffer that is outgrown is retired
// (kept allocated until nedo_gpu_cache_clear) instead of freed, so a graph
// captured with it stays valid.
template <typename T>
int ensure_dev_retiring(DeviceState* s, T** p, uint64_t* cap, uint64_t need) {
    if (*cap >= need) return 0;
    T* fresh = nullptr;
    cudaError_t e = cudaMalloc(reinterpret_cast<void**>(&fresh), need * sizeof(T));
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(batched-call buffer)");
    if (*p) s->retired.push_back(*p);
    *p = fresh;
    *cap = need;
    return 0;
}

template <typename T>
int ensure_pin(T** p, uint64_t* cap, uint64_t need) {
    if (*cap >= need) return 0;
    if (*p) cudaFreeHost(*p);
    *p = nullptr;
    *cap = 0;
    cudaError_t e = cudaHostAlloc(reinterpret_cast<void**>(p), need * sizeof(T), cudaHostAllocDefault);
    if (e != cudaSuccess) return cuda_fail(e, "cudaHostAlloc(staging)");
    *cap = need;
    return 0;
}

// A cheap content check of a host weight buffer: 64-bit mix of its first and
// last 4 KB and of 64 evenly spaced 64-byte samples (about 12 KB read per
// call).  The residency cache compares it on every host call, so a buffer
// freed and reallocated at the same address with the same size but other
// bytes (a second model mapped where the first was) is uploaded again instead
// of being served from the stale device copy.
uint64_t content_fingerprint(const void* p, uint64_t n) {
    const auto* b = static_cast<const uint8_t*>(p);
    uint64_t h = 0x9E3779B97F4A7C15ull ^ n;
    auto mix = [&h](const uint8_t* q, uint64_t len) {
        uint64_t i = 0;
        for (; i + 8 <= len; i += 8) {
            uint64_t v;
            std::memcpy(&v, q + i, 8);
            h = (h ^ v) * 0xFF51AFD7ED558CCDull;
            h ^= h >> 32;
        }
        for (; i < len; ++i) h = (h ^ q[i]) * 0x100000001B3ull;
    };
    const uint64_t edge = 4096;
    if (n <= 2 * edge + 64 * 64) {
        mix(b, n);
        return h;
    }
    mix(b, edge);
    mix(b + n - edge, edge);
    const uint64_t step = (n - 2 * edge) / 64;
    for (uint64_t k = 0; k < 64; ++k) mix(b + edge + k * step, 64);
    return h;
}

// Host weight -> device through two pinned bounce buffers: the copy of chunk
// i+1 into one buffer overlaps the DMA of chunk i from the other (a pageable
// cudaMemcpy stages through a driver buffer one chunk at a time).
constexpr uint64_t kUploadChunk = 8ull << 20;

int upload_weight(DeviceState* s, void* dst, const void* src, uint64_t n) {
    for (int k = 0; k < 2; ++k) {
        if (s->upload_pin[k] == nullptr) {
            NEDO_CUDA_TRY(cudaHostAlloc(reinterpret_cast<void**>(&s->upload_pin[k]), kUploadChunk,
                                        cudaHostAllocDefault));
            NEDO_CUDA_TRY(cudaEventCreateWithFlags(&s->upload_done[k], cudaEventDisableTiming));
        }
    }
    const auto* in = static_cast<const uint8_t*>(src);
    auto* out = static_cast<uint8_t*>(dst);
    uint64_t off = 0;
    for (uint32_t i = 0; off < n; ++i) {
        const uint32_t k = i & 1u;
        const uint64_t len = n - off < kUploadChunk ? n - off : kUploadChunk;
        // the DMA that last read this buffer is done before it is refilled
        NEDO_CUDA_TRY(cudaEventSynchronize(s->upload_done[k]));
        std::memcpy(s->upload_pin[k], in + off, len);
        NEDO_CUDA_TRY(cudaMemcpyAsync(out + off, s->upload_pin[k], len, cudaMemcpyHostToDevice, s->stream));
        NEDO_CUDA_TRY(cudaEventRecord(s->upload_done[k], s->stream));
        off += len;
    }
    NEDO_CUDA_TRY(cudaStreamSynchronize(s->stream));
    return 0;
}

int resident_weight(DeviceState* s, const void* w_host, uint64_t w_bytes, const void** w_dev) {
    const uint64_t fp = content_fingerprint(w_host, w_bytes);
    auto it = s->cache.find(w_host);
    if (it != s->cache.end() && it->second.bytes == w_bytes && it->second.fingerprint == fp) {
        *w_dev = it->second.dev;
        return 0;
    }
    if (it != s->cache.end()) {
        release_resident(it->second);
        s->cache.erase(it);
    }
    void* d = nullptr;
    cudaError_t e = cudaMalloc(&d, w_bytes ? w_bytes : 16);
    if (e == cudaErrorMemoryAllocation) {
        // Out of room: drop every other resident weight and retry once.
        cudaGetLastError();
        for (auto& kv : s->cache) release_resident(kv.second);
        s->cache.clear();
        e = cudaMalloc(&d, w_bytes ? w_bytes : 16);
    }
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(weight)");
    if (w_bytes) {
        if (int rc = upload_weight(s, d, w_host, w_bytes)) {
            cudaFree(d);
            return rc;
        }
    }
    Resident r;
    r.dev = d;
    r.bytes = w_bytes;
    r.fingerprint = fp;
    s->cache[w_host] = r;
    *w_dev = d;
    return 0;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Batches of at least this many token vectors run as one tensor-core GEMM, for
// rows of at least kTensorCoreMinCols elements.  The GEMM rounds x and d*q to fp16
// (worst case 2 * 2^-11 * sum|w*x| per output); its errors average out over the
// row, and rows of 1024 elements and more keep them inside 1e-4 * sum|w*x| on
// the test distributions.  Shorter rows use the exact int8 kernel.
constexpr uint32_t kTensorCoreMinBatch = 16;
// F16 weights are exact in the GEMM (only x is rounded), and the alternative is
// one streaming pass over the weight per token vector: from 4 vectors on one
// GEMM pass is cheaper (an F16 64000x1536 head at 8 vectors: ~43 us against
// 8 x 30 us).
constexpr uint32_t kTensorCoreMinBatchF16 = 4;

uint32_t tensor_core_min_batch(uint32_t type) { return type == kF16 ? kTensorCoreMinBatchF16 : kTensorCoreMinBatch; }
constexpr uint64_t kTensorCoreMinCols = 1024;

// The tcgen05 batch-1 kernel (gemv_tc8.cu) for the shapes it takes, when the
// environment variable NEDO_GPU_TC8=1 is set (otherwise the int8 mma.sync
// kernel of gemv_imma.cu runs them).
bool tc8_enabled() {
    static const bool on = [] {
        const char* v = std::getenv("NEDO_GPU_TC8");
        return v != nullptr && std::strcmp(v, "1") == 0;
    }();
    return on;
}

// Most token vectors one multi-vector launch takes.
constexpr uint32_t kMultiMaxVectors = 32;

// NEDO_GPU_IMMA_MULTI: "0" keeps small batches on the ring kernel (for
// comparisons), "2" / "4" / "8" fixes the vectors per token group (-1, 0 or
// that number).
int multi_vectors_per_group() {
    static const int v = [] {
        const char* e = std::getenv("NEDO_GPU_IMMA_MULTI");
        if (e == nullptr || e[0] == '\0') return 0;
        if (std::strcmp(e, "0") == 0) return -1;
        const int n = std::atoi(e);
        return n == 2 || n == 4 || n == 8 ? n : 0;
    }();
    return v;
}

// Small batches of Q8_0 / Q4_0 rows run on the multi-vector resident slice
// when it plans 2 vectors (or the fixed group size).
bool multi_applies(DeviceState* s, uint32_t type, uint64_t rows, uint64_t cols) {
    if ((type != kQ8_0 && type != kQ4_0) || multi_vectors_per_group() < 0) return false;
    const uint32_t g = multi_vectors_per_group();
    return plan_imma_multi(type, rows, cols, s->num_sms, s->max_smem, g > 0 ? g : 2u, g).ok;
}

// A batch of at most kMultiMaxVectors vectors that one multi-vector launch
// takes whole: it runs there rather than on the fp16 GEMM (exact int8 block
// dots, and one launch instead of the GEMM's conversion, GEMM and fold).
bool multi_takes_whole_batch(DeviceState* s, uint32_t type, uint64_t rows, uint64_t cols, uint32_t batch) {
    return batch >= 2 && batch <= kMultiMaxVectors && multi_applies(s, type, rows, cols) &&
           plan_imma_multi(type, rows, cols, s->num_sms, s->max_smem, batch, multi_vectors_per_group()).ok;
}

// The launches of a batch on the multi-vector slice, in order: launches of up
// to kMultiMaxVectors vectors (the most that plan), each(&plan, first, n), and
// single vectors (each(nullptr, first, 1)) for the rest.
template <typename F>
void for_each_multi_launch(DeviceState* s, uint32_t type, uint64_t rows, uint64_t cols, uint32_t batch, F&& each) {
    for (uint32_t b = 0; b < batch;) {
        const uint32_t left = batch - b;
        ImmaPlan mp;
        for (uint32_t n = left < kMultiMaxVectors ? left : kMultiMaxVectors; n >= 2 && !mp.ok; --n)
            mp = plan_imma_multi(type, rows, cols, s->num_sms, s->max_smem, n, multi_vectors_per_group());
        if (!mp.ok) {
            // one vector left, or none of the fixed group size
            for (uint32_t k = 0; k < left; ++k) each(static_cast<const ImmaPlan*>(nullptr), b + k, 1u);
            return;
        }
        const uint32_t n = mp.tokens * mp.token_groups;
        each(static_cast<const ImmaPlan*>(&mp), b, n);
        b += n;
    }
}

// The one dispatch point for every matvec launch.
int dispatch_matvec(DeviceState* s, uint32_t type, uint64_t rows, uint64_t cols, const void* w, const float* x,
                    float* y, uint32_t batch, const ArgmaxScratch* amax, cudaStream_t stream, int pdl_override = -1) {
    if (rows == 0 || batch == 0) return 0;
    const bool use_pdl = pdl_override < 0 ? g_pdl.load() != 0 : pdl_override != 0;
    if (batch == 1 && amax == nullptr && aligned16(w) && aligned16(x) && (type == kQ8_0 || type == kQ4_0) &&
        tc8_enabled()) {
        Tc8Plan tp = plan_tc8(type, rows, cols, s->num_sms, s->max_smem);
        if (tp.ok) {
            cudaError_t e = launch_tc8(tp, w, x, y, s->status, stream, use_pdl);
            if (e != cudaSuccess) return cuda_fail(e, "gemv_tc8 launch");
            return 0;
        }
    }
    if (batch == 1 && amax == nullptr && aligned16(w) && aligned16(x) && (type == kQ8_0 || type == kQ4_0)) {
        ImmaPlan ip = plan_imma(type, rows, cols, s->num_sms, s->max_smem);
        if (ip.ok) {
            cudaError_t e = launch_imma(ip, w, x, y, rows, cols, s->status, stream, use_pdl);
            if (e != cudaSuccess) return cuda_fail(e, "gemv_imma launch");
            return 0;
        }
    }
    if (batch == 1 && aligned16(w) && aligned16(x)) {
        StreamPlan plan = plan_stream(type, rows, cols, s->num_sms, s->max_smem);
        if (plan.ok) {
            cudaError_t e = launch_stream(type, plan, w, x, y, rows, cols, s->status, amax, stream, use_pdl);
            if (e != cudaSuccess) return cuda_fail(e, "gemv_stream launch");
            return 0;
        }
    }
    if (g_exact_batches.load() == 0 && batch >= tensor_core_min_batch(type) && cols >= kTensorCoreMinCols &&
        amax == nullptr && aligned16(w) && aligned16(x) && gemm_tc_supported(type, rows, cols, batch) &&
        !multi_takes_whole_batch(s, type, rows, cols, batch)) {
        // tokens as the N dimension of a tcgen05 GEMM (x rounded to fp16 once)
        const uint64_t n = static_cast<uint64_t>(batch) * cols;
        const uint32_t splits = gemm_tc_splits(rows, cols, batch, s->num_sms);
        if (int rc = ensure_dev_retiring(s, &s->xh, &s->xh_cap, n)) return rc;
        if (splits > 1) {
            if (int rc = ensure_dev_retiring(s, &s->splitk_ws, &s->splitk_cap,
                                             static_cast<uint64_t>(splits) * batch * rows))
                return rc;
        }
        cudaError_t e = launch_x_to_f16(x, s->xh, n, s->num_sms, stream, use_pdl);
        if (e != cudaSuccess) return cuda_fail(e, "x to fp16 launch");
        if (splits > 1) {
            // few tiles: K shared among CTAs, partial sums folded in split order
            e = launch_gemm_tc(type, w, s->xh, s->splitk_ws, rows, cols, batch, rows, s->status, stream, use_pdl,
                               splits, static_cast<uint64_t>(batch) * rows);
            if (e != cudaSuccess) return cuda_fail(e, "gemm_tc launch");
            e = launch_splitk_reduce(s->splitk_ws, y, splits, batch, rows, rows, s->num_sms, stream, use_pdl);
            if (e != cudaSuccess) return cuda_fail(e, "split-K fold launch");
            return 0;
        }
        e = launch_gemm_tc(type, w, s->xh, y, rows, cols, batch, rows, s->status, stream, use_pdl);
        if (e != cudaSuccess) return cuda_fail(e, "gemm_tc launch");
        return 0;
    }
    if (batch > 1 && amax == nullptr && aligned16(w) && aligned16(x) && multi_applies(s, type, rows, cols)) {
        // small batches of quantised rows on the multi-vector resident slice
        int rc = 0;
        for_each_multi_launch(s, type, rows, cols, batch, [&](const ImmaPlan* mp, uint32_t b, uint32_t n) {
            const float* xb = x + static_cast<uint64_t>(b) * cols;
            float* yb = y + static_cast<uint64_t>(b) * rows;
            if (rc) return;
            if (mp == nullptr) {
                rc = dispatch_matvec(s, type, rows, cols, w, xb, yb, 1, nullptr, stream, pdl_override);
                return;
            }
            cudaError_t e = launch_imma(*mp, w, xb, yb, rows, cols, s->status, stream, use_pdl, nullptr, cols, rows);
            if (e != cudaSuccess) rc = cuda_fail(e, "gemv_imma multi-vector launch");
            (void)n;
        });
        return rc;
    }
    if (batch > 1 && amax == nullptr && aligned16(w) && aligned16(x) && (type == kQ8_0 || type == kQ4_0)) {
        // small batches of quantised rows: the int8 tensor-pipe kernel with up to 8
        // token vectors per launch (each weight unit read once for all of them)
        ImmaPlan plans[4];
        bool ok = true;
        for (uint32_t i = 0; i < 4 && ok; ++i) {
            plans[i] = plan_imma(type, rows, cols, s->num_sms, s->max_smem, nullptr, 1u << i);
            ok = plans[i].ok;
        }
        if (ok) {
            for (uint32_t b = 0; b < batch;) {
                uint32_t i = 3;
                while ((1u << i) > batch - b) --i;
                cudaError_t e = launch_imma(plans[i], w, x + static_cast<uint64_t>(b) * cols,
                                            y + static_cast<uint64_t>(b) * rows, rows, cols, s->status, stream,
                                            use_pdl, nullptr, cols, rows);
                if (e != cudaSuccess) return cuda_fail(e, "gemv_imma launch");
                b += 1u << i;
            }
            return 0;
        }
    }
    if (batch > 1 && aligned16(w) && aligned16(x) && (cols * sizeof(float)) % 16 == 0) {
        StreamPlan plan = plan_stream(type, rows, cols, s->num_sms, s->max_smem);
        if (plan.ok) {
            for (uint32_t b = 0; b < batch; ++b) {
                cudaError_t e = launch_stream(type, plan, w, x + static_cast<uint64_t>(b) * cols,
                                              y + static_cast<uint64_t>(b) * rows, rows, cols, s->status, nullptr,
                                              stream, use_pdl);
                if (e != cudaSuccess) return cuda_fail(e, "gemv_stream launch");
            }
            return 0;
        }
    }
    cudaError_t e = launch_generic(type, w, x, y, rows, cols, batch, cols, rows, stream);
    if (e != cudaSuccess) return cuda_fail(e, "gemv_generic launch");
    if (amax) {
        e = launch_argmax(y, rows, const_cast<ArgmaxScratch*>(amax), s->num_sms, stream);
        if (e != cudaSuccess) return cuda_fail(e, "argmax launch");
    }
    return 0;
}

// Reset the failure flags and site of the device status word (its wait bound stays).
void clear_status_flags(DeviceState* s, cudaStream_t stream) {
    cudaMemsetAsync(s->status, 0, 2 * sizeof(uint32_t), stream);
    cudaStreamSynchronize(stream);
}

int read_status(DeviceState* s, cudaStream_t stream) {
    NEDO_CUDA_TRY(cudaMemcpyAsync(s->status_pin, s->status, sizeof(DeviceStatus), cudaMemcpyDeviceToHost, stream));
    NEDO_CUDA_TRY(cudaStreamSynchronize(stream));
    if (s->status_pin->flags != 0) {
        const DeviceStatus st = *s->status_pin;
        clear_status_flags(s, stream);
        char buf[160];
        std::snprintf(buf, sizeof(buf), "device kernel gave up on a bounded wait (flags=0x%x, site=%u)", st.flags,
                      st.where);
        return fail(NEDO_GPU_ERR_DEVICE, buf);
    }
    return 0;
}

// ---- argmax without any allocation --------------------------------------
// The per-CTA candidates and the completion counter of the argmax kernel live
// in this file-scope array instead of the per-device cudaMalloc'd scratch.
// Layout: cand_val[kNoAllocMaxCtas] (float), cand_idx[kNoAllocMaxCtas]
// (uint32), counter (uint32, padded to 256 bytes).  Only the counter must be
// zero before a launch: the array is zero at module load and the last CTA of
// every launch resets the counter to zero.
constexpr uint32_t kNoAllocMaxCtas = 1024;
constexpr size_t kNoAllocScratchBytes = 2u * kNoAllocMaxCtas * 4u + 256u;  // 8448
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kNoAllocMaxDevices = 64;
struct NoAllocSlot {
    uint8_t* scratch = nullptr;  // device address of g_noalloc_scratch on this device
    int num_sms = 0;
};
std::mutex g_noalloc_mu;
NoAllocSlot g_noalloc[kNoAllocMaxDevices];

// Once per device: resolve the scratch address and the SM count.
int noalloc_setup(NoAllocSlot* out) {
    int dev = 0;
    if (int rc = current_device(&dev)) return rc;
    if (dev < 0 || dev >= kNoAllocMaxDevices)
        return fail(NEDO_GPU_ERR_DEVICE, "argmax_dev_noalloc: device ordinal above 63");
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    NoAllocSlot& s = g_noalloc[dev];
    if (s.scratch == nullptr) {
        int sms = 0;
        NEDO_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
        void* p = nullptr;
        NEDO_CUDA_TRY(cudaGetSymbolAddress(&p, g_noalloc_scratch));
        s.num_sms = sms;
        s.scratch = static_cast<uint8_t*>(p);
    }
    *out = s;
    return 0;
}

}  // namespace

extern "C" {

int nedo_gpu_version(void) { return 100; }

int nedo_gpu_set_pdl(int enable) {
    const int prev = g_pdl.exchange(enable != 0 ? 1 : 0);
    return prev;
}

int nedo_gpu_set_exact_batches(int enable) { return g_exact_batches.exchange(enable != 0 ? 1 : 0); }

const char* nedo_gpu_last_error(void) { return g_last_error.c_str(); }

int nedo_gpu_matvec(uint32_t type, uint64_t rows, uint64_t cols, const void* w_host, uint64_t w_bytes,
                    const float* x_host, float* y_host) {
    uint64_t rb = 0;
    if (int rc = check_matvec_args(type, rows, cols, &rb)) return rc;
    if (rows == 0) return 0;
    if (!w_host || !x_host || !y_host) return fail(NEDO_GPU_ERR_ARG, "matvec: null pointer");
    if (w_bytes < rows * rb) return fail(NEDO_GPU_ERR_ARG, "matvec: weight span shorter than rows * row_bytes");
    DeviceState* s = nullptr;
    if (int rc = get_state(&s)) return rc;
    std::lock_guard<std::mutex> lk(s->mu);
    const void* w_dev = nullptr;
    if (int rc = resident_weight(s, w_host, w_bytes, &w_dev)) return rc;
    if (int rc = ensure_dev(&s->x_dev, &s->x_cap, cols)) return rc;
    if (int rc = ensure_dev(&s->y_dev, &s->y_cap, rows)) return rc;
    if (int rc = ensure_pin(&s->x_pin, &s->xp_cap, cols)) return rc;
    if (int rc = ensure_pin(&s->y_pin, &s->yp_cap, rows)) return rc;
    std::memcpy(s->x_pin, x_host, cols * sizeof(float));
    // The call as one sequence on the library's stream: x up, matvec, y and the
    // status word down.  The first call on a weight runs it eagerly; later calls
    // replay a CUDA graph of it (one launch instead of four).
    Resident& r = s->cache[w_host];
    const void* bufs[5] = {s->x_dev, s->y_dev, s->x_pin, s->y_pin, s->status_pin};
    auto enqueue = [&]() -> int {
        NEDO_CUDA_TRY(cudaMemcpyAsync(s->x_dev, s->x_pin, cols * sizeof(float), cudaMemcpyHostToDevice, s->stream));
        if (int rc = dispatch_matvec(s, type, rows, cols, w_dev, s->x_dev, s->y_dev, 1, nullptr, s->stream, 0))
            return rc;
        NEDO_CUDA_TRY(cudaMemcpyAsync(s->y_pin, s->y_dev, rows * sizeof(float), cudaMemcpyDeviceToHost, s->stream));
        NEDO_CUDA_TRY(
            cudaMemcpyAsync(s->status_pin, s->status, sizeof(DeviceStatus), cudaMemcpyDeviceToHost, s->stream));
        return 0;
    };
    const bool replay = r.call != nullptr && r.type == type && r.rows == rows && r.cols == cols &&
                        std::equal(bufs, bufs + 5, r.bufs);
    if (replay) {
        NEDO_CUDA_TRY(cudaGraphLaunch(r.call, s->stream));
    } else {
        if (r.call) cudaGraphExecDestroy(r.call);
        r.call = nullptr;
        if (int rc = enqueue()) return rc;
        // capture the same sequence for the next calls (a failure only costs the replay)
        cudaGraph_t g = nullptr;
        if (cudaStreamBeginCapture(s->stream, cudaStreamCaptureModeThreadLocal) == cudaSuccess) {
            const int rc = enqueue();
            const cudaError_t ec = cudaStreamEndCapture(s->stream, &g);
            if (rc == 0 && ec == cudaSuccess && g != nullptr &&
                cudaGraphInstantiate(&r.call, g, 0) == cudaSuccess) {
                r.type = type;
                r.rows = rows;
                r.cols = cols;
                std::copy(bufs, bufs + 5, r.bufs);
            } else {
                r.call = nullptr;
            }
            if (g) cudaGraphDestroy(g);
            cudaGetLastError();
        }
    }
    NEDO_CUDA_TRY(cudaStreamSynchronize(s->stream));
    if (s->status_pin->flags != 0) {
        const DeviceStatus st = *s->status_pin;
        clear_status_flags(s, s->stream);
        char buf[160];
        std::snprintf(buf, sizeof(buf), "device kernel gave up on a bounded wait (flags=0x%x, site=%u)", st.flags,
                      st.where);
        return fail(NEDO_GPU_ERR_DEVICE, buf);
    }
    std::memcpy(y_host, s->y_pin, rows * sizeof(float));
    return 0;
}

int nedo_gpu_embedding_row(uint32_t type, uint64_t rows, uint64_t cols, const void* w_host, uint64_t w_bytes,
                           uint32_t row, float* out_host) {
    if (row >= rows) return fail(NEDO_GPU_ERR_ROW, "bad embedding row");
    uint64_t rb = 0;
    if (int rc = tensor_row_bytes(type, cols, &rb)) return rc;
    if (!is_matvec_type(type)) return fail(NEDO_GPU_ERR_TYPE, "embedding type unsupported");
    if (!w_host || !out_host) return fail(NEDO_GPU_ERR_ARG, "embedding_row: null pointer");
    if (w_bytes < rows * rb) return fail(NEDO_GPU_ERR_ARG, "embedding_row: weight span shorter than rows * row_bytes");
    DeviceState* s = nullptr;
    if (int rc = get_state(&s)) return rc;
    std::lock_guard<std::mutex> lk(s->mu);
    const void* w_dev = nullptr;
    if (int rc = resident_weight(s, w_host, w_bytes, &w_dev)) return rc;
    if (int rc = ensure_dev(&s->y_dev, &s->y_cap, cols)) return rc;
    if (int rc = ensure_pin(&s->y_pin, &s->yp_cap, cols)) return rc;
    cudaError_t e = launch_dequant_rows(type, w_dev, rows, cols, row, 1, s->y_dev, s->stream);
    if (e != cudaSuccess) return cuda_fail(e, "dequant launch");
    NEDO_CUDA_TRY(cudaMemcpyAsync(s->y_pin, s->y_dev, cols * sizeof(float), cudaMemcpyDeviceToHost, s->stream));
    NEDO_CUDA_TRY(cudaStreamSynchronize(s->stream));
    std::memcpy(out_host, s->y_pin, cols * sizeof(float));
    return 0;
}

int nedo_gpu_weight_upload(const void* w_host, uint64_t w_bytes, const void** w_dev_out) {
    if (!w_host || !w_dev_out) return fail(NEDO_GPU_ERR_ARG, "weight_upload: null pointer");
    DeviceState* s = nullptr;
    if (int rc = get_state(&s)) return rc;
    std::lock_guard<std::mutex> lk(s->mu);
    return resident_weight(s, w_host, w_bytes, w_dev_out);
}

int nedo_gpu_weight_evict(const void* w_host) {
    DeviceState* s = nullptr;
    if (int rc = get_state(&s)) return rc;
    std::lock_guard<std::mutex> lk(s->mu);
    auto it = s->cache.find(w_host);
    if (it != s->cache.end()) {
        release_resident(it->second);
        s->cache.erase(it);
    }
    return 0;
}

int nedo_gpu_cache_clear(void) {
    std::lock_guard<std::mutex> lk(g_states_mu);
    int prev = 0;
    cudaGetDevice(&prev);
    for (DeviceState* s : g_states) {
        if (s == nullptr) continue;
        std::lock_guard<std::mutex> lk2(s->mu);
        cudaSetDevice(s->device);
        for (auto& kv : s->cache) release_resident(kv.second);
        s->cache.clear();
        for (void* p : s->retired) cudaFree(p);
        s->retired.clear();
    }
    cudaSetDevice(prev);
    return 0;
}

int nedo_gpu_set_wait_limit_ns(uint64_t ns) {
    DeviceState* s = nullptr;
    if (int rc = get_state(&s)) return rc;
    std::lock_guard<std::mutex> lk(s->mu);
    NEDO_CUDA_TRY(cudaMemcpy(&s->status->wait_limit_ns, &ns, sizeof(ns), cudaMemcpyHostToDevice));
    s->wait_limit_ns = ns;
    return 0;
}

int nedo_gpu_reserve(uint32_t type, uint64_t rows, uint64_t cols, uint32_t batch) {
    uint64_t rb = 0;
    if (int rc = check_matvec_args(type, rows, cols, &rb)) return rc;
    DeviceState* s = nullptr;
    if (int rc = get_state(&s)) return rc;
    if (rows == 0 || batch < tensor_core_min_batch(type) || cols < kTensorCoreMinCols ||
        !gemm_tc_supported(type, rows, cols, batch))
        return 0;  // this shape needs no shared buffer
    if (int rc = ensure_dev_retiring(s, &s->xh, &s->xh_cap, static_cast<uint64_t>(batch) * cols)) return rc;
    const uint32_t splits = gemm_tc_splits(rows, cols, batch, s->num_sms);
    if (splits > 1)
        if (int rc = ensure_dev_retiring(s, &s->splitk_ws, &s->splitk_cap,
                                         static_cast<uint64_t>(splits) * batch * rows))
            return rc;
    return 0;
}

int nedo_gpu_matvec_batch(uint32_t type, uint64_t rows, uint64_t cols, const void* w_host, uint64_t w_bytes,
                          const float* x_host, float* y_host, uint32_t batch) {
    uint64_t rb = 0;
    if (int rc = check_matvec_args(type, rows, cols, &rb)) return rc;
    if (rows == 0 || batch == 0) return 0;
    if (!w_host || !x_host || !y_host) return fail(NEDO_GPU_ERR_ARG, "matvec_batch: null pointer");
    if (w_bytes < rows * rb) return fail(NEDO_GPU_ERR_ARG, "matvec: weight span shorter than rows * row_bytes");
    DeviceState* s = nullptr;
    if (int rc = get_state(&s)) return rc;
    std::lock_guard<std::mutex> lk(s->mu);
    const void* w_dev = nullptr;
    if (int rc = resident_weight(s, w_host, w_bytes, &w_dev)) return rc;
    const uint64_t nx = static_cast<uint64_t>(batch) * cols, ny = static_cast<uint64_t>(batch) * rows;
    if (int rc = ensure_dev(&s->x_dev, &s->x_cap, nx)) return rc;
    if (int rc = ensure_dev(&s->y_dev, &s->y_cap, ny)) return rc;
    if (int rc = ensure_pin(&s->x_pin, &s->xp_cap, nx)) return rc;
    if (int rc = ensure_pin(&s->y_pin, &s->yp_cap, ny)) return rc;
    std::memcpy(s->x_pin, x_host, nx * sizeof(float));
    NEDO_CUDA_TRY(cudaMemcpyAsync(s->x_dev, s->x_pin, nx * sizeof(float), cudaMemcpyHostToDevice, s->stream));
    if (int rc = dispatch_matvec(s, type, rows, cols, w_dev, s->x_dev, s->y_dev, batch, nullptr, s->stream, 0))
        return rc;
    NEDO_CUDA_TRY(cudaMemcpyAsync(s->y_pin, s->y_dev, ny * sizeof(float), cudaMemcpyDeviceToHost, s->stream));
    if (int rc = read_status(s, s->stream)) return rc;
    std::memcpy(y_host, s->y_pin, ny * sizeof(float));
    return 0;
}

int nedo_gpu_matvec_dev(uint32_t type, uint64_t rows, uint64_t cols, const void* w_dev, const float* x_dev,
                        float* y_dev, uint32_t batch, void* stream) {
    uint64_t rb = 0;
    if (int rc = check_matvec_args(type, rows, cols, &rb)) return rc;
    if (rows == 0 || batch == 0) return 0;
    if (!w_dev || !x_dev || !y_dev) return fail(NEDO_GPU_ERR_ARG, "matvec_dev: null pointer");
    DeviceState* s = nullptr;
    if (int rc = get_state(&s)) return rc;
    return dispatch_matvec(s, type, rows, cols, w_dev, x_dev, y_dev, batch, nullptr,
                           static_cast<cudaStream_t>(stream));
}

int nedo_gpu_matvec_argmax_dev(uint32_t type, uint64_t rows, uint64_t cols, const void* w_dev, const float* x_dev,
                               float* y_dev, int64_t* index_dev, float* value_dev, void* stream) {
    uint64_t rb = 0;
    if (int rc = check_matvec_args(type, rows, cols, &rb)) return rc;
    if (rows == 0) return fail(NEDO_GPU_ERR_ARG, "argmax of an empty vector");
    if (!w_dev || !x_dev || !y_dev || !index_dev) return fail(NEDO_GPU_ERR_ARG, "matvec_argmax_dev: null pointer");
    DeviceState* s = nullptr;
    if (int rc = get_state(&s)) return rc;
    ArgmaxScratch a = s->scratch;
    a.out_index = index_dev;
    a.out_value = value_dev;
    return dispatch_matvec(s, type, rows, cols, w_dev, x_dev, y_dev, 1, &a, static_cast<cudaStream_t>(stream));
}

int nedo_gpu_argmax_dev(const float* v_dev, uint64_t n, int64_t* index_dev, float* value_dev, void* stream) {
    if (n == 0) return fail(NEDO_GPU_ERR_ARG, "argmax of an empty vector");
    if (n > 0xFFFFFFFFull) return fail(NEDO_GPU_ERR_ARG, "argmax: more than 2^32-1 elements");
    if (!v_dev || !index_dev) return fail(NEDO_GPU_ERR_ARG, "argmax_dev: null pointer");
    DeviceState* s = nullptr;
    if (int rc = get_state(&s)) return rc;
    ArgmaxScratch a = s->scratch;
    a.out_index = index_dev;
    a.out_value = value_dev;
    cudaError_t e = launch_argmax(v_dev, n, &a, s->num_sms, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "argmax launch");
    return 0;
}

int nedo_gpu_argmax_dev_noalloc(const float* v_dev, uint64_t n, int64_t* index_dev, float* value_dev,
                                void* stream) {
    if (n == 0) return fail(NEDO_GPU_ERR_ARG, "argmax of an empty vector");
    if (n > 0xFFFFFFFFull) return fail(NEDO_GPU_ERR_ARG, "argmax: more than 2^32-1 elements");
    if (!v_dev || !index_dev) return fail(NEDO_GPU_ERR_ARG, "argmax_dev_noalloc: null pointer");
    NoAllocSlot s;
    if (int rc = noalloc_setup(&s)) return rc;
    // the same CTA count as launch_argmax: one candidate slot per CTA
    uint64_t ctas = (n + 1023) / 1024;
    if (ctas > static_cast<uint64_t>(s.num_sms)) ctas = static_cast<uint64_t>(s.num_sms);
    if (ctas > kNoAllocMaxCtas)
        return fail(NEDO_GPU_ERR_ARG, "argmax_dev_noalloc: needs " + std::to_string(ctas) +
                                          " candidate slots, the static scratch holds " +
                                          std::to_string(kNoAllocMaxCtas));
    ArgmaxScratch a{};
    a.cand_val = reinterpret_cast<float*>(s.scratch);
    a.cand_idx = reinterpret_cast<uint32_t*>(s.scratch + kNoAllocMaxCtas * 4u);
    a.counter = reinterpret_cast<uint32_t*>(s.scratch + 2u * kNoAllocMaxCtas * 4u);
    a.out_index = index_dev;
    a.out_value = value_dev;
    cudaError_t e = launch_argmax(v_dev, n, &a, s.num_sms, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "argmax launch");
    return 0;
}

int nedo_gpu_topk_dev(const float* v_dev, uint64_t n, uint32_t k, uint32_t* ids_dev, float* vals_dev, void* stream) {
    if (n == 0) return fail(NEDO_GPU_ERR_ARG, "topk of an empty vector");
    if (n > 0xFFFFFFFFull) return fail(NEDO_GPU_ERR_ARG, "topk: more than 2^32-1 elements");
    if (k == 0 || k > kTopkMax || k > n)
        return fail(NEDO_GPU_ERR_ARG, "topk: k must be in [1, min(n, " + std::to_string(kTopkMax) + ")]");
    if (!v_dev || !ids_dev) return fail(NEDO_GPU_ERR_ARG, "topk_dev: null pointer");
    DeviceState* s = nullptr;
    if (int rc = get_state(&s)) return rc;
    TopkScratch t{s->topk_cand, s->topk_counter, ids_dev, vals_dev};
    cudaError_t e = launch_topk(v_dev, n, k, t, s->num_sms, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "topk launch");
    return 0;
}

// Host-pointer LM head: x up, the matvec into the library's device y, then the
// greedy pick (k == 0) or the top k logits; only the result comes back.
static int lm_head_host(uint32_t type, uint64_t rows, uint64_t cols, const void* w_host, uint64_t w_bytes,
                 const float* x_host, uint32_t k, uint32_t* ids_host, float* vals_host, int64_t* index_host,
                 float* value_host) {
    uint64_t rb = 0;
    if (int rc = check_matvec_args(type, rows, cols, &rb)) return rc;
    if (rows == 0) return fail(NEDO_GPU_ERR_ARG, "LM head with no rows");
    if (!w_host || !x_host) return fail(NEDO_GPU_ERR_ARG, "lm_head: null pointer");
    if (w_bytes < rows * rb) return fail(NEDO_GPU_ERR_ARG, "matvec: weight span shorter than rows * row_bytes");
    if (k > kTopkMax || k > rows)
        return fail(NEDO_GPU_ERR_ARG, "lm_head_topk: k must be in [1, min(rows, " + std::to_string(kTopkMax) + ")]");
    DeviceState* s = nullptr;
    if (int rc = get_state(&s)) return rc;
    std::lock_guard<std::mutex> lk(s->mu);
    const void* w_dev = nullptr;
    if (int rc = resident_weight(s, w_host, w_bytes, &w_dev)) return rc;
    if (int rc = ensure_dev(&s->x_dev, &s->x_cap, cols)) return rc;
    if (int rc = ensure_dev(&s->y_dev, &s->y_cap, rows)) return rc;
    if (int rc = ensure_pin(&s->x_pin, &s->xp_cap, cols)) return rc;
    std::memcpy(s->x_pin, x_host, cols * sizeof(float));
    NEDO_CUDA_TRY(cudaMemcpyAsync(s->x_dev, s->x_pin, cols * sizeof(float), cudaMemcpyHostToDevice, s->stream));
    if (k == 0) {
        ArgmaxScratch a = s->scratch;
        a.out_index = s->amax_index;
        a.out_value = s->amax_value;
        if (int rc = dispatch_matvec(s, type, rows, cols, w_dev, s->x_dev, s->y_dev, 1, &a, s->stream, 0)) return rc;
        NEDO_CUDA_TRY(cudaMemcpyAsync(s->topk_ids_pin, s->amax_index, sizeof(int64_t) + sizeof(float),
                                      cudaMemcpyDeviceToHost, s->stream));
    } else {
        if (int rc = dispatch_matvec(s, type, rows, cols, w_dev, s->x_dev, s->y_dev, 1, nullptr, s->stream, 0))
            return rc;
        TopkScratch t{s->topk_cand, s->topk_counter, s->topk_ids, s->topk_vals};
        cudaError_t e = launch_topk(s->y_dev, rows, k, t, s->num_sms, s->stream);
        if (e != cudaSuccess) return cuda_fail(e, "topk launch");
        NEDO_CUDA_TRY(cudaMemcpyAsync(s->topk_ids_pin, s->topk_ids, k * sizeof(uint32_t), cudaMemcpyDeviceToHost,
                                      s->stream));
        NEDO_CUDA_TRY(cudaMemcpyAsync(s->topk_vals_pin, s->topk_vals, k * sizeof(float), cudaMemcpyDeviceToHost,
                                      s->stream));
    }
    if (int rc = read_status(s, s->stream)) return rc;
    if (k == 0) {
        int64_t idx;
        float val;
        std::memcpy(&idx, s->topk_ids_pin, sizeof(idx));
        std::memcpy(&val, reinterpret_cast<const uint8_t*>(s->topk_ids_pin) + sizeof(idx), sizeof(val));
        if (index_host) *index_host = idx;
        if (value_host) *value_host = val;
    } else {
        std::memcpy(ids_host, s->topk_ids_pin, k * sizeof(uint32_t));
        if (vals_host) std::memcpy(vals_host, s->topk_vals_pin, k * sizeof(float));
    }
    return 0;
}

int nedo_gpu_lm_head_topk(uint32_t type, uint64_t rows, uint64_t cols, const void* w_host, uint64_t w_bytes,
                          const float* x_host, uint32_t k, uint32_t* ids_host, float* vals_host) {
    if (k == 0) return fail(NEDO_GPU_ERR_ARG, "lm_head_topk: k must be in [1, min(rows, 256)]");
    if (!ids_host) return fail(NEDO_GPU_ERR_ARG, "lm_head_topk: null pointer");
    return lm_head_host(type, rows, cols, w_host, w_bytes, x_host, k, ids_host, vals_host, nullptr, nullptr);
}

int nedo_gpu_lm_head_argmax(uint32_t type, uint64_t rows, uint64_t cols, const void* w_host, uint64_t w_bytes,
                            const float* x_host, int64_t* index_host, float* value_host) {
    if (!index_host) return fail(NEDO_GPU_ERR_ARG, "lm_head_argmax: null pointer");
    return lm_head_host(type, rows, cols, w_host, w_bytes, x_host, 0, nullptr, nullptr, index_host, value_host);
}

int nedo_gpu_matvec_allgather_dev(uint32_t type, uint64_t rows, uint64_t cols, const void* w_dev, const float* x_dev,
                                  float* y_dev, const uint64_t* peer_y, const uint64_t* peer_signal, uint32_t npeers,
                                  uint64_t row_offset, void* stream) {
    uint64_t rb = 0;
    if (int rc = check_matvec_args(type, rows, cols, &rb)) return rc;
    if (rows == 0) return 0;
    if (!w_dev || !x_dev || !y_dev || (npeers && (!peer_y || !peer_signal)))
        return fail(NEDO_GPU_ERR_ARG, "matvec_allgather_dev: null pointer");
    if (npeers > kMaxPeers) return fail(NEDO_GPU_ERR_ARG, "matvec_allgather_dev: more than 7 peers");
    DeviceState* s = nullptr;
    if (int rc = get_state(&s)) return rc;
    ImmaPlan ip;
    if ((type == kQ8_0 || type == kQ4_0) && aligned16(w_dev) && aligned16(x_dev))
        ip = plan_imma(type, rows, cols, s->num_sms, s->max_smem);
    if (!ip.ok)
        return fail(NEDO_GPU_ERR_ARG,
                    "matvec_allgather_dev: the fused all-gather needs a Q8_0/Q4_0 shape of the int8 tensor-pipe kernel");
    PeerGather g;
    g.npeers = npeers;
    g.row_offset = row_offset;
    for (uint32_t k = 0; k < npeers; ++k) {
        g.peer_y[k] = reinterpret_cast<float*>(static_cast<uintptr_t>(peer_y[k]));
        g.peer_signal[k] = reinterpret_cast<uint32_t*>(static_cast<uintptr_t>(peer_signal[k]));
    }
    cudaError_t e = launch_imma(ip, w_dev, x_dev, y_dev, rows, cols, s->status, static_cast<cudaStream_t>(stream),
                                g_pdl.load() != 0, &g);
    if (e != cudaSuccess) return cuda_fail(e, "gemv_imma launch (all-gather)");
    return 0;
}

int nedo_gpu_allgather_wait_dev(uint32_t* signal_dev, uint32_t* expected_dev, uint32_t increment, void* stream) {
    if (!signal_dev || !expected_dev) return fail(NEDO_GPU_ERR_ARG, "allgather_wait_dev: null pointer");
    DeviceState* s = nullptr;
    if (int rc = get_state(&s)) return rc;
    cudaError_t e = launch_gather_wait(signal_dev, expected_dev, increment, s->status, static_cast<cudaStream_t>(stream),
                                       g_pdl.load() != 0);
    if (e != cudaSuccess) return cuda_fail(e, "all-gather wait launch");
    return 0;
}

int nedo_gpu_dequant_rows_dev(uint32_t type, uint64_t rows, uint64_t cols, const void* w_dev, uint64_t row_begin,
                              uint64_t row_count, float* out_dev, void* stream) {
    if (row_begin >= rows || row_count > rows - row_begin) return fail(NEDO_GPU_ERR_ROW, "bad embedding row");
    uint64_t rb = 0;
    if (int rc = tensor_row_bytes(type, cols, &rb)) return rc;
    if (!is_matvec_type(type)) return fail(NEDO_GPU_ERR_TYPE, "embedding type unsupported");
    if (!w_dev || !out_dev) return fail(NEDO_GPU_ERR_ARG, "dequant_rows_dev: null pointer");
    DeviceState* s = nullptr;
    if (int rc = get_state(&s)) return rc;
    cudaError_t e = launch_dequant_rows(type, w_dev, rows, cols, row_begin, row_count, out_dev,
                                        static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "dequant launch");
    return 0;
}

int nedo_gpu_status(void* stream) {
    DeviceState* s = nullptr;
    if (int rc = get_state(&s)) return rc;
    return read_status(s, static_cast<cudaStream_t>(stream));
}

int nedo_gpu_plan_info(uint32_t type, uint64_t rows, uint64_t cols, uint32_t batch, uint32_t* out, int n) {
    if (!out || n < 8) return fail(NEDO_GPU_ERR_ARG, "plan_info: need 8 output slots");
    uint64_t rb = 0;
    if (int rc = check_matvec_args(type, rows, cols, &rb)) return rc;
    DeviceState* s = nullptr;
    if (int rc = get_state(&s)) return rc;
    std::memset(out, 0, sizeof(uint32_t) * static_cast<size_t>(n));
    const bool tc = g_exact_batches.load() == 0 && batch >= tensor_core_min_batch(type) &&
                    cols >= kTensorCoreMinCols && gemm_tc_supported(type, rows, cols, batch) &&
                    !multi_takes_whole_batch(s, type, rows, cols, batch);
    if (batch <= 1 && (type == kQ8_0 || type == kQ4_0) && tc8_enabled()) {
        Tc8Plan tp = plan_tc8(type, rows, cols, s->num_sms, s->max_smem);
        if (tp.ok) {
            out[0] = 6;
            out[1] = tp.grid;
            out[2] = tp.threads;
            out[3] = tp.smem_bytes;
            out[4] = 16;
            out[5] = tp.slots;
            out[6] = tp.unit_bytes;
            out[7] = 8;  // loader + epilogue warps
            if (n > 8) out[8] = 1;
            return 0;
        }
    }
    if (!tc && (type == kQ8_0 || type == kQ4_0)) {  // int8 tensor-pipe launches
        const uint32_t tokens = batch >= 8 ? 8u : batch >= 4 ? 4u : batch >= 2 ? 2u : 1u;
        ImmaPlan ip = plan_imma(type, rows, cols, s->num_sms, s->max_smem, nullptr, tokens);
        // ring kernel: launches of 8, 4, 2 and 1 vectors
        uint32_t launches = batch <= 1 ? 1u : batch / 8u + static_cast<uint32_t>(__builtin_popcount(batch % 8u));
        if (batch >= 2 && multi_applies(s, type, rows, cols)) {
            // the first multi-vector launch, and the launch count, as dispatch_matvec plans them
            bool first = true;
            launches = 0;
            for_each_multi_launch(s, type, rows, cols, batch, [&](const ImmaPlan* mp, uint32_t, uint32_t) {
                ++launches;
                if (first && mp != nullptr) ip = *mp;
                first = false;
            });
        }
        if (ip.ok) {
            out[0] = 4;
            out[1] = ip.grid;
            out[2] = (ip.warps + 1) * 32;
            out[3] = ip.smem_bytes;
            out[4] = ip.tile_rows;
            out[5] = ip.slots;
            out[6] = ip.unit_bytes;
            out[7] = ip.warps;
            if (n > 8) out[8] = launches;
            return 0;
        }
    }
    if (batch <= 1) {
        StreamPlan p = plan_stream(type, rows, cols, s->num_sms, s->max_smem);
        if (p.ok) {
            out[0] = 1;
            out[1] = p.grid;
            out[2] = p.threads;
            out[3] = p.smem_bytes;
            out[4] = p.rows_per_tile;
            out[5] = p.slots;
            out[6] = p.slot_bytes;
            out[7] = p.warps;
            if (n > 8) out[8] = 1;
            return 0;
        }
    }
    if (tc) {
        out[0] = 5;  // tcgen05 GEMM: 256-row x 256-token tiles, K split over CTAs when tiles are few
        out[1] = gemm_tc_launch_ctas(type, rows, cols, batch, s->num_sms);
        out[2] = 320;
        out[4] = 128;
        out[5] = gemm_tc_splits(rows, cols, batch, s->num_sms);  // K splits (> 1: a fold kernel follows)
        if (n > 8) out[8] = out[5] > 1 ? 3u : 2u;  // x to fp16, the GEMM (, the fold)
        return 0;
    }
    out[0] = batch > 1 ? 3 : 2;
    if (n > 8) out[8] = batch > 1 && out[0] == 3 ? batch : 1u;
    return 0;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Device-resident decode forward pass (src/model.cpp:212-260).
//
// Layout in HBM: every weight uploaded once; q, k and v of a layer stored as
// one [q | k | v] matrix and gate and up as one [gate | up] matrix, so each pair
// or triple that shares its input is one matvec launch (rows concatenated, row
// bytes unchanged); the fp32 KV cache [layer][window][kv_heads * head_dim] for
// keys and for values; fp32 activations x, xn, qkv, att, tmp, gu and the logits.
// A pass is 3 + 5 * layers launches on one stream (3 + 8 * layers where the
// norms and the SiLU gate cannot be fused into the projections) (programmatic dependent
// launch between them), captured once as a CUDA graph that also uploads the
// token and position and downloads the greedy pick and the status word.
namespace {

struct DecLayer {
    uint32_t an_type = 0, fn_type = 0, qkv_type = 0, o_type = 0, gu_type = 0, down_type = 0;
    const void *an = nullptr, *fn = nullptr, *qkv = nullptr, *o = nullptr, *gu = nullptr, *down = nullptr;
    // the projection runs the resident-slice int8 kernel with the preceding
    // RMSNorm (qkv, gu) or SiLU gate (down) fused into its x-table build
    bool qkv_fused = false, gu_fused = false, down_fused = false;
};

// A projection with its input transform fused (XPrologue), on the resident-slice plan.
// The decode pass's resident-slice plans: work items of at most 2 tiles, so
// every int8 projection of the pass runs the same kernel instance.  A pass
// cycles through its kernels once per layer; with the 5-tile instance beside
// the 2-tile one their code no longer stayed in the SMs' instruction caches
// (measured: 0.90 ms per pass against 0.80 with one instance).
ImmaPlan decoder_slice_plan(const DeviceState* s, uint32_t type, uint64_t rows, uint64_t cols) {
    ImmaTuning tune;
    tune.max_tile_group = 2;
    return plan_imma(type, rows, cols, s->num_sms, s->max_smem, &tune);
}

int matvec_fused(DeviceState* s, uint32_t type, uint64_t rows, uint64_t cols, const void* w, const float* x, float* y,
                 const XPrologue* pro, cudaStream_t stream) {
    ImmaPlan ip = decoder_slice_plan(s, type, rows, cols);
    if (!ip.ok || !ip.slice) return fail(NEDO_GPU_ERR_ARG, "fused projection without a resident-slice plan");
    cudaError_t e = launch_imma(ip, w, x, y, rows, cols, s->status, stream, true, nullptr, 0, 0, pro);
    if (e != cudaSuccess) return cuda_fail(e, "gemv_imma (fused) launch");
    return 0;
}

bool fusable(const DeviceState* s, uint32_t type, uint64_t rows, uint64_t cols) {
    if (type != kQ8_0 && type != kQ4_0) return false;
    if (tc8_enabled()) return false;  // the opt-in tcgen05 kernel takes these shapes instead
    const ImmaPlan ip = decoder_slice_plan(s, type, rows, cols);
    return ip.ok && ip.slice;
}

struct DecPin {
    DecodeIo io;
    int64_t index;
    float value;
    uint32_t pad;
    DeviceStatus status;
};

}  // namespace

struct nedo_gpu_decoder {
    DeviceState* s = nullptr;
    nedo_gpu_decoder_config cfg{};
    uint32_t window = 0, qd = 0, kvd = 0;
    uint64_t emb_rows = 0, head_rows = 0;
    uint32_t emb_type = 0, onorm_type = 0, head_type = 0;
    const void *emb = nullptr, *onorm = nullptr, *head = nullptr;
    const float* route = nullptr;
    std::vector<DecLayer> layers;
    std::vector<void*> owned;
    float *x = nullptr, *x2 = nullptr, *xn = nullptr, *qkv = nullptr, *att = nullptr, *tmp = nullptr, *gu = nullptr;
    float *logits = nullptr, *kcache = nullptr, *vcache = nullptr;
    float* attn_part = nullptr;  // attention split partials [heads][splits][head_dim + 2]
    uint32_t* attn_counter = nullptr;  // [heads] finished splits (reset by the combining CTA)
    DecodeIo* io = nullptr;
    int64_t* amax = nullptr;  // index, then the value (float) in the next 8 bytes
    ArgmaxScratch scratch{};
    DecPin* pin = nullptr;
    float* logits_pin = nullptr;
    cudaStream_t stream = nullptr;      // the stream the passes run on
    cudaStream_t own_stream = nullptr;  // created with the decoder
    cudaGraphExec_t graph[2] = {nullptr, nullptr};  // without / with the logits download
    bool eager_done[2] = {false, false};
    cudaGraphExec_t gen_graph = nullptr;  // one pass + the on-device advance (generation)
    uint32_t* ids = nullptr;              // [context] picks of a generation
};

namespace {

int dec_alloc(nedo_gpu_decoder* d, void** p, uint64_t bytes) {
    cudaError_t e = cudaMalloc(p, bytes ? bytes : 16);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(decoder)");
    d->owned.push_back(*p);
    return 0;
}

// Upload one or more tensors back to back into one device buffer.
int dec_upload(nedo_gpu_decoder* d, const nedo_gpu_tensor_view* const* parts, int n, const void** out) {
    uint64_t total = 0;
    for (int i = 0; i < n; ++i) total += parts[i]->nbytes;
    void* dev = nullptr;
    if (int rc = dec_alloc(d, &dev, total)) return rc;
    uint64_t off = 0;
    for (int i = 0; i < n; ++i) {
        if (int rc = upload_weight(d->s, static_cast<uint8_t*>(dev) + off, parts[i]->data, parts[i]->nbytes)) return rc;
        off += parts[i]->nbytes;
    }
    *out = dev;
    return 0;
}

std::string tensor_label(uint64_t i) {
    static const char* kTop[4] = {"token_embd.weight", "output_norm.weight", "output.weight",
                                  "blk.0.ffn_gate_tid2eid.weight"};
    static const char* kLayer[9] = {"attn_norm", "attn_q", "attn_k", "attn_v", "attn_output",
                                    "ffn_norm", "ffn_gate", "ffn_up", "ffn_down"};
    if (i < 4) return kTop[i];
    return "blk." + std::to_string((i - 4) / 9) + "." + kLayer[(i - 4) % 9] + ".weight";
}

// A rank-2 projection [cols, rows] of a matvec type, its bytes the rows' bytes.
int check_matrix(const nedo_gpu_tensor_view& t, uint64_t i, uint64_t cols, uint64_t rows) {
    const std::string name = tensor_label(i);
    if (t.data == nullptr) return fail(NEDO_GPU_ERR_ARG, "missing tensor: " + name);
    if (t.ndims != 2) return fail(NEDO_GPU_ERR_ARG, "matvec requires rank-2 tensor: " + name);
    if (!is_matvec_type(t.type)) return fail(NEDO_GPU_ERR_TYPE, "matvec tensor type not supported: " + name);
    uint64_t rb = 0;
    if (int rc = tensor_row_bytes(t.type, t.shape[0], &rb)) return rc;
    if (t.shape[0] != cols || t.shape[1] != rows || t.nbytes != rb * rows)
        return fail(NEDO_GPU_ERR_ARG, "tensor shape does not match the configuration: " + name);
    return 0;
}

int check_norm(const nedo_gpu_tensor_view& t, uint64_t i, uint64_t n) {
    const std::string name = tensor_label(i);
    if (t.data == nullptr) return fail(NEDO_GPU_ERR_ARG, "missing tensor: " + name);
    if (t.ndims != 1 || t.shape[0] != n) return fail(NEDO_GPU_ERR_ARG, "bad RMSNorm tensor: " + name);
    if (t.type != 0 && t.type != kF16) return fail(NEDO_GPU_ERR_TYPE, "unsupported RMSNorm tensor type: " + name);
    if (t.nbytes != n * (t.type == 0 ? 4u : 2u)) return fail(NEDO_GPU_ERR_ARG, "bad RMSNorm tensor: " + name);
    return 0;
}

// The pass, enqueued on d->stream (captured or eager).
int dec_enqueue(nedo_gpu_decoder* d) {
    DeviceState* s = d->s;
    const nedo_gpu_decoder_config& c = d->cfg;
    cudaStream_t st = d->stream;
    const bool pdl = true;
    const uint32_t hd = c.head_dim;
    const float inv_sqrt_hd = 1.0f / std::sqrt(static_cast<float>(hd));
    cudaError_t e = launch_embed(d->emb_type, d->emb, c.dim, d->emb_rows, d->io, d->x, s->status, st, pdl);
    if (e != cudaSuccess) return cuda_fail(e, "embedding launch");
    const size_t cache_layer = static_cast<size_t>(d->window) * d->kvd;
    // the residual stream lives in xcur; a fused norm writes x + delta to the
    // other buffer (CTA 0 of the projection), so the two alternate
    float* xcur = d->x;
    float* xalt = d->x2;
    const float* pending = nullptr;  // a residual not yet added to xcur
    auto norm_into = [&](bool fused, const void* nw, uint32_t nwt, uint32_t type, uint64_t rows, const void* w,
                         float* y, const float* kc, const float* vc) -> int {
        if (fused) {
            XPrologue pro;
            pro.mode = kPrologueNorm;
            pro.delta = pending;
            pro.w = nw;
            pro.wtype = nwt == 0 ? 0u : 1u;
            pro.eps = c.rms_eps;
            pro.x_out = xalt;
            if (kc != nullptr) {
                // the q|k|v projection also brings this layer's cached keys and values into L2
                pro.kcache = kc;
                pro.vcache = vc;
                pro.io = d->io;
                pro.window = d->window;
                pro.row_bytes = d->kvd * static_cast<uint32_t>(sizeof(float));
            }
            if (int rc = matvec_fused(s, type, rows, c.dim, w, xcur, y, &pro, st)) return rc;
            std::swap(xcur, xalt);
        } else {
            cudaError_t ee = launch_add_rmsnorm(xcur, pending, nw, nwt == 0 ? 0u : 1u, d->xn, c.dim, c.rms_eps, st, pdl);
            if (ee != cudaSuccess) return cuda_fail(ee, "rmsnorm launch");
            if (int rc = dispatch_matvec(s, type, rows, c.dim, w, d->xn, y, 1, nullptr, st, 1)) return rc;
        }
        pending = nullptr;
        return 0;
    };
    for (uint32_t li = 0; li < c.layers; ++li) {
        const DecLayer& L = d->layers[li];
        float* kc = d->kcache + li * cache_layer;
        float* vc = d->vcache + li * cache_layer;
        if (int rc = norm_into(L.qkv_fused, L.an, L.an_type, L.qkv_type, d->qd + 2u * d->kvd, L.qkv, d->qkv, kc, vc))
            return rc;
        e = launch_attention(d->qkv, kc, vc, d->att, d->attn_part, d->attn_counter, d->io, c.heads, c.kv_heads, hd,
                             d->window, c.rope_theta, inv_sqrt_hd, st, pdl);
        if (e != cudaSuccess) return cuda_fail(e, "attention launch");
        // the output projection on the pass's slice instance where it has one
        if (fusable(s, L.o_type, c.dim, d->qd)) {
            if (int rc = matvec_fused(s, L.o_type, c.dim, d->qd, L.o, d->att, d->tmp, nullptr, st)) return rc;
        } else if (int rc = dispatch_matvec(s, L.o_type, c.dim, d->qd, L.o, d->att, d->tmp, 1, nullptr, st, 1)) {
            return rc;
        }
        pending = d->tmp;
        if (int rc = norm_into(L.gu_fused, L.fn, L.fn_type, L.gu_type, 2u * c.ffn, L.gu, d->gu, nullptr, nullptr))
            return rc;
        // MorphFFN occupies the trailing morph_layers blocks (src/model.cpp:200)
        const bool morph = d->route != nullptr && li + c.morph_layers >= c.layers;
        if (L.down_fused) {
            XPrologue pro;
            pro.mode = kPrologueSilu;
            pro.up = d->gu + c.ffn;
            pro.route = morph ? d->route : nullptr;
            pro.io = d->io;
            pro.m_shared = c.morph_shared;
            pro.m_root = c.morph_root;
            pro.m_suffix = c.morph_suffix;
            if (int rc = matvec_fused(s, L.down_type, c.dim, c.ffn, L.down, d->gu, d->tmp, &pro, st)) return rc;
        } else {
            e = launch_silu_mul(d->gu, c.ffn, morph ? d->route : nullptr, d->io, c.morph_shared, c.morph_root,
                                c.morph_suffix, st, pdl);
            if (e != cudaSuccess) return cuda_fail(e, "silu launch");
            if (int rc = dispatch_matvec(s, L.down_type, c.dim, c.ffn, L.down, d->gu, d->tmp, 1, nullptr, st, 1))
                return rc;
        }
        pending = d->tmp;
    }
    e = launch_add_rmsnorm(xcur, pending, d->onorm, d->onorm_type == 0 ? 0u : 1u, d->xn, c.dim, c.rms_eps, st, pdl);
    if (e != cudaSuccess) return cuda_fail(e, "rmsnorm launch");
    ArgmaxScratch a = d->scratch;
    a.out_index = d->amax;
    a.out_value = reinterpret_cast<float*>(d->amax + 1);
    return dispatch_matvec(s, d->head_type, d->head_rows, c.dim, d->head, d->xn, d->logits, 1, &a, st, 1);
}

// io upload, the pass, the result and status downloads (and the logits).
int dec_step_ops(nedo_gpu_decoder* d, bool with_logits) {
    NEDO_CUDA_TRY(cudaMemcpyAsync(d->io, &d->pin->io, sizeof(DecodeIo), cudaMemcpyHostToDevice, d->stream));
    if (int rc = dec_enqueue(d)) return rc;
    NEDO_CUDA_TRY(cudaMemcpyAsync(&d->pin->index, d->amax, sizeof(int64_t) + sizeof(float), cudaMemcpyDeviceToHost,
                                  d->stream));
    NEDO_CUDA_TRY(cudaMemcpyAsync(&d->pin->status, d->s->status, sizeof(DeviceStatus), cudaMemcpyDeviceToHost,
                                  d->stream));
    if (with_logits)
        NEDO_CUDA_TRY(cudaMemcpyAsync(d->logits_pin, d->logits, d->head_rows * sizeof(float), cudaMemcpyDeviceToHost,
                                      d->stream));
    return 0;
}

void dec_free(nedo_gpu_decoder* d) {
    for (auto& g : d->graph)
        if (g) cudaGraphExecDestroy(g);
    if (d->gen_graph) cudaGraphExecDestroy(d->gen_graph);
    if (d->stream) cudaStreamSynchronize(d->stream);
    for (void* p : d->owned) cudaFree(p);
    if (d->pin) cudaFreeHost(d->pin);
    if (d->logits_pin) cudaFreeHost(d->logits_pin);
    if (d->own_stream) cudaStreamDestroy(d->own_stream);
    delete d;
}

// Runs `fn` with the decoder's device current, restoring the caller's.
template <typename F>
int on_device(int dev, F fn) {
    int prev = 0;
    NEDO_CUDA_TRY(cudaGetDevice(&prev));
    if (prev != dev) NEDO_CUDA_TRY(cudaSetDevice(dev));
    const int rc = fn();
    if (prev != dev) cudaSetDevice(prev);
    return rc;
}

}  // namespace

extern "C" {

int nedo_gpu_decoder_create(const nedo_gpu_decoder_config* cfg, const nedo_gpu_tensor_view* t, uint64_t n,
                            nedo_gpu_decoder** out) {
    if (!cfg || !t || !out) return fail(NEDO_GPU_ERR_ARG, "decoder_create: null pointer");
    *out = nullptr;
    const nedo_gpu_decoder_config c = *cfg;
    // src/model.cpp:158-160
    if (!c.heads || !c.kv_heads || c.heads % c.kv_heads || c.dim != c.heads * c.head_dim)
        return fail(NEDO_GPU_ERR_ARG, "invalid GQA dimensions");
    if (!c.context) return fail(NEDO_GPU_ERR_ARG, "context_length is zero");
    if (c.head_dim == 0 || c.head_dim > 1024u) return fail(NEDO_GPU_ERR_ARG, "head_dim must be in 1..1024");
    if (c.dim == 0 || c.ffn == 0 || c.vocab == 0) return fail(NEDO_GPU_ERR_ARG, "empty model dimensions");
    if (c.dim > 25600) return fail(NEDO_GPU_ERR_ARG, "embedding_length above 25600 (RMSNorm stages it in shared memory)");
    if (n != 4u + 9ull * c.layers) return fail(NEDO_GPU_ERR_ARG, "decoder_create: expected 4 + 9 * layers tensors");
    const uint32_t qd = c.heads * c.head_dim, kvd = c.kv_heads * c.head_dim;
    // embedding and head
    if (t[0].data == nullptr || t[0].ndims != 2 || t[0].shape[0] != c.dim || t[0].shape[1] < c.vocab)
        return fail(NEDO_GPU_ERR_ARG, "bad embedding tensor: token_embd.weight");
    if (!is_matvec_type(t[0].type)) return fail(NEDO_GPU_ERR_TYPE, "embedding type unsupported");
    if (int rc = check_matrix(t[0], 0, c.dim, t[0].shape[1])) return rc;
    if (int rc = check_norm(t[1], 1, c.dim)) return rc;
    const nedo_gpu_tensor_view& head = t[2].data ? t[2] : t[0];
    if (int rc = check_matrix(head, t[2].data ? 2 : 0, c.dim, head.shape[1])) return rc;
    if (head.shape[1] < c.vocab) return fail(NEDO_GPU_ERR_ARG, "LM head has fewer rows than vocab_size");
    if (t[3].data) {
        if (t[3].type != 0 || t[3].ndims != 2 || t[3].shape[0] != 2 || t[3].shape[1] != c.vocab ||
            t[3].nbytes != 8ull * c.vocab)
            return fail(NEDO_GPU_ERR_ARG, "MorphFFN token-id routing table shape/type [2,vocab] F32");
        if (c.morph_shared + c.morph_root + c.morph_suffix != c.ffn)
            return fail(NEDO_GPU_ERR_ARG, "MorphFFN widths do not sum to feed_forward_length");
        if (c.morph_layers > c.layers) return fail(NEDO_GPU_ERR_ARG, "MorphFFN layer count exceeds block count");
    }
    for (uint32_t li = 0; li < c.layers; ++li) {
        const uint64_t b = 4ull + 9ull * li;
        if (int rc = check_norm(t[b + 0], b + 0, c.dim)) return rc;
        if (int rc = check_matrix(t[b + 1], b + 1, c.dim, qd)) return rc;
        if (int rc = check_matrix(t[b + 2], b + 2, c.dim, kvd)) return rc;
        if (int rc = check_matrix(t[b + 3], b + 3, c.dim, kvd)) return rc;
        if (int rc = check_matrix(t[b + 4], b + 4, qd, c.dim)) return rc;
        if (int rc = check_norm(t[b + 5], b + 5, c.dim)) return rc;
        if (int rc = check_matrix(t[b + 6], b + 6, c.dim, c.ffn)) return rc;
        if (int rc = check_matrix(t[b + 7], b + 7, c.dim, c.ffn)) return rc;
        if (int rc = check_matrix(t[b + 8], b + 8, c.ffn, c.dim)) return rc;
        if (t[b + 1].type != t[b + 2].type || t[b + 1].type != t[b + 3].type)
            return fail(NEDO_GPU_ERR_TYPE, "q, k and v projections of a layer must share one type");
        if (t[b + 6].type != t[b + 7].type)
            return fail(NEDO_GPU_ERR_TYPE, "gate and up projections of a layer must share one type");
    }
    const uint32_t sl = c.sliding ? c.sliding : c.context;
    const uint32_t window = std::max<uint32_t>(1u, std::min<uint32_t>(sl, c.context));
    if (c.head_dim % 8u) return fail(NEDO_GPU_ERR_ARG, "head_dim must be a multiple of 8");

    DeviceState* s = nullptr;
    if (int rc = get_state(&s)) return rc;
    auto* d = new nedo_gpu_decoder();
    d->s = s;
    d->cfg = c;
    d->window = window;
    d->qd = qd;
    d->kvd = kvd;
    auto build = [&]() -> int {
        NEDO_CUDA_TRY(cudaStreamCreateWithFlags(&d->own_stream, cudaStreamNonBlocking));
        d->stream = d->own_stream;
        const nedo_gpu_tensor_view* p1[1];
        p1[0] = &t[0];
        if (int rc = dec_upload(d, p1, 1, &d->emb)) return rc;
        d->emb_type = t[0].type;
        d->emb_rows = t[0].shape[1];
        p1[0] = &t[1];
        if (int rc = dec_upload(d, p1, 1, &d->onorm)) return rc;
        d->onorm_type = t[1].type;
        if (t[2].data) {
            p1[0] = &t[2];
            if (int rc = dec_upload(d, p1, 1, &d->head)) return rc;
        } else {
            d->head = d->emb;  // tied (src/model.cpp:94)
        }
        d->head_type = head.type;
        d->head_rows = head.shape[1];
        if (t[3].data) {
            const void* r = nullptr;
            p1[0] = &t[3];
            if (int rc = dec_upload(d, p1, 1, &r)) return rc;
            d->route = static_cast<const float*>(r);
        }
        d->layers.resize(c.layers);
        for (uint32_t li = 0; li < c.layers; ++li) {
            const uint64_t b = 4ull + 9ull * li;
            DecLayer& L = d->layers[li];
            p1[0] = &t[b + 0];
            if (int rc = dec_upload(d, p1, 1, &L.an)) return rc;
            L.an_type = t[b + 0].type;
            const nedo_gpu_tensor_view* qkv[3] = {&t[b + 1], &t[b + 2], &t[b + 3]};
            if (int rc = dec_upload(d, qkv, 3, &L.qkv)) return rc;
            L.qkv_type = t[b + 1].type;
            p1[0] = &t[b + 4];
            if (int rc = dec_upload(d, p1, 1, &L.o)) return rc;
            L.o_type = t[b + 4].type;
            p1[0] = &t[b + 5];
            if (int rc = dec_upload(d, p1, 1, &L.fn)) return rc;
            L.fn_type = t[b + 5].type;
            const nedo_gpu_tensor_view* gu[2] = {&t[b + 6], &t[b + 7]};
            if (int rc = dec_upload(d, gu, 2, &L.gu)) return rc;
            L.gu_type = t[b + 6].type;
            p1[0] = &t[b + 8];
            if (int rc = dec_upload(d, p1, 1, &L.down)) return rc;
            L.down_type = t[b + 8].type;
            L.qkv_fused = fusable(s, L.qkv_type, qd + 2ull * kvd, c.dim);
            L.gu_fused = fusable(s, L.gu_type, 2ull * c.ffn, c.dim);
            L.down_fused = fusable(s, L.down_type, c.dim, c.ffn);
        }
        void* p = nullptr;
        auto vec = [&](float** f, uint64_t count) -> int {
            if (int rc = dec_alloc(d, &p, count * sizeof(float))) return rc;
            *f = static_cast<float*>(p);
            return 0;
        };
        if (int rc = vec(&d->x, c.dim)) return rc;
        if (int rc = vec(&d->x2, c.dim)) return rc;
        if (int rc = vec(&d->xn, c.dim)) return rc;
        if (int rc = vec(&d->qkv, qd + 2ull * kvd)) return rc;
        if (int rc = vec(&d->att, qd)) return rc;
        if (int rc = vec(&d->tmp, c.dim)) return rc;
        if (int rc = vec(&d->gu, 2ull * c.ffn)) return rc;
        if (int rc = vec(&d->logits, d->head_rows)) return rc;
        if (int rc = vec(&d->attn_part, static_cast<uint64_t>(c.heads) * attention_splits(window) * (c.head_dim + 2u)))
            return rc;
        if (int rc = dec_alloc(d, &p, c.heads * sizeof(uint32_t))) return rc;
        d->attn_counter = static_cast<uint32_t*>(p);
        NEDO_CUDA_TRY(cudaMemsetAsync(d->attn_counter, 0, c.heads * sizeof(uint32_t), d->stream));
        const uint64_t cache = static_cast<uint64_t>(c.layers) * window * kvd;
        if (int rc = vec(&d->kcache, cache ? cache : 1)) return rc;
        if (int rc = vec(&d->vcache, cache ? cache : 1)) return rc;
        NEDO_CUDA_TRY(cudaMemsetAsync(d->kcache, 0, (cache ? cache : 1) * sizeof(float), d->stream));
        NEDO_CUDA_TRY(cudaMemsetAsync(d->vcache, 0, (cache ? cache : 1) * sizeof(float), d->stream));
        if (int rc = dec_alloc(d, &p, sizeof(DecodeIo))) return rc;
        d->io = static_cast<DecodeIo*>(p);
        if (int rc = dec_alloc(d, &p, static_cast<uint64_t>(c.context) * sizeof(uint32_t))) return rc;
        d->ids = static_cast<uint32_t*>(p);
        if (int rc = dec_alloc(d, &p, 16)) return rc;
        d->amax = static_cast<int64_t*>(p);
        const size_t ncand = static_cast<size_t>(s->num_sms) + 1;
        if (int rc = dec_alloc(d, &p, ncand * sizeof(float))) return rc;
        d->scratch.cand_val = static_cast<float*>(p);
        if (int rc = dec_alloc(d, &p, ncand * sizeof(uint32_t))) return rc;
        d->scratch.cand_idx = static_cast<uint32_t*>(p);
        if (int rc = dec_alloc(d, &p, sizeof(uint32_t))) return rc;
        d->scratch.counter = static_cast<uint32_t*>(p);
        NEDO_CUDA_TRY(cudaMemsetAsync(d->scratch.counter, 0, sizeof(uint32_t), d->stream));
        NEDO_CUDA_TRY(cudaHostAlloc(reinterpret_cast<void**>(&d->pin), sizeof(DecPin), cudaHostAllocDefault));
        NEDO_CUDA_TRY(cudaHostAlloc(reinterpret_cast<void**>(&d->logits_pin), d->head_rows * sizeof(float),
                                    cudaHostAllocDefault));
        NEDO_CUDA_TRY(cudaStreamSynchronize(d->stream));
        return 0;
    };
    if (int rc = build()) {
        dec_free(d);
        return rc;
    }
    *out = d;
    return 0;
}

int nedo_gpu_decoder_forward(nedo_gpu_decoder* d, uint32_t token, uint64_t pos, float* logits_host,
                             uint32_t* argmax_out) {
    if (!d) return fail(NEDO_GPU_ERR_ARG, "decoder_forward: null decoder");
    if (token >= d->cfg.vocab || token >= d->emb_rows) return fail(NEDO_GPU_ERR_ARG, "prompt token id out of range");
    if (pos >= d->cfg.context) return fail(NEDO_GPU_ERR_ARG, "position beyond context_length");
    return on_device(d->s->device, [&]() -> int {
        d->pin->io.pos = pos;
        d->pin->io.token = token;
        const int k = logits_host ? 1 : 0;
        if (d->graph[k] == nullptr && d->eager_done[k]) {
            // second call of this kind: capture the pass once (it re-reads io from device memory)
            cudaGraph_t g = nullptr;
            NEDO_CUDA_TRY(cudaStreamBeginCapture(d->stream, cudaStreamCaptureModeThreadLocal));
            const int rc = dec_step_ops(d, k == 1);
            cudaError_t e = cudaStreamEndCapture(d->stream, &g);
            if (rc) {
                if (g) cudaGraphDestroy(g);
                return rc;
            }
            if (e != cudaSuccess) return cuda_fail(e, "cudaStreamEndCapture(decoder)");
            e = cudaGraphInstantiate(&d->graph[k], g, 0);
            cudaGraphDestroy(g);
            if (e != cudaSuccess) return cuda_fail(e, "cudaGraphInstantiate(decoder)");
        }
        if (d->graph[k]) {
            NEDO_CUDA_TRY(cudaGraphLaunch(d->graph[k], d->stream));
        } else {
            // first call of this kind runs eagerly (kernel attributes and plans settle)
            if (int rc = dec_step_ops(d, k == 1)) return rc;
            d->eager_done[k] = true;
        }
        NEDO_CUDA_TRY(cudaStreamSynchronize(d->stream));
        if (d->pin->status.flags != 0) {
            const DeviceStatus st = d->pin->status;
            clear_status_flags(d->s, d->stream);
            char buf[160];
            std::snprintf(buf, sizeof(buf), "device kernel failed in the decode pass (flags=0x%x, site=%u)", st.flags,
                          st.where);
            return fail(NEDO_GPU_ERR_DEVICE, buf);
        }
        if (argmax_out) *argmax_out = static_cast<uint32_t>(d->pin->index);
        if (logits_host) std::memcpy(logits_host, d->logits_pin, d->head_rows * sizeof(float));
        return 0;
    });
}

int nedo_gpu_decoder_set_stream(nedo_gpu_decoder* d, void* stream) {
    if (!d) return fail(NEDO_GPU_ERR_ARG, "decoder_set_stream: null decoder");
    return on_device(d->s->device, [&]() -> int {
        NEDO_CUDA_TRY(cudaStreamSynchronize(d->stream));
        for (auto& g : d->graph) {
            if (g) cudaGraphExecDestroy(g);
            g = nullptr;
        }
        if (d->gen_graph) cudaGraphExecDestroy(d->gen_graph);
        d->gen_graph = nullptr;
        d->eager_done[0] = d->eager_done[1] = false;
        d->stream = stream ? static_cast<cudaStream_t>(stream) : d->own_stream;
        return 0;
    });
}

int nedo_gpu_decoder_generate(nedo_gpu_decoder* d, uint32_t token, uint64_t pos, uint32_t n, uint32_t* ids_host) {
    if (!d || (n && !ids_host)) return fail(NEDO_GPU_ERR_ARG, "decoder_generate: null pointer");
    if (token >= d->cfg.vocab || token >= d->emb_rows) return fail(NEDO_GPU_ERR_ARG, "prompt token id out of range");
    if (n == 0) return 0;
    if (pos + n > d->cfg.context) return fail(NEDO_GPU_ERR_ARG, "generation beyond context_length");
    // every pick must be a valid next token: the head may have more rows than vocab
    if (d->head_rows > d->emb_rows) return fail(NEDO_GPU_ERR_ARG, "LM head has more rows than the embedding");
    return on_device(d->s->device, [&]() -> int {
        if (!d->eager_done[0]) {
            // settle kernel attributes and plans with one eager pass first
            d->pin->io.pos = pos;
            d->pin->io.token = token;
            d->pin->io.step = 0;
            if (int rc = dec_step_ops(d, false)) return rc;
            NEDO_CUDA_TRY(cudaStreamSynchronize(d->stream));
            d->eager_done[0] = true;
        }
        if (d->gen_graph == nullptr) {
            cudaGraph_t g = nullptr;
            NEDO_CUDA_TRY(cudaStreamBeginCapture(d->stream, cudaStreamCaptureModeThreadLocal));
            int rc = dec_enqueue(d);
            if (rc == 0) {
                cudaError_t e = launch_advance(d->io, d->amax, d->ids, d->cfg.context, d->stream);
                if (e != cudaSuccess) rc = cuda_fail(e, "advance launch");
            }
            cudaError_t e = cudaStreamEndCapture(d->stream, &g);
            if (rc) {
                if (g) cudaGraphDestroy(g);
                return rc;
            }
            if (e != cudaSuccess) return cuda_fail(e, "cudaStreamEndCapture(decoder generate)");
            e = cudaGraphInstantiate(&d->gen_graph, g, 0);
            cudaGraphDestroy(g);
            if (e != cudaSuccess) return cuda_fail(e, "cudaGraphInstantiate(decoder generate)");
        }
        d->pin->io.pos = pos;
        d->pin->io.token = token;
        d->pin->io.step = 0;
        NEDO_CUDA_TRY(cudaMemcpyAsync(d->io, &d->pin->io, sizeof(DecodeIo), cudaMemcpyHostToDevice, d->stream));
        for (uint32_t k = 0; k < n; ++k) NEDO_CUDA_TRY(cudaGraphLaunch(d->gen_graph, d->stream));
        NEDO_CUDA_TRY(cudaMemcpyAsync(ids_host, d->ids, n * sizeof(uint32_t), cudaMemcpyDeviceToHost, d->stream));
        NEDO_CUDA_TRY(cudaMemcpyAsync(&d->pin->status, d->s->status, sizeof(DeviceStatus), cudaMemcpyDeviceToHost,
                                      d->stream));
        NEDO_CUDA_TRY(cudaStreamSynchronize(d->stream));
        if (d->pin->status.flags != 0) {
            const DeviceStatus st = d->pin->status;
            clear_status_flags(d->s, d->stream);
            char buf[160];
            std::snprintf(buf, sizeof(buf), "device kernel failed in the decode pass (flags=0x%x, site=%u)", st.flags,
                          st.where);
            return fail(NEDO_GPU_ERR_DEVICE, buf);
        }
        return 0;
    });
}

int nedo_gpu_decoder_logits_dev(nedo_gpu_decoder* d, const float** logits_dev) {
    if (!d || !logits_dev) return fail(NEDO_GPU_ERR_ARG, "decoder_logits_dev: null pointer");
    *logits_dev = d->logits;
    return 0;
}

int nedo_gpu_decoder_reset(nedo_gpu_decoder* d) {
    if (!d) return fail(NEDO_GPU_ERR_ARG, "decoder_reset: null decoder");
    return on_device(d->s->device, [&]() -> int {
        const size_t bytes = static_cast<size_t>(d->cfg.layers) * d->window * d->kvd * sizeof(float);
        if (bytes) {
            NEDO_CUDA_TRY(cudaMemsetAsync(d->kcache, 0, bytes, d->stream));
            NEDO_CUDA_TRY(cudaMemsetAsync(d->vcache, 0, bytes, d->stream));
        }
        NEDO_CUDA_TRY(cudaStreamSynchronize(d->stream));
        return 0;
    });
}

void nedo_gpu_decoder_destroy(nedo_gpu_decoder* d) {
    if (!d) return;
    on_device(d->s->device, [&]() -> int {
        dec_free(d);
        return 0;
    });
}

}  // extern "C"
