// common.cuh -- small sm_100a building blocks shared by the matvec kernels:
// mbarrier + bulk-copy (TMA, no multicast) wrappers, bounded waits, fp16 decode,
// packed fp32x2 arithmetic and warp reductions.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace nedo_gpu {

// GGUF tensor type codes (reference include/nedo/gguf.hpp:18-19).
enum : uint32_t { kF16 = 1, kQ4_0 = 2, kQ8_0 = 8 };

// Device-side error bits, OR-ed into DeviceStatus::flags by a kernel that had to
// give up (never by trapping).
enum : uint32_t {
    kErrWaitTimeout = 1u,   // an mbarrier wait exceeded its time bound
    kErrBadLaunch = 2u,     // a kernel saw launch parameters it cannot honour
    kErrArgument = 4u,      // a kernel read an out-of-range value from device memory (a token id)
};

struct DeviceStatus {
    uint32_t flags;
    uint32_t where;          // site id of the first failure (diagnostics only)
    uint64_t wait_limit_ns;  // bound of every spin-wait (set by the host; 0 = kWaitLimitNs)
};

// Default upper bound of every spin-wait in these kernels.  Any wait that a
// correct launch performs ends in microseconds; two seconds means something is
// wrong.  The host may lower it per device (DeviceStatus::wait_limit_ns).
constexpr uint64_t kWaitLimitNs = 2000000000ull;

// The bound a kernel applies: read only once a wait has already failed its
// first try, so the load costs nothing on the fast path.
__device__ __forceinline__ uint64_t wait_limit_ns(const DeviceStatus* st) {
    if (st == nullptr) return kWaitLimitNs;
    const uint64_t v = *reinterpret_cast<const volatile uint64_t*>(&st->wait_limit_ns);
    return v != 0 ? v : kWaitLimitNs;
}

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

// Make mbarrier initialisation visible to the async (TMA) proxy.
__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// try_wait with a suspend-time hint: a waiting thread sleeps (up to ~0.5 us)
// instead of spinning on issue slots the computing warps need.
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity), "r"(500u)
        : "memory");
    return ok != 0;
}

// Bounded wait on an mbarrier phase.  Returns false (and records the failure)
// when the time limit passes; the caller must then wind down without touching
// the guarded buffer.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, DeviceStatus* st, uint32_t site) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    const uint64_t limit = wait_limit_ns(st);
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if (global_timer_ns() - t0 > limit) {
            if (st != nullptr) {
                if (atomicOr(&st->flags, kErrWaitTimeout) == 0u) st->where = site;
            }
            return false;
        }
    }
}

// One-dimensional bulk copy global -> this CTA's shared memory, completing on
// `bar` with a transaction count of `bytes`.  Both addresses 16-byte aligned,
// `bytes` a multiple of 16.  No cluster multicast.
__device__ __forceinline__ void bulk_copy_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                              uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
        : "memory");
}

// L2 policy for data many CTAs read (the activation vector).
__device__ __forceinline__ uint64_t l2_policy_evict_last() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// L2 policy for data a few CTAs read once each (a weight tile several token groups share).
__device__ __forceinline__ uint64_t l2_policy_evict_normal() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// L2 policy for data read exactly once (the weight stream).
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

__device__ __forceinline__ void named_barrier_sync(uint32_t id, uint32_t nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

__device__ __forceinline__ float half_bits_to_float(uint32_t bits16) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(bits16 & 0xFFFFu)));
}

__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }
__device__ __forceinline__ float2 fadd2(float2 a, float2 b) { return __fadd2_rn(a, b); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    return v;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

// (a & mask) | bits as a single LOP3 with all three operands in registers
// (two 32-bit immediates do not fit one instruction).
__device__ __forceinline__ uint32_t lop_and_or(uint32_t a, uint32_t mask, uint32_t bits) {
    uint32_t d;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(mask), "r"(bits));
    return d;
}

// (a & mask) ^ bits as a single LOP3.
__device__ __forceinline__ uint32_t lop_and_xor(uint32_t a, uint32_t mask, uint32_t bits) {
    uint32_t d;
    asm("lop3.b32 %0, %1, %2, %3, 0x6A;" : "=r"(d) : "r"(a), "r"(mask), "r"(bits));
    return d;
}

}  // namespace nedo_gpu
