// allgather.cu -- completion wait of the fused all-gather.
//
// A row-sharded matvec (rows are independent: reference src/kernels.cpp:166-168)
// running with a PeerGather stores its rows straight into every peer's gathered
// y over NVLink and, per CTA, adds 1 to each peer's signal word after a
// system-scope fence.  This one-thread kernel runs next on the receiving
// rank's stream: it waits until its signal word has advanced by `increment`
// (peers x CTAs per launch) past the expected value kept in device memory,
// then advances that value, so the same launch works unchanged in a CUDA graph
// replayed many times.  The wait is bounded (2 s by default, the device's
// DeviceStatus::wait_limit_ns when set); on timeout it records the failure in
// DeviceStatus and still advances the expected value by `increment`.  Every
// step thus consumes exactly `increment` arrivals: signals of a step that
// arrive after its wait gave up count toward that step, never toward the
// next one, so a late peer cannot make the next step read stale rows.  The
// gathered buffer of a step that reported NEDO_GPU_ERR_DEVICE is invalid.
//
// With programmatic dependent launch the wait kernel starts while this rank's
// matvec is still running (its CTA fits beside the matvec's), so the peers'
// signals are watched as they arrive; griddepcontrol.wait then covers this
// rank's own rows before the kernel ends, and the next kernel on the stream
// may begin its prologue as soon as the wait kernel starts.
#include "common.cuh"
#include "launch.h"

namespace nedo_gpu {
namespace {

__global__ void gather_wait_kernel(uint32_t* signal, uint32_t* expected, uint32_t increment, DeviceStatus* status) {
    asm volatile("griddepcontrol.launch_dependents;");
    if (threadIdx.x != 0) {
        asm volatile("griddepcontrol.wait;" ::: "memory");
        return;
    }
    const uint32_t target = *expected + increment;  // wraps with the counter
    volatile uint32_t* sig = signal;
    const uint64_t t0 = global_timer_ns();
    const uint64_t limit = wait_limit_ns(status);
    // counters wrap: "reached" is a non-negative signed distance
    while (static_cast<int32_t>(*sig - target) < 0) {
        if (global_timer_ns() - t0 > limit) {
            if (atomicOr(&status->flags, kErrWaitTimeout) == 0u) status->where = 40u;
            asm volatile("griddepcontrol.wait;" ::: "memory");
            *expected = target;  // this step's arrivals stay this step's, late or not
            return;
        }
        __nanosleep(200);
    }
    asm volatile("griddepcontrol.wait;" ::: "memory");  // this rank's own rows are complete
    // acquire: the peers' stores that preceded their signal are visible to
    // every later kernel on this stream
    __threadfence_system();
    *expected = target;
}

}  // namespace

cudaError_t launch_gather_wait(uint32_t* signal, uint32_t* expected, uint32_t increment, DeviceStatus* status,
                               cudaStream_t stream, bool pdl) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(32);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, gather_wait_kernel, signal, expected, increment, status);
}

}  // namespace nedo_gpu
