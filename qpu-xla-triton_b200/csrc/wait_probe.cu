// qpucuda_context_probe_wait_expiry (include/qpucuda_runtime.h): makes one bounded mbarrier wait
// run out on the device and reports it the way every operator reports an expired kernel wait.
//
// The kernel is one warp. Lane 0 initialises an mbarrier that expects one arrival and waits on
// its first phase with sm100::wait_bounded_ns, the wait all tcgen05 / bulk-copy kernels of this
// library use; nothing ever arrives, so after limit_ns of %globaltimer the wait records
// kKernelWaitTimeout in the context's error word and returns false, and the kernel returns. The
// host side is the ordinary operator epilogue: wait_stream reads the error word, returns
// QPUCUDA_TIMEOUT and poisons the context (the reference's rule, qpu_llama_runtime.c:616-619).
#include "qpucuda_internal.h"
#include "sm100_sync.cuh"

namespace qpucuda {
namespace {

__global__ void __launch_bounds__(32) wait_expiry_probe_kernel(uint64_t limit_ns, unsigned int *error_word) {
    __shared__ __align__(8) uint64_t barrier;
    __shared__ int abort_flag;
    if (threadIdx.x == 0) {
        sm100::mbar_init(sm100::smem_u32(&barrier), 1);
        abort_flag = 0;
        sm100::mbar_init_fence();
    }
    __syncwarp();
    if (threadIdx.x == 0) {
        // Phase 0 never completes: the bound is what ends this wait.
        (void)sm100::wait_bounded_ns(sm100::smem_u32(&barrier), 0, &abort_flag, error_word, limit_ns);
    }
    __syncwarp();
}

}  // namespace
}  // namespace qpucuda

using namespace qpucuda;

extern "C" qpucuda_status qpucuda_context_probe_wait_expiry(qpucuda_context *context, uint64_t wait_limit_ns) {
    if (context == nullptr) return QPUCUDA_INVALID_ARGUMENT;
    if (wait_limit_ns == 0 || wait_limit_ns > kKernelWaitLimitNs) {
        return fail(context, QPUCUDA_INVALID_ARGUMENT, "wait-expiry probe: the bound must be 1 .. %llu ns",
                    static_cast<unsigned long long>(kKernelWaitLimitNs));
    }
    std::lock_guard<std::mutex> lock(context->mutex);
    const qpucuda_status status = begin_submit(context);
    if (status != QPUCUDA_OK) return status;
    DeviceGuard guard(context->device);
    wait_expiry_probe_kernel<<<1, 32, 0, context->stream>>>(wait_limit_ns, context->d_error);
    const cudaError_t error = cudaGetLastError();
    if (error != cudaSuccess) return cuda_fail(context, error, "wait-expiry probe launch");
    return wait_stream(context);
}
