// W8A8 linear over caller-provided buffers with no allocation at all.
//
// Some callers of this library cannot call cudaMalloc when they run the
// operator: code that executes under an allocator it must not re-enter (a
// framework's memory-pool callback, a real-time loop with a frozen memory
// budget), or a process whose device memory is fully committed up front. The
// prepared linear allocates its activation scratch (the int8 rows and their
// scales) at prepare time, so it cannot serve them. This entry point runs the
// same two kernels (row quantizer, then the tcgen05 GEMM or the GEMV with the
// fused dequant/bias epilogue) with that scratch placed in a fixed device array
// compiled into the library, and calls no allocating routine.
//
// The array's host-side name is not a device address: at set-up, once per
// device, with that device current, cudaGetSymbolAddress yields the address the
// kernels get. That set-up happens inside the first call on each device, which
// also loads and configures every kernel the entry point can launch; it may
// allocate (CUDA's lazy module loading), so make that first call at start-up,
// outside any region where allocation is forbidden and before any stream capture.
#include <climits>
#include <mutex>

#include "qpucuda_internal.h"
#include "qpucuda_w8a8.h"

using namespace qpucuda;

namespace {

// Fixed scratch: rows * padded K int8 activations, then rows fp32 row scales (256-byte aligned).
static __device__ __align__(256) uint8_t g_static_scratch[QPUCUDA_STATIC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;

// Per device: the array's address and the id of the CUDA context it was resolved in. A device
// reset (or a released and re-created primary context) gives a new context id, and the set-up
// runs again there instead of handing the kernels an address of the old context.
struct ScratchSlot {
    unsigned long long context_id = 0;
    uint8_t *address = nullptr;
};
std::mutex g_setup_mutex;
ScratchSlot g_slots[kMaxDevices];

using CtxGetCurrentFn = CUresult (*)(CUcontext *);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long *);

template <typename Fn>
Fn driver_function(const char *name) {
    void *pointer = nullptr;
    cudaDriverEntryPointQueryResult query;
    if (cudaGetDriverEntryPoint(name, &pointer, cudaEnableDefault, &query) != cudaSuccess ||
        query != cudaDriverEntryPointSuccess) {
        (void)cudaGetLastError();
        return nullptr;
    }
    return reinterpret_cast<Fn>(pointer);
}

// Id of the context current on this thread; false when none is bound yet (or the driver lacks
// the query), in which case the set-up simply runs again.
bool current_context_id(unsigned long long *id) {
    static const CtxGetCurrentFn get_current = driver_function<CtxGetCurrentFn>("cuCtxGetCurrent");
    static const CtxGetIdFn get_id = driver_function<CtxGetIdFn>("cuCtxGetId");
    CUcontext context = nullptr;
    if (get_current == nullptr || get_id == nullptr || get_current(&context) != CUDA_SUCCESS || context == nullptr) {
        return false;
    }
    return get_id(context, id) == CUDA_SUCCESS;
}

// The scratch address for the context's device (current, via DeviceGuard), set up on first use
// in each CUDA context: symbol lookup, then every kernel variant loaded and configured.
qpucuda_status scratch_address(qpucuda_context *context, uint8_t **address) {
    if (context->device < 0 || context->device >= kMaxDevices) {
        return fail(context, QPUCUDA_CAPABILITY_MISSING, "no-alloc W8A8 linear: device ordinal beyond %d", kMaxDevices);
    }
    unsigned long long id = 0;
    bool have_id = current_context_id(&id);
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    ScratchSlot &slot = g_slots[context->device];
    if (have_id && slot.address != nullptr && slot.context_id == id) {
        *address = slot.address;
        return QPUCUDA_OK;
    }
    void *pointer = nullptr;
    cudaError_t error = cudaGetSymbolAddress(&pointer, g_static_scratch);
    if (error != cudaSuccess || pointer == nullptr) {
        return cuda_fail(context, error, "no-alloc W8A8 linear: cudaGetSymbolAddress", QPUCUDA_DEVICE_UNAVAILABLE);
    }
    error = preload_quantize_rows_int8();
    if (error == cudaSuccess) error = preload_w8a8_gemv();
    if (error == cudaSuccess && context->cc_major == 10 && context->cc_minor == 0)
        error = preload_w8a8_gemm_sm100(context->sm_count);
    if (error != cudaSuccess) {
        return cuda_fail(context, error, "no-alloc W8A8 linear: kernel set-up", QPUCUDA_DEVICE_UNAVAILABLE);
    }
    if (!have_id) have_id = current_context_id(&id);  // the lookup above bound the context
    slot.context_id = have_id ? id : 0;
    slot.address = have_id ? static_cast<uint8_t *>(pointer) : nullptr;  // no id: set up again next call
    *address = static_cast<uint8_t *>(pointer);
    return QPUCUDA_OK;
}

}  // namespace

extern "C" {

qpucuda_status qpucuda_w8a8_linear_execute_static(qpucuda_context *context, const float *source, size_t source_stride,
                                                  uint32_t rows, const int8_t *weight, size_t weight_stride,
                                                  const float *weight_scales, const float *bias, uint32_t k,
                                                  uint32_t n, float *destination, size_t destination_stride) {
    if (context == nullptr) return QPUCUDA_INVALID_ARGUMENT;
    const uint32_t k_pad = (k + 15u) & ~15u;
    if (source == nullptr || weight == nullptr || weight_scales == nullptr || destination == nullptr || rows == 0 ||
        k == 0 || n == 0 || source_stride < k || weight_stride < k_pad || weight_stride % 16 != 0 ||
        (reinterpret_cast<uintptr_t>(weight) & 15u) != 0 || destination_stride < n ||
        static_cast<uint64_t>(k) * 127u * 127u > static_cast<uint64_t>(INT32_MAX)) {
        return fail(context, QPUCUDA_INVALID_ARGUMENT,
                    "no-alloc W8A8 linear: weight rows must be 16-byte aligned with stride >= K rounded up to 16, "
                    "and K * 127^2 <= INT32_MAX");
    }
    const uint64_t activation_bytes = static_cast<uint64_t>(rows) * k_pad;
    const uint64_t scales_offset = (activation_bytes + 255u) & ~static_cast<uint64_t>(255u);
    if (scales_offset + static_cast<uint64_t>(rows) * sizeof(float) > QPUCUDA_STATIC_SCRATCH_BYTES) {
        return fail(context, QPUCUDA_INVALID_ARGUMENT,
                    "no-alloc W8A8 linear: rows * padded K (%llu bytes) plus row scales exceed the fixed %u-byte "
                    "scratch; use the prepared linear for larger batches",
                    static_cast<unsigned long long>(activation_bytes), static_cast<unsigned>(QPUCUDA_STATIC_SCRATCH_BYTES));
    }
    if (rows > 8 && !(context->cc_major == 10 && context->cc_minor == 0)) {
        return fail(context, QPUCUDA_CAPABILITY_MISSING, "the tcgen05 int8 GEMM needs an sm_100 device");
    }
    std::lock_guard<std::mutex> lock(context->mutex);
    qpucuda_status status = begin_submit(context);
    if (status != QPUCUDA_OK) return status;
    DeviceGuard guard(context->device);
    uint8_t *scratch = nullptr;
    status = scratch_address(context, &scratch);
    if (status != QPUCUDA_OK) return status;
    int8_t *quantized = reinterpret_cast<int8_t *>(scratch);
    float *row_scales = reinterpret_cast<float *>(scratch + scales_offset);
    // The quantizer rewrites every byte the GEMM reads (all rows x padded K, zeros in the padding,
    // and every row scale), so nothing left from an earlier call needs clearing.
    cudaError_t error = launch_quantize_rows_int8(source, source_stride, rows, k, k_pad, quantized, k_pad, row_scales,
                                                  context->d_error, context->stream);
    if (error != cudaSuccess) return cuda_fail(context, error, "no-alloc W8A8 linear: quantize");
    GemmEpilogue epilogue;
    epilogue.mode = bias != nullptr ? EpilogueMode::kDequantizeBias : EpilogueMode::kDequantize;
    epilogue.row_scales = row_scales;
    epilogue.col_scales = weight_scales;
    epilogue.bias = bias;
    epilogue.out = destination;
    epilogue.out_stride = destination_stride;
    if (rows <= 8) {
        error = launch_w8a8_gemv(quantized, k_pad, weight, weight_stride, rows, n, k_pad, epilogue, context->sm_count,
                                 context->stream);
    } else {
        error = run_w8a8_gemm(quantized, k_pad, weight, weight_stride, rows, n, k_pad, epilogue, context->d_error,
                              context->sm_count, context->stream);
    }
    if (error == cudaErrorInvalidValue) return cuda_fail(context, error, "no-alloc W8A8 linear", QPUCUDA_INVALID_ARGUMENT);
    if (error != cudaSuccess) return cuda_fail(context, error, "no-alloc W8A8 linear");
    return QPUCUDA_OK;
}

}  // extern "C"
