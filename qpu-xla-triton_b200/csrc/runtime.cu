// qpucuda context: device selection, stream, bounded waits, status strings,
// host-side fault injection. Mirrors the conventions of the reference's
// native runtime (integrations/llama_cpp/src/qpu_llama_runtime.c):
// 10 s default wait timeout (:22, :293-295), failure_mask checks before the
// matching operation (:160, :301, :625, :698-716), a context poisoned after a
// failed wait that rejects further submissions with IO_FAILED (:616-623).
#include <time.h>

#include <chrono>
#include <cstdio>
#include <cstring>
#include <new>
#include <thread>
#include <vector>

#include "qpucuda_internal.h"

namespace qpucuda {

namespace {
constexpr uint64_t kDefaultTimeoutNs = 10ull * 1000ull * 1000ull * 1000ull;
}

uint64_t monotonic_ns() {
    timespec value;
    if (clock_gettime(CLOCK_MONOTONIC, &value) != 0) return 0;
    return static_cast<uint64_t>(value.tv_sec) * 1000000000ull + static_cast<uint64_t>(value.tv_nsec);
}

bool multiply_size(size_t left, size_t right, size_t *result) {
    if (left != 0 && right > SIZE_MAX / left) return false;
    *result = left * right;
    return true;
}

bool valid_range(size_t total, size_t offset, size_t size) { return offset <= total && size <= total - offset; }

void parallel_memcpy(void *destination, const void *source, size_t bytes) {
    constexpr size_t kChunkFloor = 8u << 20;
    const unsigned hardware = std::thread::hardware_concurrency();
    // Eight threads saturate a B200 host's memory copy rate (74 GB/s on 16 cores, 448 MiB);
    // more threads than half the cores ran slower.
    size_t workers = bytes / kChunkFloor;
    if (workers > 8) workers = 8;
    if (hardware >= 2 && workers > hardware / 2) workers = hardware / 2;
    if (workers <= 1) {
        std::memcpy(destination, source, bytes);
        return;
    }
    const size_t chunk = (bytes + workers - 1) / workers;
    auto copy_chunk = [=](size_t index) {
        const size_t begin = index * chunk;
        if (begin >= bytes) return;
        const size_t length = begin + chunk <= bytes ? chunk : bytes - begin;
        std::memcpy(static_cast<uint8_t *>(destination) + begin, static_cast<const uint8_t *>(source) + begin, length);
    };
    std::vector<std::thread> threads;
    size_t started = 0;
    try {
        threads.reserve(workers);
        for (; started < workers; ++started) threads.emplace_back(copy_chunk, started);
    } catch (...) {
        // No thread or memory to spare: nothing may throw across the C ABI, so the chunks that
        // found no thread are copied by the caller's thread below.
    }
    for (size_t index = started; index < workers; ++index) copy_chunk(index);
    for (auto &thread : threads) thread.join();
}

qpucuda_status fail(qpucuda_context *context, qpucuda_status status, const char *format, ...) {
    if (context != nullptr) {
        va_list args;
        va_start(args, format);
        vsnprintf(context->last_error, sizeof(context->last_error), format, args);
        va_end(args);
    }
    return status;
}

qpucuda_status cuda_fail(qpucuda_context *context, cudaError_t error, const char *operation,
                         qpucuda_status status) {
    (void)cudaGetLastError();  // clear a sticky launch error so later calls see their own
    return fail(context, status, "%s: %s", operation, cudaGetErrorString(error));
}

qpucuda_status begin_submit(qpucuda_context *context) {
    if (context->poisoned) {
        return fail(context, QPUCUDA_IO_FAILED, "CUDA context is poisoned after a wait failure");
    }
    if ((context->failure_mask & QPUCUDA_FAIL_SUBMISSION) != 0) {
        return fail(context, QPUCUDA_SUBMISSION_FAILED, "injected kernel submission failure");
    }
    return QPUCUDA_OK;
}

qpucuda_status wait_stream(qpucuda_context *context) {
    cudaError_t error = cudaMemcpyAsync(context->h_error, context->d_error, sizeof(unsigned int),
                                        cudaMemcpyDeviceToHost, context->stream);
    if (error == cudaSuccess) error = cudaEventRecord(context->done_event, context->stream);
    if (error != cudaSuccess) {
        context->poisoned = true;
        return cuda_fail(context, error, "record completion event", QPUCUDA_IO_FAILED);
    }
    const uint64_t start = monotonic_ns();
    uint64_t polls = 0;
    for (;;) {
        error = cudaEventQuery(context->done_event);
        if (error == cudaSuccess) break;
        if (error != cudaErrorNotReady) {
            context->poisoned = true;
            return cuda_fail(context, error, "wait for CUDA work", QPUCUDA_IO_FAILED);
        }
        const uint64_t elapsed = monotonic_ns() - start;
        if (elapsed > context->timeout_ns) {
            context->poisoned = true;
            return fail(context, QPUCUDA_TIMEOUT, "CUDA work did not complete within %llu ns",
                        static_cast<unsigned long long>(context->timeout_ns));
        }
        // Spin briefly for short kernels, then back off.
        if (++polls > 2000) std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
    if ((context->failure_mask & QPUCUDA_FAIL_WAIT) != 0) {
        context->poisoned = true;
        return fail(context, QPUCUDA_TIMEOUT, "injected wait timeout");
    }
    if (*context->h_error != kKernelOk) {
        context->poisoned = true;
        return fail(context, QPUCUDA_TIMEOUT, "a kernel barrier wait exceeded its bound (code %u)",
                    *context->h_error);
    }
    return QPUCUDA_OK;
}

DeviceGuard::DeviceGuard(int device) {
    if (cudaGetDevice(&previous_) == cudaSuccess && previous_ != device) {
        changed_ = cudaSetDevice(device) == cudaSuccess;
    }
}

DeviceGuard::~DeviceGuard() {
    if (changed_) (void)cudaSetDevice(previous_);
}

namespace {
using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled_fn() {
    static EncodeTiledFn fn = []() -> EncodeTiledFn {
        void *pointer = nullptr;
        cudaDriverEntryPointQueryResult query;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &pointer, cudaEnableDefault, &query) != cudaSuccess ||
            query != cudaDriverEntryPointSuccess) {
            return nullptr;
        }
        return reinterpret_cast<EncodeTiledFn>(pointer);
    }();
    return fn;
}
}  // namespace

bool encode_tensor_map_2d_u8(CUtensorMap *map, const void *base, uint64_t inner_bytes, uint64_t rows,
                             uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_rows) {
    EncodeTiledFn fn = encode_tiled_fn();
    if (fn == nullptr) return false;
    if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0 || (row_stride_bytes & 15u) != 0) return false;
    const cuuint64_t dims[2] = {inner_bytes, rows};
    const cuuint64_t strides[1] = {row_stride_bytes};
    const cuuint32_t box[2] = {box_inner, box_rows};
    const cuuint32_t element_strides[2] = {1, 1};
    const CUresult result =
        fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims, strides, box, element_strides,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return result == CUDA_SUCCESS;
}

bool encode_tensor_map_2d_b32(CUtensorMap *map, const void *base, uint64_t columns, uint64_t rows,
                              uint64_t row_stride_bytes, uint32_t box_columns, uint32_t box_rows) {
    EncodeTiledFn fn = encode_tiled_fn();
    if (fn == nullptr) return false;
    if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0 || (row_stride_bytes & 15u) != 0) return false;
    const cuuint64_t dims[2] = {columns, rows};
    const cuuint64_t strides[1] = {row_stride_bytes};
    const cuuint32_t box[2] = {box_columns, box_rows};
    const cuuint32_t element_strides[2] = {1, 1};
    const CUresult result =
        fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<void *>(base), dims, strides, box, element_strides,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return result == CUDA_SUCCESS;
}

bool encode_tensor_map_2d_f32(CUtensorMap *map, const void *base, uint64_t columns, uint64_t rows,
                              uint64_t row_stride_bytes, uint32_t box_columns, uint32_t box_rows) {
    EncodeTiledFn fn = encode_tiled_fn();
    if (fn == nullptr) return false;
    if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0 || (row_stride_bytes & 15u) != 0 || (box_columns * 4u) % 16u != 0) {
        return false;
    }
    const cuuint64_t dims[2] = {columns, rows};
    const cuuint64_t strides[1] = {row_stride_bytes};
    const cuuint32_t box[2] = {box_columns, box_rows};
    const cuuint32_t element_strides[2] = {1, 1};
    const CUresult result =
        fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void *>(base), dims, strides, box, element_strides,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return result == CUDA_SUCCESS;
}

}  // namespace qpucuda

using namespace qpucuda;

extern "C" {

qpucuda_status qpucuda_context_create(const qpucuda_context_config *config, qpucuda_context **result) {
    if (result == nullptr) return QPUCUDA_INVALID_ARGUMENT;
    *result = nullptr;
    qpucuda_context *context = new (std::nothrow) qpucuda_context();
    if (context == nullptr) return QPUCUDA_ALLOCATION_FAILED;
    context->timeout_ns = config != nullptr && config->timeout_ns != 0 ? config->timeout_ns : kDefaultTimeoutNs;
    context->failure_mask = config != nullptr ? config->failure_mask : 0;
    if ((context->failure_mask & QPUCUDA_FAIL_DEVICE_OPEN) != 0) {
        delete context;
        return QPUCUDA_DEVICE_UNAVAILABLE;
    }
    int device = config != nullptr ? config->device_ordinal : -1;
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess || count <= 0) {
        (void)cudaGetLastError();
        delete context;
        return QPUCUDA_DEVICE_UNAVAILABLE;
    }
    if (device < 0 && cudaGetDevice(&device) != cudaSuccess) device = 0;
    if (device >= count) {
        delete context;
        return QPUCUDA_INVALID_ARGUMENT;
    }
    context->device = device;
    DeviceGuard guard(device);
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) {
        delete context;
        return QPUCUDA_DEVICE_UNAVAILABLE;
    }
    std::snprintf(context->device_name, sizeof(context->device_name), "%s", prop.name);
    context->sm_count = prop.multiProcessorCount;
    context->cc_major = prop.major;
    context->cc_minor = prop.minor;
    context->l2_bytes = prop.l2CacheSize;
    context->global_bytes = prop.totalGlobalMem;
    if ((context->failure_mask & QPUCUDA_FAIL_ALLOCATION) != 0 ||
        cudaStreamCreateWithFlags(&context->own_stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaEventCreateWithFlags(&context->done_event, cudaEventDisableTiming) != cudaSuccess ||
        cudaMalloc(reinterpret_cast<void **>(&context->d_error), sizeof(unsigned int)) != cudaSuccess ||
        cudaMallocHost(reinterpret_cast<void **>(&context->h_error), sizeof(unsigned int)) != cudaSuccess ||
        cudaMemset(context->d_error, 0, sizeof(unsigned int)) != cudaSuccess) {
        (void)cudaGetLastError();
        qpucuda_context_destroy(context);
        return QPUCUDA_ALLOCATION_FAILED;
    }
    *context->h_error = 0;
    context->stream = config != nullptr && config->stream != nullptr ? static_cast<cudaStream_t>(config->stream)
                                                                     : context->own_stream;
    *result = context;
    return QPUCUDA_OK;
}

void qpucuda_context_destroy(qpucuda_context *context) {
    if (context == nullptr) return;
    {
        DeviceGuard guard(context->device);
        if (context->done_event != nullptr && !context->poisoned) (void)wait_stream(context);
        if (context->done_event != nullptr) cudaEventDestroy(context->done_event);
        if (context->own_stream != nullptr) cudaStreamDestroy(context->own_stream);
        if (context->d_error != nullptr) cudaFree(context->d_error);
        if (context->h_error != nullptr) cudaFreeHost(context->h_error);
        (void)cudaGetLastError();
    }
    delete context;
}

const char *qpucuda_context_last_error(const qpucuda_context *context) {
    return context != nullptr ? context->last_error : "no context";
}

qpucuda_status qpucuda_context_capabilities(const qpucuda_context *context, qpucuda_capabilities *result) {
    if (context == nullptr || result == nullptr) return QPUCUDA_INVALID_ARGUMENT;
    std::memset(result, 0, sizeof(*result));
    std::snprintf(result->device_name, sizeof(result->device_name), "%s", context->device_name);
    result->device_ordinal = context->device;
    result->compute_capability_major = context->cc_major;
    result->compute_capability_minor = context->cc_minor;
    result->multiprocessor_count = context->sm_count;
    result->global_memory_bytes = context->global_bytes;
    result->l2_cache_bytes = context->l2_bytes;
    result->supports_tcgen05 = context->cc_major == 10 && context->cc_minor == 0 ? 1 : 0;
    return QPUCUDA_OK;
}

void qpucuda_context_set_failure_mask(qpucuda_context *context, uint32_t failure_mask) {
    if (context == nullptr) return;
    std::lock_guard<std::mutex> lock(context->mutex);
    context->failure_mask = failure_mask;
}

qpucuda_status qpucuda_context_set_stream(qpucuda_context *context, void *stream) {
    if (context == nullptr) return QPUCUDA_INVALID_ARGUMENT;
    std::lock_guard<std::mutex> lock(context->mutex);
    context->stream = static_cast<cudaStream_t>(stream);
    return QPUCUDA_OK;
}

void *qpucuda_context_stream(const qpucuda_context *context) {
    return context != nullptr ? static_cast<void *>(context->stream) : nullptr;
}

void *qpucuda_context_library_stream(const qpucuda_context *context) {
    return context != nullptr ? static_cast<void *>(context->own_stream) : nullptr;
}

qpucuda_status qpucuda_context_synchronize(qpucuda_context *context) {
    if (context == nullptr) return QPUCUDA_INVALID_ARGUMENT;
    std::lock_guard<std::mutex> lock(context->mutex);
    if (context->poisoned) return fail(context, QPUCUDA_IO_FAILED, "CUDA context is poisoned after a wait failure");
    DeviceGuard guard(context->device);
    return wait_stream(context);
}

int qpucuda_context_poisoned(const qpucuda_context *context) {
    return context != nullptr && context->poisoned ? 1 : 0;
}

const char *qpucuda_status_string(qpucuda_status status) {
    switch (status) {
        case QPUCUDA_OK: return "ok";
        case QPUCUDA_INVALID_ARGUMENT: return "invalid argument";
        case QPUCUDA_DEVICE_UNAVAILABLE: return "device unavailable";
        case QPUCUDA_CAPABILITY_MISSING: return "capability missing";
        case QPUCUDA_ALLOCATION_FAILED: return "allocation failed";
        case QPUCUDA_IO_FAILED: return "I/O failed";
        case QPUCUDA_SUBMISSION_FAILED: return "submission failed";
        case QPUCUDA_TIMEOUT: return "timeout";
        case QPUCUDA_HASH_MISMATCH: return "hash mismatch";
        case QPUCUDA_INTERNAL_ERROR: return "internal error";
    }
    return "unknown status";
}

const char *qpucuda_build_info(void) { return QPUCUDA_VERSION " sm_100a"; }

}  // extern "C"
