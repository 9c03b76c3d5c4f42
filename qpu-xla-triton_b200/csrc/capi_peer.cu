// Peer memory for the fused W8A8 linear + all-gather (include/qpucuda_peer.h):
// device buffers that the other processes of a one-node job map with CUDA IPC.
// No counterpart in the reference (its output split joins in host memory,
// src/qpu_xla/models/tinyllama/quantization.py:350-514).
#include <cstring>

#include "qpucuda_internal.h"
#include "qpucuda_peer.h"

using namespace qpucuda;

static_assert(sizeof(cudaIpcMemHandle_t) == QPUCUDA_PEER_HANDLE_BYTES, "IPC handle size");
static_assert(QPUCUDA_MAX_PEERS == kGemmMaxPeers, "peer limits must agree");

extern "C" {

qpucuda_status qpucuda_peer_buffer_create(qpucuda_context *context, size_t bytes, void **device_pointer,
                                          unsigned char *handle) {
    if (context == nullptr) return QPUCUDA_INVALID_ARGUMENT;
    if (device_pointer == nullptr || handle == nullptr || bytes == 0) {
        return fail(context, QPUCUDA_INVALID_ARGUMENT, "peer buffer: invalid arguments");
    }
    *device_pointer = nullptr;
    if ((context->failure_mask & QPUCUDA_FAIL_ALLOCATION) != 0) {
        return fail(context, QPUCUDA_ALLOCATION_FAILED, "injected device allocation failure");
    }
    std::lock_guard<std::mutex> lock(context->mutex);
    DeviceGuard guard(context->device);
    void *pointer = nullptr;
    cudaError_t error = cudaMalloc(&pointer, bytes);
    if (error != cudaSuccess) return cuda_fail(context, error, "peer buffer allocation", QPUCUDA_ALLOCATION_FAILED);
    cudaIpcMemHandle_t ipc;
    error = cudaIpcGetMemHandle(&ipc, pointer);
    if (error != cudaSuccess) {
        cudaFree(pointer);
        return cuda_fail(context, error, "peer buffer handle", QPUCUDA_ALLOCATION_FAILED);
    }
    std::memcpy(handle, &ipc, sizeof(ipc));
    *device_pointer = pointer;
    return QPUCUDA_OK;
}

qpucuda_status qpucuda_peer_buffer_open(qpucuda_context *context, const unsigned char *handle,
                                        void **device_pointer) {
    if (context == nullptr) return QPUCUDA_INVALID_ARGUMENT;
    if (device_pointer == nullptr || handle == nullptr) {
        return fail(context, QPUCUDA_INVALID_ARGUMENT, "peer buffer: invalid arguments");
    }
    *device_pointer = nullptr;
    std::lock_guard<std::mutex> lock(context->mutex);
    DeviceGuard guard(context->device);
    cudaIpcMemHandle_t ipc;
    std::memcpy(&ipc, handle, sizeof(ipc));
    void *pointer = nullptr;
    const cudaError_t error = cudaIpcOpenMemHandle(&pointer, ipc, cudaIpcMemLazyEnablePeerAccess);
    if (error != cudaSuccess) return cuda_fail(context, error, "peer buffer mapping", QPUCUDA_CAPABILITY_MISSING);
    *device_pointer = pointer;
    return QPUCUDA_OK;
}

qpucuda_status qpucuda_peer_buffer_close(qpucuda_context *context, void *device_pointer) {
    if (context == nullptr) return QPUCUDA_INVALID_ARGUMENT;
    if (device_pointer == nullptr) return fail(context, QPUCUDA_INVALID_ARGUMENT, "peer buffer: NULL pointer");
    std::lock_guard<std::mutex> lock(context->mutex);
    DeviceGuard guard(context->device);
    const cudaError_t error = cudaIpcCloseMemHandle(device_pointer);
    if (error != cudaSuccess) return cuda_fail(context, error, "peer buffer unmapping", QPUCUDA_INVALID_ARGUMENT);
    return QPUCUDA_OK;
}

qpucuda_status qpucuda_peer_buffer_destroy(qpucuda_context *context, void *device_pointer) {
    if (context == nullptr) return QPUCUDA_INVALID_ARGUMENT;
    if (device_pointer == nullptr) return fail(context, QPUCUDA_INVALID_ARGUMENT, "peer buffer: NULL pointer");
    std::lock_guard<std::mutex> lock(context->mutex);
    DeviceGuard guard(context->device);
    const cudaError_t error = cudaFree(device_pointer);
    if (error != cudaSuccess) return cuda_fail(context, error, "peer buffer free", QPUCUDA_INVALID_ARGUMENT);
    return QPUCUDA_OK;
}

qpucuda_status qpucuda_peer_copy_rows(qpucuda_context *context, void *destination, size_t destination_pitch,
                                      const void *source, size_t source_pitch, size_t width_bytes, size_t rows,
                                      void *stream) {
    if (context == nullptr) return QPUCUDA_INVALID_ARGUMENT;
    if (destination == nullptr || source == nullptr || width_bytes == 0 || rows == 0 || destination_pitch < width_bytes ||
        source_pitch < width_bytes) {
        return fail(context, QPUCUDA_INVALID_ARGUMENT, "peer copy: invalid arguments");
    }
    DeviceGuard guard(context->device);
    cudaStream_t target = stream != nullptr ? static_cast<cudaStream_t>(stream) : context->stream;
    const cudaError_t error = cudaMemcpy2DAsync(destination, destination_pitch, source, source_pitch, width_bytes, rows,
                                                cudaMemcpyDeviceToDevice, target);
    if (error != cudaSuccess) return cuda_fail(context, error, "peer copy", QPUCUDA_IO_FAILED);
    return QPUCUDA_OK;
}

}  // extern "C"
