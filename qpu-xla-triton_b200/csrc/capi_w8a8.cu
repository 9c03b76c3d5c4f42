// Prepared W8A8 linear (include/qpucuda_w8a8.h): the C-ABI form of
// PreparedW8A8Linear (src/qpu_xla/models/tinyllama/quantization.py:57-878).
//
// Per call: quantize the fp32 rows into the plan's int8 scratch (quantization.py:156-171),
// then either the int8 GEMV (rows <= 8; the reference's batch == 1 GEMV choice,
// :184) or the tcgen05 GEMM, with the dequant (+bias) epilogue fused
// (gemm_int8.py:166-184). Weight rows are padded with zeros to a multiple of 16
// bytes of K, as the reference pads its packed operands (quantization.py:85-87).
#include <cfloat>
#include <climits>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <new>
#include <chrono>
#include <thread>
#include <vector>

#include "qpucuda_internal.h"
#include "qpucuda_peer.h"
#include "qpucuda_w8a8.h"

using namespace qpucuda;

struct qpucuda_w8a8_linear {
    qpucuda_context *context = nullptr;
    uint32_t k = 0;        // input features
    uint32_t k_pad = 0;    // K rounded up to 16
    uint32_t columns = 0;  // resident output columns
    uint32_t max_batch = 0;
    bool has_bias = false;
    int8_t *d_weight = nullptr;        // [columns][k_pad]
    float *d_weight_scales = nullptr;  // [columns]
    float *d_bias = nullptr;           // [columns] or null
    int8_t *d_quantized = nullptr;     // scratch [max_batch][k_pad]
    float *d_row_scales = nullptr;     // scratch [max_batch]
    // Split-K workspace for batches of 9..splitk_rows rows whose output tiles leave most SMs idle:
    // int32 partial rows [splitk_max][splitk_rows][columns], or null when no batch needs it.
    int32_t *d_splitk = nullptr;
    uint32_t splitk_max = 1;
    uint32_t splitk_rows = 0;  // a multiple of kGemmBlockM
    CUtensorMap map_weight;
    CUtensorMap map_quantized;
    bool maps_ready = false;
    // Host-buffer path: device source/output and pinned output staging, allocated on first use.
    float *h_destination = nullptr;
    float *d_source = nullptr;
    float *d_destination = nullptr;
    // Host-buffer path for large batches: copy streams and per-slice events, made on first use.
    cudaStream_t copy_in = nullptr;
    cudaStream_t copy_out = nullptr;
    std::vector<cudaEvent_t> events;
    // Asynchronous submissions: a page-locked copy of the kernel error word per plan, read after
    // the submission's completion event.
    unsigned int *h_submit_error = nullptr;
    size_t resident_bytes = 0;
    bool busy = false;
    std::mutex mutex;
};

namespace {

constexpr uint32_t kGemvMaxRows = 8;

bool accumulation_fits(uint32_t k) { return static_cast<uint64_t>(k) * 127u * 127u <= static_cast<uint64_t>(INT32_MAX); }

void free_linear(qpucuda_w8a8_linear *linear) {
    DeviceGuard guard(linear->context->device);
    cudaFree(linear->d_weight);
    cudaFree(linear->d_weight_scales);
    cudaFree(linear->d_bias);
    cudaFree(linear->d_quantized);
    cudaFree(linear->d_row_scales);
    cudaFree(linear->d_splitk);
    if (linear->h_submit_error != nullptr) cudaFreeHost(linear->h_submit_error);
    cudaFree(linear->d_source);
    cudaFree(linear->d_destination);
    cudaFreeHost(linear->h_destination);
    if (linear->copy_in != nullptr) cudaStreamDestroy(linear->copy_in);
    if (linear->copy_out != nullptr) cudaStreamDestroy(linear->copy_out);
    for (cudaEvent_t event : linear->events) cudaEventDestroy(event);
    (void)cudaGetLastError();
    delete linear;
}

constexpr uint32_t kSliceRows = 1024;

bool ensure_pipeline(qpucuda_w8a8_linear *linear, uint32_t slices) {
    // Each stream on its own: after a failed creation the other stays usable, and a null handle
    // (the legacy default stream) is never used as a copy stream.
    for (cudaStream_t *stream : {&linear->copy_in, &linear->copy_out}) {
        if (*stream == nullptr && cudaStreamCreateWithFlags(stream, cudaStreamNonBlocking) != cudaSuccess) {
            *stream = nullptr;
            (void)cudaGetLastError();
            return false;
        }
    }
    const size_t needed = 2u * slices + 3u;
    try {
        linear->events.reserve(needed);
    } catch (...) {
        return false;  // no exception crosses the C ABI
    }
    while (linear->events.size() < needed) {
        cudaEvent_t event = nullptr;
        if (cudaEventCreateWithFlags(&event, cudaEventDisableTiming) != cudaSuccess) {
            (void)cudaGetLastError();
            return false;
        }
        linear->events.push_back(event);  // capacity reserved above: does not throw
    }
    return true;
}

qpucuda_status enqueue(qpucuda_w8a8_linear *linear, const float *source, size_t source_stride,
                       const int8_t *quantized, size_t quantized_stride, const float *row_scales, uint32_t rows,
                       float *destination, size_t destination_stride);

// Pipelined host-buffer execution: slice s is copied in on copy_in, quantized and multiplied on
// the context stream after its copy, and copied out to host_out (the plan's pinned staging, or
// the caller's page-locked destination in direct mode) on copy_out after its
// GEMM (events 1 + 2s copied in, 2 + 2s computed); the last copy-out is joined back into the
// context stream, whose bounded wait then covers every copy and kernel of the call.
qpucuda_status enqueue_sliced(qpucuda_w8a8_linear *linear, const float *source, uint32_t rows, uint32_t slices,
                              float *host_out, bool join = true) {
    qpucuda_context *context = linear->context;
    cudaEvent_t *events = linear->events.data();
    // The source copies only write this plan's device staging, which nothing else reads and whose
    // previous reader (this plan's previous invocation) has finished: a plan admits one invocation
    // at a time and every host-buffer call is waited before the next. So they do not wait for
    // earlier work on the context stream, and the next plan's source streams in while this one
    // computes and copies out (three queued 70B FFN projections: 28.4 -> 22.2 ms, the PCIe floor
    // of the same copies being 21.5 ms). The result copies follow their slice's compute anyway.
    cudaError_t error = cudaEventRecord(events[0], context->stream);
    if (error == cudaSuccess) error = cudaStreamWaitEvent(linear->copy_out, events[0], 0);
    if (error != cudaSuccess) return cuda_fail(context, error, "order W8A8 copy streams");
    for (uint32_t s = 0; s < slices; ++s) {
        const uint32_t first = s * kSliceRows;
        const uint32_t count = rows - first < kSliceRows ? rows - first : kSliceRows;
        cudaEvent_t copied = events[1 + 2 * s], computed = events[2 + 2 * s];
        error = cudaMemcpyAsync(linear->d_source + static_cast<size_t>(first) * linear->k,
                                source + static_cast<size_t>(first) * linear->k,
                                static_cast<size_t>(count) * linear->k * sizeof(float), cudaMemcpyHostToDevice,
                                linear->copy_in);
        if (error == cudaSuccess) error = cudaEventRecord(copied, linear->copy_in);
        if (error == cudaSuccess) error = cudaStreamWaitEvent(context->stream, copied, 0);
        if (error != cudaSuccess) return cuda_fail(context, error, "copy W8A8 source slice");
        const qpucuda_status status =
            enqueue(linear, linear->d_source + static_cast<size_t>(first) * linear->k, linear->k, nullptr, 0, nullptr,
                    count, linear->d_destination + static_cast<size_t>(first) * linear->columns, linear->columns);
        if (status != QPUCUDA_OK) return status;
        error = cudaEventRecord(computed, context->stream);
        if (error == cudaSuccess) error = cudaStreamWaitEvent(linear->copy_out, computed, 0);
        if (error == cudaSuccess)
            error = cudaMemcpyAsync(host_out + static_cast<size_t>(first) * linear->columns,
                                    linear->d_destination + static_cast<size_t>(first) * linear->columns,
                                    static_cast<size_t>(count) * linear->columns * sizeof(float),
                                    cudaMemcpyDeviceToHost, linear->copy_out);
        if (error != cudaSuccess) return cuda_fail(context, error, "copy W8A8 destination slice");
    }
    if (!join) return QPUCUDA_OK;  // an asynchronous submission waits on the copy stream itself
    cudaEvent_t done = events[1 + 2 * slices];
    error = cudaEventRecord(done, linear->copy_out);
    if (error == cudaSuccess) error = cudaStreamWaitEvent(context->stream, done, 0);
    if (error != cudaSuccess) return cuda_fail(context, error, "join W8A8 copy streams");
    return QPUCUDA_OK;
}

// Bounded drain of both copy streams after a failure, so the plan's staging is not reused while
// a copy into or out of it may still be running (the context is poisoned or failed by then).
void drain_copies(qpucuda_w8a8_linear *linear) {
    const uint64_t start = monotonic_ns();
    for (cudaStream_t stream : {linear->copy_in, linear->copy_out}) {
        while (cudaStreamQuery(stream) == cudaErrorNotReady && monotonic_ns() - start <= linear->context->timeout_ns) {
            std::this_thread::sleep_for(std::chrono::microseconds(50));
        }
    }
    (void)cudaGetLastError();
}

// Enqueue quantize + GEMM/GEMV + epilogue for `rows` rows already resident on the device.
// With peers, the same outputs are also written to each peer destination at the same
// offsets: by the GEMM epilogue itself, or, on the GEMV path (a few rows), by one 2-D copy
// per peer after the local result.
qpucuda_status enqueue_to(qpucuda_w8a8_linear *linear, const float *source, size_t source_stride,
                          const int8_t *quantized, size_t quantized_stride, const float *row_scales, uint32_t rows,
                          float *destination, size_t destination_stride, float *const *peers, uint32_t peer_count) {
    qpucuda_context *context = linear->context;
    cudaStream_t stream = context->stream;
    GemmEpilogue epilogue;
    epilogue.mode = linear->has_bias ? EpilogueMode::kDequantizeBias : EpilogueMode::kDequantize;
    epilogue.col_scales = linear->d_weight_scales;
    epilogue.bias = linear->d_bias;
    epilogue.out = destination;
    epilogue.out_stride = destination_stride;
    // A single fp32 row: the GEMV quantizes it itself (one launch instead of two) when the row is
    // short enough; it still leaves the int8 row and scale in the plan scratch.
    cudaError_t fused = cudaErrorNotSupported;
    if (source != nullptr && rows == 1) {
        epilogue.row_scales = linear->d_row_scales;
        fused = launch_w8a8_gemv_quantize(source, linear->k, linear->d_quantized, linear->d_row_scales,
                                          linear->d_weight, linear->k_pad, linear->columns, linear->k_pad, epilogue,
                                          context->sm_count, stream);
        if (fused != cudaSuccess && fused != cudaErrorNotSupported) return cuda_fail(context, fused, "W8A8 GEMV launch");
    }
    if (source != nullptr && fused != cudaSuccess) {
        const cudaError_t error = launch_quantize_rows_int8(source, source_stride, rows, linear->k, linear->k_pad,
                                                            linear->d_quantized, linear->k_pad, linear->d_row_scales,
                                                            context->d_error, stream);
        if (error != cudaSuccess) return cuda_fail(context, error, "quantize activations");
    }
    if (source != nullptr) {
        quantized = linear->d_quantized;
        quantized_stride = linear->k_pad;
        row_scales = linear->d_row_scales;
    }
    epilogue.row_scales = row_scales;
    cudaError_t error = cudaSuccess;
    if (rows <= kGemvMaxRows) {
        if (fused != cudaSuccess) {
            error = launch_w8a8_gemv(quantized, quantized_stride, linear->d_weight, linear->k_pad, rows,
                                     linear->columns, linear->k_pad, epilogue, context->sm_count, stream);
        }
        for (uint32_t p = 0; error == cudaSuccess && p < peer_count; ++p) {
            error = cudaMemcpy2DAsync(peers[p], destination_stride * sizeof(float), destination,
                                      destination_stride * sizeof(float), static_cast<size_t>(linear->columns) * sizeof(float),
                                      rows, cudaMemcpyDeviceToDevice, stream);
        }
    } else {
        epilogue.peer_count = peer_count;
        for (uint32_t p = 0; p < peer_count; ++p) epilogue.peer_out[p] = peers[p];
        uint32_t used_splits = 0;
        // slices for this batch: as many as the SMs left by its tiles allow, up to the workspace's
        const uint32_t tiles = ((rows + kGemmBlockM - 1) / kGemmBlockM) * ((linear->columns + kGemmBlockN - 1) / kGemmBlockN);
        uint32_t splits = static_cast<uint32_t>(context->sm_count) / tiles;
        splits = splits < linear->splitk_max ? splits : linear->splitk_max;
        if (peer_count == 0 && rows <= linear->splitk_rows && splits >= 2 && linear->d_splitk != nullptr &&
            quantized == linear->d_quantized && linear->maps_ready) {
            // few output tiles: K slices into the workspace, then one reduce + epilogue launch
            error = launch_w8a8_gemm_sm100_splitk(&linear->map_quantized, &linear->map_weight, rows, linear->columns,
                                                  linear->k_pad, linear->d_splitk, splits, context->d_error,
                                                  context->sm_count, stream, &used_splits);
            if (error == cudaSuccess)
                error = launch_w8a8_splitk_reduce(linear->d_splitk, used_splits, rows, linear->columns, epilogue,
                                                  context->sm_count, stream);
        } else if (quantized == linear->d_quantized && linear->maps_ready) {
            error = launch_w8a8_gemm_sm100(&linear->map_quantized, &linear->map_weight, rows, linear->columns,
                                           linear->k_pad, epilogue, context->d_error, context->sm_count, stream);
        } else {
            error = run_w8a8_gemm(quantized, quantized_stride, linear->d_weight, linear->k_pad, rows, linear->columns,
                                  linear->k_pad, epilogue, context->d_error, context->sm_count, stream);
        }
    }
    if (error == cudaErrorInvalidValue) return cuda_fail(context, error, "W8A8 GEMM launch", QPUCUDA_INVALID_ARGUMENT);
    if (error != cudaSuccess) return cuda_fail(context, error, "W8A8 GEMM launch");
    return QPUCUDA_OK;
}

qpucuda_status enqueue(qpucuda_w8a8_linear *linear, const float *source, size_t source_stride,
                       const int8_t *quantized, size_t quantized_stride, const float *row_scales, uint32_t rows,
                       float *destination, size_t destination_stride) {
    return enqueue_to(linear, source, source_stride, quantized, quantized_stride, row_scales, rows, destination,
                      destination_stride, nullptr, 0);
}

}  // namespace

extern "C" {

qpucuda_status qpucuda_w8a8_linear_prepare(qpucuda_context *context, const qpucuda_w8a8_linear_desc *desc,
                                           qpucuda_w8a8_linear **result) {
    if (context == nullptr || desc == nullptr || result == nullptr) return QPUCUDA_INVALID_ARGUMENT;
    *result = nullptr;
    const uint32_t count = desc->resident_output_count != 0 ? desc->resident_output_count
                                                             : (desc->output_features > desc->resident_output_start
                                                                    ? desc->output_features - desc->resident_output_start
                                                                    : 0);
    if (desc->weight_values == nullptr || desc->weight_scales == nullptr || desc->input_features == 0 ||
        desc->output_features == 0 || desc->max_batch == 0 || count == 0 ||
        desc->resident_output_start > desc->output_features ||
        count > desc->output_features - desc->resident_output_start ||
        (desc->memory != QPUCUDA_MEMORY_HOST && desc->memory != QPUCUDA_MEMORY_DEVICE)) {
        return fail(context, QPUCUDA_INVALID_ARGUMENT, "w8a8 prepare: invalid weight descriptor");
    }
    if (!accumulation_fits(desc->input_features)) {
        // quantization.py:90-91
        return fail(context, QPUCUDA_INVALID_ARGUMENT, "prepared W8A8 linear accumulation can overflow int32");
    }
    const size_t start = desc->resident_output_start;
    if (desc->memory == QPUCUDA_MEMORY_HOST) {
        // QuantizedMatrixInt8 invariant (quantization.py:45-46): finite, positive scales.
        for (uint32_t i = 0; i < count; ++i) {
            const float s = desc->weight_scales[start + i];
            if (!std::isfinite(s) || s <= 0.0f) {
                return fail(context, QPUCUDA_INVALID_ARGUMENT, "quantized matrix scales must be finite and positive");
            }
        }
    }
    std::lock_guard<std::mutex> lock(context->mutex);
    if (context->poisoned) return fail(context, QPUCUDA_IO_FAILED, "CUDA context is poisoned after a wait failure");
    if ((context->failure_mask & QPUCUDA_FAIL_ALLOCATION) != 0) {
        return fail(context, QPUCUDA_ALLOCATION_FAILED, "injected device allocation failure");
    }
    qpucuda_w8a8_linear *linear = new (std::nothrow) qpucuda_w8a8_linear();
    if (linear == nullptr) return QPUCUDA_ALLOCATION_FAILED;
    linear->context = context;
    linear->k = desc->input_features;
    linear->k_pad = (desc->input_features + 15u) & ~15u;
    linear->columns = count;
    linear->max_batch = desc->max_batch;
    linear->has_bias = desc->bias != nullptr;
    DeviceGuard guard(context->device);
    const size_t weight_bytes = static_cast<size_t>(count) * linear->k_pad;
    const size_t scratch_bytes = static_cast<size_t>(desc->max_batch) * linear->k_pad;
    cudaError_t error = cudaMalloc(reinterpret_cast<void **>(&linear->d_weight), weight_bytes);
    if (error == cudaSuccess) error = cudaMalloc(reinterpret_cast<void **>(&linear->d_weight_scales), count * sizeof(float));
    if (error == cudaSuccess && linear->has_bias)
        error = cudaMalloc(reinterpret_cast<void **>(&linear->d_bias), count * sizeof(float));
    if (error == cudaSuccess) error = cudaMalloc(reinterpret_cast<void **>(&linear->d_quantized), scratch_bytes);
    if (error == cudaSuccess)
        error = cudaMalloc(reinterpret_cast<void **>(&linear->d_row_scales), desc->max_batch * sizeof(float));
    // Split-K pays when a batch's output tiles (single-CTA, 128 x 256) fill at most half of the SMs
    // and the K stages are enough to share out: at most 8 slices, tiles x slices <= SMs. The
    // workspace covers the batches up to splitk_rows rows that qualify, within 64 MiB.
    const uint32_t row_block_tiles = (count + kGemmBlockN - 1) / kGemmBlockN;
    const uint32_t k_stages = (linear->k_pad + kGemmBlockK - 1) / kGemmBlockK;
    const uint32_t sms = context->sm_count > 0 ? static_cast<uint32_t>(context->sm_count) : 1u;
    uint32_t splitk = sms / row_block_tiles;
    splitk = splitk < 8u ? splitk : 8u;
    splitk = splitk < k_stages / 2u ? splitk : k_stages / 2u;
    const uint32_t batch_rows = (desc->max_batch + kGemmBlockM - 1) / kGemmBlockM * kGemmBlockM;
    uint32_t splitk_rows = sms / (2u * row_block_tiles) * kGemmBlockM;
    splitk_rows = splitk_rows < batch_rows ? splitk_rows : batch_rows;
    while (splitk_rows > kGemmBlockM &&
           static_cast<size_t>(splitk) * splitk_rows * count * sizeof(int32_t) > (size_t{64} << 20)) {
        splitk_rows -= kGemmBlockM;
    }
    const size_t splitk_bytes = static_cast<size_t>(splitk) * splitk_rows * count * sizeof(int32_t);
    if (error == cudaSuccess && splitk >= 2 && splitk_rows >= kGemmBlockM && desc->max_batch > kGemvMaxRows &&
        count % 4 == 0 && context->cc_major == 10 && context->cc_minor == 0) {
        error = cudaMalloc(reinterpret_cast<void **>(&linear->d_splitk), splitk_bytes);
        linear->splitk_max = splitk;
        linear->splitk_rows = splitk_rows;
    }
    if (error != cudaSuccess) {
        free_linear(linear);
        return cuda_fail(context, error, "allocate W8A8 plan", QPUCUDA_ALLOCATION_FAILED);
    }
    const cudaMemcpyKind kind = desc->memory == QPUCUDA_MEMORY_HOST ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToDevice;
    cudaStream_t stream = context->stream;
    error = cudaMemsetAsync(linear->d_weight, 0, weight_bytes, stream);
    if (error == cudaSuccess) error = cudaMemsetAsync(linear->d_quantized, 0, scratch_bytes, stream);
    if (error == cudaSuccess)
        error = cudaMemcpy2DAsync(linear->d_weight, linear->k_pad, desc->weight_values + start * desc->input_features,
                                  desc->input_features, desc->input_features, count, kind, stream);
    if (error == cudaSuccess)
        error = cudaMemcpyAsync(linear->d_weight_scales, desc->weight_scales + start, count * sizeof(float), kind, stream);
    if (error == cudaSuccess && linear->has_bias)
        error = cudaMemcpyAsync(linear->d_bias, desc->bias + start, count * sizeof(float), kind, stream);
    if (error != cudaSuccess) {
        free_linear(linear);
        return cuda_fail(context, error, "copy W8A8 weights", QPUCUDA_IO_FAILED);
    }
    const qpucuda_status waited = wait_stream(context);
    if (waited != QPUCUDA_OK) {
        free_linear(linear);
        return waited;
    }
    // Tensor maps for the resident weight and the activation scratch (sm_100 only).
    if (context->cc_major == 10 && context->cc_minor == 0) {
        linear->maps_ready =
            encode_tensor_map_2d_u8(&linear->map_weight, linear->d_weight, linear->k_pad, count, linear->k_pad,
                                    kGemmBlockK, kGemmWeightBoxRows) &&
            encode_tensor_map_2d_u8(&linear->map_quantized, linear->d_quantized, linear->k_pad, desc->max_batch,
                                    linear->k_pad, kGemmBlockK, kGemmBlockM);
    }
    linear->resident_bytes = weight_bytes + count * sizeof(float) * (linear->has_bias ? 2 : 1) + scratch_bytes +
                             desc->max_batch * sizeof(float) + (linear->d_splitk != nullptr ? splitk_bytes : 0);
    *result = linear;
    return QPUCUDA_OK;
}

void qpucuda_w8a8_linear_destroy(qpucuda_w8a8_linear *linear) {
    if (linear == nullptr) return;
    free_linear(linear);
}

size_t qpucuda_w8a8_linear_resident_bytes(const qpucuda_w8a8_linear *linear) {
    return linear != nullptr ? linear->resident_bytes : 0;
}

qpucuda_status qpucuda_w8a8_linear_execute_device(qpucuda_w8a8_linear *linear, const float *source,
                                                  size_t source_stride, uint32_t rows, float *destination,
                                                  size_t destination_stride) {
    if (linear == nullptr) return QPUCUDA_INVALID_ARGUMENT;
    qpucuda_context *context = linear->context;
    if (source == nullptr || destination == nullptr || rows == 0 || rows > linear->max_batch ||
        source_stride < linear->k || destination_stride < linear->columns) {
        return fail(context, QPUCUDA_INVALID_ARGUMENT, "prepared W8A8 linear source exceeds the plan shape");
    }
    if (rows > kGemvMaxRows && !(context->cc_major == 10 && context->cc_minor == 0)) {
        return fail(context, QPUCUDA_CAPABILITY_MISSING, "the tcgen05 int8 GEMM needs an sm_100 device");
    }
    std::lock_guard<std::mutex> lock(context->mutex);
    qpucuda_status status = begin_submit(context);
    if (status != QPUCUDA_OK) return status;
    DeviceGuard guard(context->device);
    return enqueue(linear, source, source_stride, nullptr, 0, nullptr, rows, destination, destination_stride);
}

qpucuda_status qpucuda_w8a8_linear_execute_device_fanout(qpucuda_w8a8_linear *linear, const float *source,
                                                         size_t source_stride, uint32_t rows, float *destination,
                                                         float *const *peer_destinations, uint32_t peer_count,
                                                         size_t destination_stride) {
    if (linear == nullptr) return QPUCUDA_INVALID_ARGUMENT;
    qpucuda_context *context = linear->context;
    if (source == nullptr || destination == nullptr || rows == 0 || rows > linear->max_batch ||
        source_stride < linear->k || destination_stride < linear->columns || peer_count > QPUCUDA_MAX_PEERS ||
        (peer_count != 0 && peer_destinations == nullptr)) {
        return fail(context, QPUCUDA_INVALID_ARGUMENT, "W8A8 fan-out: invalid arguments");
    }
    for (uint32_t p = 0; p < peer_count; ++p) {
        if (peer_destinations[p] == nullptr) return fail(context, QPUCUDA_INVALID_ARGUMENT, "W8A8 fan-out: null peer");
    }
    if (rows > kGemvMaxRows && !(context->cc_major == 10 && context->cc_minor == 0)) {
        return fail(context, QPUCUDA_CAPABILITY_MISSING, "the tcgen05 int8 GEMM needs an sm_100 device");
    }
    std::lock_guard<std::mutex> lock(context->mutex);
    qpucuda_status status = begin_submit(context);
    if (status != QPUCUDA_OK) return status;
    DeviceGuard guard(context->device);
    return enqueue_to(linear, source, source_stride, nullptr, 0, nullptr, rows, destination, destination_stride,
                      peer_destinations, peer_count);
}

qpucuda_status qpucuda_w8a8_linear_execute_device_layout(qpucuda_w8a8_linear *linear, const float *source,
                                                         const qpucuda_matrix_layout *source_layout, uint32_t rows,
                                                         float *destination,
                                                         const qpucuda_matrix_layout *destination_layout) {
    if (linear == nullptr) return QPUCUDA_INVALID_ARGUMENT;
    qpucuda_context *context = linear->context;
    if (source == nullptr || destination == nullptr || source_layout == nullptr || destination_layout == nullptr ||
        rows == 0 || rows > linear->max_batch || source_layout->column_stride == 0 ||
        destination_layout->column_stride == 0) {
        return fail(context, QPUCUDA_INVALID_ARGUMENT, "W8A8 layout execute: invalid arguments");
    }
    // A layout whose rows would overlap (e.g. row-major with a row stride shorter than the row)
    // is rejected; batches are taken as given.
    if ((source_layout->column_stride == 1 && source_layout->row_stride < linear->k &&
         (source_layout->rows_per_batch == 0 || source_layout->rows_per_batch > 1)) ||
        (destination_layout->column_stride == 1 && destination_layout->row_stride < linear->columns &&
         (destination_layout->rows_per_batch == 0 || destination_layout->rows_per_batch > 1))) {
        return fail(context, QPUCUDA_INVALID_ARGUMENT, "W8A8 layout execute: rows overlap");
    }
    if (!(context->cc_major == 10 && context->cc_minor == 0)) {
        return fail(context, QPUCUDA_CAPABILITY_MISSING, "the tcgen05 int8 GEMM needs an sm_100 device");
    }
    auto batch_rows = [rows](uint64_t value) {
        return value == 0 || value >= rows ? 0xFFFFFFFFu : static_cast<uint32_t>(value);
    };
    std::lock_guard<std::mutex> lock(context->mutex);
    qpucuda_status status = begin_submit(context);
    if (status != QPUCUDA_OK) return status;
    DeviceGuard guard(context->device);
    cudaStream_t stream = context->stream;
    const uint32_t source_rows_per_batch = batch_rows(source_layout->rows_per_batch);
    cudaError_t error = launch_quantize_rows_int8_layout(
        source, rows, linear->k, linear->k_pad, source_rows_per_batch == 0xFFFFFFFFu ? rows : source_rows_per_batch,
        source_layout->batch_stride, source_layout->row_stride, source_layout->column_stride, linear->d_quantized,
        linear->k_pad, linear->d_row_scales, stream);
    if (error != cudaSuccess) return cuda_fail(context, error, "quantize activations");
    GemmEpilogue epilogue;
    epilogue.mode = linear->has_bias ? EpilogueMode::kDequantizeBias : EpilogueMode::kDequantize;
    epilogue.row_scales = linear->d_row_scales;
    epilogue.col_scales = linear->d_weight_scales;
    epilogue.bias = linear->d_bias;
    epilogue.out = destination;
    epilogue.out_stride = destination_layout->row_stride;
    epilogue.rows_per_batch = batch_rows(destination_layout->rows_per_batch);
    epilogue.batch_stride = destination_layout->batch_stride;
    epilogue.col_stride = destination_layout->column_stride;
    error = linear->maps_ready
                ? launch_w8a8_gemm_sm100(&linear->map_quantized, &linear->map_weight, rows, linear->columns,
                                         linear->k_pad, epilogue, context->d_error, context->sm_count, stream)
                : run_w8a8_gemm(linear->d_quantized, linear->k_pad, linear->d_weight, linear->k_pad, rows,
                                linear->columns, linear->k_pad, epilogue, context->d_error, context->sm_count, stream);
    if (error == cudaErrorInvalidValue) return cuda_fail(context, error, "W8A8 GEMM launch", QPUCUDA_INVALID_ARGUMENT);
    if (error != cudaSuccess) return cuda_fail(context, error, "W8A8 GEMM launch");
    return QPUCUDA_OK;
}

qpucuda_status qpucuda_w8a8_linear_execute_prepared_device(qpucuda_w8a8_linear *linear, const int8_t *quantized,
                                                           size_t quantized_stride, const float *row_scales,
                                                           uint32_t rows, float *destination,
                                                           size_t destination_stride) {
    if (linear == nullptr) return QPUCUDA_INVALID_ARGUMENT;
    qpucuda_context *context = linear->context;
    if (quantized == nullptr || row_scales == nullptr || destination == nullptr || rows == 0 ||
        rows > linear->max_batch || quantized_stride < linear->k_pad || quantized_stride % 16 != 0 ||
        (reinterpret_cast<uintptr_t>(quantized) & 15u) != 0 || destination_stride < linear->columns) {
        return fail(context, QPUCUDA_INVALID_ARGUMENT,
                    "prepared W8A8 linear: quantized rows need a 16-byte aligned stride >= the padded K");
    }
    if (rows > kGemvMaxRows && !(context->cc_major == 10 && context->cc_minor == 0)) {
        return fail(context, QPUCUDA_CAPABILITY_MISSING, "the tcgen05 int8 GEMM needs an sm_100 device");
    }
    std::lock_guard<std::mutex> lock(context->mutex);
    qpucuda_status status = begin_submit(context);
    if (status != QPUCUDA_OK) return status;
    DeviceGuard guard(context->device);
    return enqueue(linear, nullptr, 0, quantized, quantized_stride, row_scales, rows, destination, destination_stride);
}

}  // extern "C"

namespace {

bool page_locked(const void *pointer) {
    cudaPointerAttributes attributes;
    if (cudaPointerGetAttributes(&attributes, pointer) != cudaSuccess) {
        (void)cudaGetLastError();
        return false;
    }
    return attributes.type == cudaMemoryTypeHost;
}

// Host-buffer execution. Staged (direct == false): results land in plan-owned pinned staging and
// reach the caller's destination only after a successful wait. Direct: the destination is the
// caller's page-locked memory and the device-to-host copies write it in place.
qpucuda_status execute_host(qpucuda_w8a8_linear *linear, const qpucuda_w8a8_execution *execution, bool direct) {
    if (linear == nullptr || execution == nullptr) return QPUCUDA_INVALID_ARGUMENT;
    qpucuda_context *context = linear->context;
    const uint32_t rows = execution->rows;
    size_t source_bytes = 0, destination_bytes = 0;
    if (execution->source == nullptr || execution->destination == nullptr || rows == 0 || rows > linear->max_batch ||
        !multiply_size(static_cast<size_t>(rows) * linear->k, sizeof(float), &source_bytes) ||
        !multiply_size(static_cast<size_t>(rows) * linear->columns, sizeof(float), &destination_bytes) ||
        execution->source_size < source_bytes || execution->destination_size < destination_bytes) {
        return fail(context, QPUCUDA_INVALID_ARGUMENT, "prepared W8A8 linear source exceeds the plan shape");
    }
    if (rows > kGemvMaxRows && !(context->cc_major == 10 && context->cc_minor == 0)) {
        return fail(context, QPUCUDA_CAPABILITY_MISSING, "the tcgen05 int8 GEMM needs an sm_100 device");
    }
    if (direct && (!page_locked(execution->destination) ||
                   !page_locked(reinterpret_cast<const char *>(execution->destination) + destination_bytes - 1))) {
        return fail(context, QPUCUDA_INVALID_ARGUMENT,
                    "direct W8A8 execution needs a page-locked destination (cudaMallocHost or cudaHostRegister)");
    }
    {
        std::lock_guard<std::mutex> guard(linear->mutex);
        if (linear->busy) {
            return fail(context, QPUCUDA_INTERNAL_ERROR,
                        "prepared W8A8 linear plan already has an in-flight invocation");
        }
        linear->busy = true;
    }
    std::lock_guard<std::mutex> lock(context->mutex);
    DeviceGuard device_guard(context->device);
    auto release = [linear](qpucuda_status status) {
        std::lock_guard<std::mutex> guard(linear->mutex);
        linear->busy = false;
        return status;
    };
    qpucuda_status status = begin_submit(context);
    if (status != QPUCUDA_OK) return release(status);
    const size_t max_source = static_cast<size_t>(linear->max_batch) * linear->k * sizeof(float);
    const size_t max_destination = static_cast<size_t>(linear->max_batch) * linear->columns * sizeof(float);
    if (linear->d_source == nullptr) {
        if ((context->failure_mask & QPUCUDA_FAIL_ALLOCATION) != 0 ||
            cudaMallocHost(reinterpret_cast<void **>(&linear->h_destination), max_destination) != cudaSuccess ||
            cudaMalloc(reinterpret_cast<void **>(&linear->d_source), max_source) != cudaSuccess ||
            cudaMalloc(reinterpret_cast<void **>(&linear->d_destination), max_destination) != cudaSuccess) {
            (void)cudaGetLastError();
            cudaFreeHost(linear->h_destination);
            cudaFree(linear->d_source);
            cudaFree(linear->d_destination);
            linear->h_destination = nullptr;
            linear->d_source = linear->d_destination = nullptr;
            return release(fail(context, QPUCUDA_ALLOCATION_FAILED, "allocate W8A8 host staging"));
        }
    }
    // The source is copied straight from the caller's buffer (a DMA when it is pinned). The
    // result lands in plan-owned pinned staging first and reaches the caller only after a
    // successful wait, so a failed or timed-out wait never writes the caller's destination.
    // Batches above kSliceRows rows are pipelined in row slices: host-to-device copies on one
    // stream, quantize + GEMM on the context stream and device-to-host copies on another, so
    // the two PCIe directions overlap each other and the compute.
    const uint32_t slices = rows > kSliceRows ? (rows + kSliceRows - 1) / kSliceRows : 1;
    if (slices > 1 && !ensure_pipeline(linear, slices)) {
        return release(fail(context, QPUCUDA_ALLOCATION_FAILED, "create W8A8 copy streams"));
    }
    float *host_out = direct ? execution->destination : linear->h_destination;
    cudaError_t error = cudaSuccess;
    if (slices == 1) {
        error = cudaMemcpyAsync(linear->d_source, execution->source, source_bytes, cudaMemcpyHostToDevice,
                                context->stream);
        if (error != cudaSuccess) return release(cuda_fail(context, error, "copy W8A8 source"));
        status = enqueue(linear, linear->d_source, linear->k, nullptr, 0, nullptr, rows, linear->d_destination,
                         linear->columns);
        if (status != QPUCUDA_OK) return release(status);
        error = cudaMemcpyAsync(host_out, linear->d_destination, destination_bytes, cudaMemcpyDeviceToHost,
                                context->stream);
        if (error != cudaSuccess) return release(cuda_fail(context, error, "copy W8A8 destination"));
    } else {
        status = enqueue_sliced(linear, static_cast<const float *>(execution->source), rows, slices, host_out);
        if (status != QPUCUDA_OK) {
            (void)wait_stream(context);  // drain whatever was issued before the failure (bounded)
            drain_copies(linear);
            return release(status);
        }
    }
    status = wait_stream(context);
    if (status == QPUCUDA_OK) {
        if (!direct) parallel_memcpy(execution->destination, linear->h_destination, destination_bytes);
    } else if (slices > 1) {
        drain_copies(linear);
    }
    return release(status);
}

}  // namespace

extern "C" {

struct qpucuda_w8a8_submission {
    qpucuda_w8a8_linear *linear = nullptr;
    cudaEvent_t done = nullptr;  // the plan's completion event of this submission
    uint32_t slices = 1;
    bool waited = false;
    qpucuda_status status = QPUCUDA_OK;
};

qpucuda_status qpucuda_w8a8_linear_submit_direct(qpucuda_w8a8_linear *linear, const qpucuda_w8a8_execution *execution,
                                                 qpucuda_w8a8_submission **submission) {
    if (linear == nullptr || execution == nullptr || submission == nullptr) return QPUCUDA_INVALID_ARGUMENT;
    *submission = nullptr;
    qpucuda_context *context = linear->context;
    const uint32_t rows = execution->rows;
    size_t source_bytes = 0, destination_bytes = 0;
    if (execution->source == nullptr || execution->destination == nullptr || rows == 0 || rows > linear->max_batch ||
        !multiply_size(static_cast<size_t>(rows) * linear->k, sizeof(float), &source_bytes) ||
        !multiply_size(static_cast<size_t>(rows) * linear->columns, sizeof(float), &destination_bytes) ||
        execution->source_size < source_bytes || execution->destination_size < destination_bytes) {
        return fail(context, QPUCUDA_INVALID_ARGUMENT, "prepared W8A8 linear source exceeds the plan shape");
    }
    if (rows > kGemvMaxRows && !(context->cc_major == 10 && context->cc_minor == 0)) {
        return fail(context, QPUCUDA_CAPABILITY_MISSING, "the tcgen05 int8 GEMM needs an sm_100 device");
    }
    if (!page_locked(execution->destination) ||
        !page_locked(reinterpret_cast<const char *>(execution->destination) + destination_bytes - 1)) {
        return fail(context, QPUCUDA_INVALID_ARGUMENT,
                    "a W8A8 submission needs a page-locked destination (cudaMallocHost or cudaHostRegister)");
    }
    qpucuda_w8a8_submission *handle = new (std::nothrow) qpucuda_w8a8_submission();
    if (handle == nullptr) return QPUCUDA_ALLOCATION_FAILED;
    {
        std::lock_guard<std::mutex> guard(linear->mutex);
        if (linear->busy) {
            delete handle;
            return fail(context, QPUCUDA_INTERNAL_ERROR, "prepared W8A8 linear plan already has an in-flight invocation");
        }
        linear->busy = true;
    }
    std::lock_guard<std::mutex> lock(context->mutex);
    DeviceGuard device_guard(context->device);
    auto release = [linear, handle](qpucuda_status status) {
        std::lock_guard<std::mutex> guard(linear->mutex);
        linear->busy = false;
        delete handle;
        return status;
    };
    qpucuda_status status = begin_submit(context);
    if (status != QPUCUDA_OK) return release(status);
    const size_t max_source = static_cast<size_t>(linear->max_batch) * linear->k * sizeof(float);
    const size_t max_destination = static_cast<size_t>(linear->max_batch) * linear->columns * sizeof(float);
    if (linear->d_source == nullptr) {
        if ((context->failure_mask & QPUCUDA_FAIL_ALLOCATION) != 0 ||
            cudaMalloc(reinterpret_cast<void **>(&linear->d_source), max_source) != cudaSuccess ||
            cudaMalloc(reinterpret_cast<void **>(&linear->d_destination), max_destination) != cudaSuccess) {
            (void)cudaGetLastError();
            cudaFree(linear->d_source);
            cudaFree(linear->d_destination);
            linear->d_source = linear->d_destination = nullptr;
            return release(fail(context, QPUCUDA_ALLOCATION_FAILED, "allocate W8A8 device staging"));
        }
    }
    if (linear->h_submit_error == nullptr &&
        cudaMallocHost(reinterpret_cast<void **>(&linear->h_submit_error), sizeof(unsigned int)) != cudaSuccess) {
        (void)cudaGetLastError();
        linear->h_submit_error = nullptr;
        return release(fail(context, QPUCUDA_ALLOCATION_FAILED, "allocate W8A8 submission error word"));
    }
    const uint32_t slices = rows > kSliceRows ? (rows + kSliceRows - 1) / kSliceRows : 1;
    if (!ensure_pipeline(linear, slices)) {
        return release(fail(context, QPUCUDA_ALLOCATION_FAILED, "create W8A8 copy streams"));
    }
    float *host_out = execution->destination;
    cudaError_t error = cudaSuccess;
    if (slices == 1) {
        error = cudaMemcpyAsync(linear->d_source, execution->source, source_bytes, cudaMemcpyHostToDevice, context->stream);
        if (error != cudaSuccess) return release(cuda_fail(context, error, "copy W8A8 source"));
        status = enqueue(linear, linear->d_source, linear->k, nullptr, 0, nullptr, rows, linear->d_destination,
                         linear->columns);
        if (status != QPUCUDA_OK) return release(status);
        error = cudaMemcpyAsync(host_out, linear->d_destination, destination_bytes, cudaMemcpyDeviceToHost,
                                context->stream);
        if (error == cudaSuccess)
            error = cudaMemcpyAsync(linear->h_submit_error, context->d_error, sizeof(unsigned int),
                                    cudaMemcpyDeviceToHost, context->stream);
        handle->done = linear->events[2 * slices + 2];
        if (error == cudaSuccess) error = cudaEventRecord(handle->done, context->stream);
        if (error != cudaSuccess) return release(cuda_fail(context, error, "copy W8A8 destination"));
    } else {
        // The device-to-host copies stay on the plan's copy stream: the next submission's
        // host-to-device copies and kernels do not wait for them.
        status = enqueue_sliced(linear, static_cast<const float *>(execution->source), rows, slices, host_out, false);
        if (status == QPUCUDA_OK) {
            cudaEvent_t computed = linear->events[1 + 2 * slices];
            handle->done = linear->events[2 * slices + 2];
            error = cudaMemcpyAsync(linear->h_submit_error, context->d_error, sizeof(unsigned int),
                                    cudaMemcpyDeviceToHost, context->stream);
            if (error == cudaSuccess) error = cudaEventRecord(computed, context->stream);
            if (error == cudaSuccess) error = cudaStreamWaitEvent(linear->copy_out, computed, 0);
            if (error == cudaSuccess) error = cudaEventRecord(handle->done, linear->copy_out);
            if (error != cudaSuccess) status = cuda_fail(context, error, "record W8A8 submission");
        }
        if (status != QPUCUDA_OK) {
            (void)wait_stream(context);  // drain whatever was issued before the failure (bounded)
            drain_copies(linear);
            return release(status);
        }
    }
    handle->linear = linear;
    handle->slices = slices;
    *submission = handle;
    return QPUCUDA_OK;
}

qpucuda_status qpucuda_w8a8_submission_wait(qpucuda_w8a8_submission *submission) {
    if (submission == nullptr) return QPUCUDA_INVALID_ARGUMENT;
    if (submission->waited) return submission->status;
    qpucuda_w8a8_linear *linear = submission->linear;
    qpucuda_context *context = linear->context;
    DeviceGuard device_guard(context->device);
    qpucuda_status status = QPUCUDA_OK;
    const uint64_t start = monotonic_ns();
    uint64_t polls = 0;
    for (;;) {
        const cudaError_t error = cudaEventQuery(submission->done);
        if (error == cudaSuccess) break;
        if (error != cudaErrorNotReady) {
            std::lock_guard<std::mutex> lock(context->mutex);
            context->poisoned = true;
            status = cuda_fail(context, error, "wait for a W8A8 submission", QPUCUDA_IO_FAILED);
            break;
        }
        if (monotonic_ns() - start > context->timeout_ns) {
            std::lock_guard<std::mutex> lock(context->mutex);
            context->poisoned = true;
            status = fail(context, QPUCUDA_TIMEOUT, "W8A8 submission did not complete within %llu ns",
                          static_cast<unsigned long long>(context->timeout_ns));
            break;
        }
        if (++polls > 2000) std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
    if (status == QPUCUDA_OK && (context->failure_mask & QPUCUDA_FAIL_WAIT) != 0) {
        std::lock_guard<std::mutex> lock(context->mutex);
        context->poisoned = true;
        status = fail(context, QPUCUDA_TIMEOUT, "injected wait timeout");
    }
    if (status == QPUCUDA_OK && *linear->h_submit_error != kKernelOk) {
        std::lock_guard<std::mutex> lock(context->mutex);
        context->poisoned = true;
        status = fail(context, QPUCUDA_TIMEOUT, "a kernel barrier wait exceeded its bound (code %u)", *linear->h_submit_error);
    }
    if (status != QPUCUDA_OK && submission->slices > 1) drain_copies(linear);
    {
        std::lock_guard<std::mutex> guard(linear->mutex);
        linear->busy = false;
    }
    submission->waited = true;
    submission->status = status;
    return status;
}

void qpucuda_w8a8_submission_destroy(qpucuda_w8a8_submission *submission) {
    if (submission == nullptr) return;
    if (!submission->waited) (void)qpucuda_w8a8_submission_wait(submission);
    delete submission;
}

qpucuda_status qpucuda_w8a8_linear_execute(qpucuda_w8a8_linear *linear, const qpucuda_w8a8_execution *execution) {
    return execute_host(linear, execution, false);
}

qpucuda_status qpucuda_w8a8_linear_execute_direct(qpucuda_w8a8_linear *linear,
                                                  const qpucuda_w8a8_execution *execution) {
    return execute_host(linear, execution, true);
}

qpucuda_status qpucuda_w8a8_linear_scratch(const qpucuda_w8a8_linear *linear, const int8_t **quantized,
                                           size_t *quantized_stride, const float **row_scales) {
    if (linear == nullptr || quantized == nullptr || quantized_stride == nullptr || row_scales == nullptr) {
        return QPUCUDA_INVALID_ARGUMENT;
    }
    *quantized = linear->d_quantized;
    *quantized_stride = linear->k_pad;
    *row_scales = linear->d_row_scales;
    return QPUCUDA_OK;
}

}  // extern "C"
