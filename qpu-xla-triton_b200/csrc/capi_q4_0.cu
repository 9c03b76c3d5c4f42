// Prepared GGML Q4_0 x Q8_0 linear (include/qpucuda_q4_0.h), the CUDA drop-in
// for integrations/llama_cpp/src/qpu_llama_q4_0.c: same argument rules
// (prepare :205-225, submit :465-495), the same busy flag (:504-511), the same
// column-window copy-out after the wait (:795-806) and the same status codes.
#include <cstdlib>
#include <cstring>
#include <new>

#include "qpucuda_internal.h"
#include "qpucuda_q4_0.h"

#ifndef QPUCUDA_Q4_0_SOURCE_HASH
#define QPUCUDA_Q4_0_SOURCE_HASH "unversioned"
#endif

using namespace qpucuda;

namespace {
constexpr uint32_t kBlockElements = 32;
constexpr uint32_t kWeightBlockBytes = 18;
constexpr uint32_t kActivationBlockBytes = 34;
constexpr uint32_t kOutputTile = 16;
constexpr uint32_t kMaxRows = 4;
}  // namespace

struct qpucuda_q4_0_linear {
    qpucuda_context *context = nullptr;
    uint32_t blocks = 0;
    uint32_t output_columns = 0;
    uint32_t rows = 0;
    uint32_t resident_column_start = 0;
    uint32_t resident_column_count = 0;
    uint8_t *d_nibbles = nullptr;     // [resident][blocks][16]
    uint16_t *d_scales = nullptr;     // [resident][scale_stride], zero padded
    uint8_t *d_activation = nullptr;  // [rows][blocks][34] staging
    uint8_t *d_mx = nullptr;          // rows > 4: split activation for the tensor-core path
    int8_t *d_mx_values = nullptr;    // rows > 4: codes as int8 (code - 8), [resident][blocks_pad * 32]
    float *d_mx_scales_t = nullptr;   // rows > 4: fp32 scales, [blocks_pad][resident]
    float *d_output = nullptr;        // [rows][resident] staging
    uint8_t *h_activation = nullptr;  // pinned
    float *h_output = nullptr;        // pinned
    size_t resident_bytes = 0;
    bool busy = false;
    std::mutex mutex;
};

struct qpucuda_q4_0_submission {
    qpucuda_q4_0_linear *linear = nullptr;
    uint8_t *destination = nullptr;
    size_t destination_offset = 0;
    uint32_t rows = 0;
    uint32_t column_start = 0;
    uint32_t column_count = 0;
    uint64_t complete_start = 0;
    uint64_t input_access_end = 0;
    uint64_t input_pack_end = 0;
    uint64_t input_copy_end = 0;
    uint64_t submit_start = 0;
    uint64_t submit_end = 0;
    bool active = false;
};

namespace {

void free_linear(qpucuda_q4_0_linear *linear) {
    DeviceGuard guard(linear->context->device);
    cudaFree(linear->d_nibbles);
    cudaFree(linear->d_scales);
    cudaFree(linear->d_activation);
    cudaFree(linear->d_mx);
    cudaFree(linear->d_mx_values);
    cudaFree(linear->d_mx_scales_t);
    cudaFree(linear->d_output);
    cudaFreeHost(linear->h_activation);
    cudaFreeHost(linear->h_output);
    (void)cudaGetLastError();
    delete linear;
}

void release(qpucuda_q4_0_linear *linear) {
    std::lock_guard<std::mutex> guard(linear->mutex);
    linear->busy = false;
}

Q40Weights weights_of(const qpucuda_q4_0_linear *linear) {
    Q40Weights weights;
    weights.nibbles = linear->d_nibbles;
    weights.scales = linear->d_scales;
    weights.columns = linear->resident_column_count;
    weights.blocks = linear->blocks;
    weights.scale_stride = q4_0_scale_stride(linear->blocks);
    weights.mx_values = linear->d_mx_values;
    weights.mx_scales_t = linear->d_mx_scales_t;
    return weights;
}

// rows <= 4: the decode matvec over Q8_0 blocks (or fp32 rows); more rows: the tiled
// tensor-core path through the plan's split-activation scratch.
cudaError_t launch_linear(const qpucuda_q4_0_linear *linear, const uint8_t *q8_0, const float *f32, size_t f32_stride,
                          uint32_t rows, uint32_t interleave, float *destination, size_t destination_stride,
                          uint32_t local_start, uint32_t output_column_start, uint32_t column_count) {
    qpucuda_context *context = linear->context;
    if (rows > kMaxRows) {
        return launch_q4_0_mx(weights_of(linear), q8_0, f32, f32_stride, rows, interleave, linear->d_mx, destination,
                              destination_stride, local_start, output_column_start, column_count, context->d_error,
                              context->sm_count, context->stream);
    }
    if (f32 != nullptr) {
        return launch_q4_0_f32_gemv(weights_of(linear), f32, f32_stride, rows, destination, destination_stride,
                                    local_start, output_column_start, column_count, context->sm_count, context->stream);
    }
    return launch_q4_0_q8_0_gemv(weights_of(linear), q8_0, rows, interleave, destination, destination_stride,
                                 local_start, output_column_start, column_count, context->d_error, context->sm_count,
                                 context->stream);
}

bool window_ok(const qpucuda_q4_0_linear *linear, uint32_t column_start, uint32_t column_count) {
    return column_count != 0 && column_start % kOutputTile == 0 && column_count % kOutputTile == 0 &&
           column_start >= linear->resident_column_start && column_count <= linear->resident_column_count &&
           column_start - linear->resident_column_start <= linear->resident_column_count - column_count;
}

}  // namespace

extern "C" {

const char *qpucuda_q4_0_kernel_source_hash(void) { return QPUCUDA_Q4_0_SOURCE_HASH; }

qpucuda_status qpucuda_q4_0_linear_prepare(qpucuda_context *context, const qpucuda_q4_0_linear_desc *desc,
                                           qpucuda_q4_0_linear **result) {
    if (result != nullptr) *result = nullptr;
    // Argument rules of qpu_llama_q4_0_linear_prepare (qpu_llama_q4_0.c:205-225).
    if (context == nullptr || desc == nullptr || result == nullptr || desc->weights == nullptr ||
        desc->expected_source_hash == nullptr || desc->rows == 0 || desc->rows > 4u * UINT16_MAX ||
        desc->input_columns == 0 || desc->input_columns % kBlockElements != 0 || desc->output_columns == 0 ||
        desc->resident_column_count == 0 || desc->resident_column_start % kOutputTile != 0 ||
        desc->resident_column_count % kOutputTile != 0 ||
        (desc->weight_mode != QPUCUDA_Q4_0_WEIGHT_EXACT && desc->weight_mode != QPUCUDA_Q4_0_WEIGHT_COLUMN_W8 &&
         desc->weight_mode != QPUCUDA_Q4_0_WEIGHT_ROWCOL_W8A8) ||
        (desc->weight_mode != QPUCUDA_Q4_0_WEIGHT_EXACT && desc->rows <= 4u) ||
        desc->resident_column_start > desc->output_columns ||
        desc->resident_column_count > desc->output_columns - desc->resident_column_start) {
        return QPUCUDA_INVALID_ARGUMENT;
    }
    *result = nullptr;
    if (desc->weight_mode != QPUCUDA_Q4_0_WEIGHT_EXACT) {
        return fail(context, QPUCUDA_CAPABILITY_MISSING,
                    "Q4_0 linear: only the exact weight mode is implemented (no re-quantized W8 modes)");
    }
    const size_t blocks = desc->input_columns / kBlockElements;
    size_t weight_row_bytes = 0, required_source_bytes = 0;
    if (!multiply_size(blocks, kWeightBlockBytes, &weight_row_bytes) ||
        !multiply_size(desc->output_columns, weight_row_bytes, &required_source_bytes) ||
        desc->weight_size < required_source_bytes) {
        return QPUCUDA_INVALID_ARGUMENT;
    }
    if ((context->failure_mask & QPUCUDA_FAIL_SOURCE_HASH) != 0) {
        return fail(context, QPUCUDA_HASH_MISMATCH, "injected source hash mismatch");
    }
    if (std::strcmp(desc->expected_source_hash, QPUCUDA_Q4_0_SOURCE_HASH) != 0) {
        return fail(context, QPUCUDA_HASH_MISMATCH, "Q4_0 kernel source hash does not match the expected hash");
    }
    std::lock_guard<std::mutex> lock(context->mutex);
    if (context->poisoned) return fail(context, QPUCUDA_IO_FAILED, "CUDA context is poisoned after a wait failure");
    if ((context->failure_mask & QPUCUDA_FAIL_ALLOCATION) != 0) {
        return fail(context, QPUCUDA_ALLOCATION_FAILED, "injected device allocation failure");
    }
    qpucuda_q4_0_linear *linear = new (std::nothrow) qpucuda_q4_0_linear();
    if (linear == nullptr) return QPUCUDA_ALLOCATION_FAILED;
    linear->context = context;
    linear->blocks = static_cast<uint32_t>(blocks);
    linear->output_columns = desc->output_columns;
    linear->rows = desc->rows;
    linear->resident_column_start = desc->resident_column_start;
    linear->resident_column_count = desc->resident_column_count;
    DeviceGuard guard(context->device);
    const size_t resident_blocks = static_cast<size_t>(desc->resident_column_count) * blocks;
    const size_t scale_bytes = static_cast<size_t>(desc->resident_column_count) * q4_0_scale_stride(linear->blocks) * 2;
    const size_t native_bytes = resident_blocks * kWeightBlockBytes;
    const size_t activation_bytes = static_cast<size_t>(desc->rows) * blocks * kActivationBlockBytes;
    const size_t output_bytes = static_cast<size_t>(desc->rows) * desc->resident_column_count * sizeof(float);
    const size_t mx_bytes = desc->rows > kMaxRows ? q4_0_mx_scratch_bytes(desc->rows, linear->blocks) : 0;
    // Rows > 4 on sm_100: the tcgen05 MX kernel reads the codes expanded to int8 and the scales as
    // fp32, block-major (made once here from the repacked weights), when a call of the plan's rows
    // over its resident columns would give it a wave of tiles.
    const bool mx_tcgen05 = mx_bytes != 0 && context->cc_major == 10 && context->cc_minor == 0 &&
                            q4_0_mx_sm100_fills_wave(desc->rows, desc->resident_column_count, context->sm_count);
    const size_t mx_blocks_pad = q4_0_mx_blocks_pad(linear->blocks);
    const size_t mx_value_bytes = mx_tcgen05 ? static_cast<size_t>(desc->resident_column_count) * mx_blocks_pad * 32 : 0;
    const size_t mx_scale_bytes = mx_tcgen05 ? static_cast<size_t>(desc->resident_column_count) * mx_blocks_pad * 4 : 0;
    uint8_t *d_native = nullptr;
    cudaError_t error = cudaMalloc(reinterpret_cast<void **>(&linear->d_nibbles), resident_blocks * 16);
    if (error == cudaSuccess) error = cudaMalloc(reinterpret_cast<void **>(&linear->d_scales), scale_bytes);
    if (error == cudaSuccess) error = cudaMalloc(reinterpret_cast<void **>(&linear->d_activation), activation_bytes);
    if (error == cudaSuccess) error = cudaMalloc(reinterpret_cast<void **>(&linear->d_output), output_bytes);
    if (error == cudaSuccess && mx_bytes != 0) error = cudaMalloc(reinterpret_cast<void **>(&linear->d_mx), mx_bytes);
    if (error == cudaSuccess && mx_tcgen05)
        error = cudaMalloc(reinterpret_cast<void **>(&linear->d_mx_values), mx_value_bytes);
    if (error == cudaSuccess && mx_tcgen05)
        error = cudaMalloc(reinterpret_cast<void **>(&linear->d_mx_scales_t), mx_scale_bytes);
    if (error == cudaSuccess) error = cudaMallocHost(reinterpret_cast<void **>(&linear->h_activation), activation_bytes);
    if (error == cudaSuccess) error = cudaMallocHost(reinterpret_cast<void **>(&linear->h_output), output_bytes);
    if (error == cudaSuccess) error = cudaMalloc(reinterpret_cast<void **>(&d_native), native_bytes);
    if (error != cudaSuccess) {
        cudaFree(d_native);
        free_linear(linear);
        return cuda_fail(context, error, "allocate Q4_0 plan", QPUCUDA_ALLOCATION_FAILED);
    }
    // The weights pointer is only read here (copied, then repacked on the device), qpu_llama_q4_0.c:327-391.
    const uint8_t *source = static_cast<const uint8_t *>(desc->weights) +
                            static_cast<size_t>(desc->resident_column_start) * weight_row_bytes;
    error = cudaMemcpyAsync(d_native, source, native_bytes, cudaMemcpyHostToDevice, context->stream);
    if (error == cudaSuccess) error = cudaMemsetAsync(linear->d_scales, 0, scale_bytes, context->stream);
    if (error == cudaSuccess)
        error = launch_q4_0_repack(d_native, desc->resident_column_count, linear->blocks,
                                   q4_0_scale_stride(linear->blocks), linear->d_nibbles, linear->d_scales,
                                   context->stream);
    if (error == cudaSuccess && mx_tcgen05)
        error = launch_q4_0_mx_expand(linear->d_nibbles, linear->d_scales, desc->resident_column_count, linear->blocks,
                                      static_cast<uint32_t>(mx_blocks_pad), q4_0_scale_stride(linear->blocks),
                                      linear->d_mx_values, linear->d_mx_scales_t, context->stream);
    qpucuda_status status = error == cudaSuccess ? wait_stream(context)
                                                 : cuda_fail(context, error, "stage Q4_0 weights", QPUCUDA_IO_FAILED);
    cudaFree(d_native);
    if (status != QPUCUDA_OK) {
        free_linear(linear);
        return status;
    }
    linear->resident_bytes =
        resident_blocks * kWeightBlockBytes + activation_bytes + output_bytes + mx_bytes + mx_value_bytes + mx_scale_bytes;
    *result = linear;
    return QPUCUDA_OK;
}

void qpucuda_q4_0_linear_destroy(qpucuda_q4_0_linear *linear) {
    if (linear == nullptr) return;
    free_linear(linear);
}

size_t qpucuda_q4_0_linear_resident_bytes(const qpucuda_q4_0_linear *linear) {
    return linear != nullptr ? linear->resident_bytes : 0;
}

qpucuda_status qpucuda_q4_0_linear_submit(qpucuda_q4_0_linear *linear, const qpucuda_q4_0_execution *execution,
                                          qpucuda_q4_0_submission **result) {
    const uint32_t rows = execution != nullptr && execution->rows != 0 ? execution->rows
                                                                       : (linear != nullptr ? linear->rows : 0);
    // Argument rules of qpu_llama_q4_0_linear_submit (qpu_llama_q4_0.c:465-495).
    if (linear == nullptr || execution == nullptr || result == nullptr || execution->activation == nullptr ||
        execution->destination == nullptr || rows == 0 || rows > linear->rows ||
        !window_ok(linear, execution->column_start, execution->column_count)) {
        return QPUCUDA_INVALID_ARGUMENT;
    }
    if (execution->activation_interleave != 0 && execution->activation_interleave != 4 &&
        execution->activation_interleave != 8) {
        return QPUCUDA_INVALID_ARGUMENT;
    }
    *result = nullptr;
    size_t activation_row_bytes = 0, activation_bytes = 0, destination_elements = 0, destination_bytes = 0;
    if (!multiply_size(linear->blocks, kActivationBlockBytes, &activation_row_bytes) ||
        !multiply_size(rows, activation_row_bytes, &activation_bytes) ||
        !multiply_size(rows, linear->output_columns, &destination_elements) ||
        !multiply_size(destination_elements, sizeof(float), &destination_bytes) ||
        !valid_range(execution->activation_size, execution->activation_offset, activation_bytes) ||
        !valid_range(execution->destination_size, execution->destination_offset, destination_bytes)) {
        return QPUCUDA_INVALID_ARGUMENT;
    }
    qpucuda_q4_0_submission *submission = new (std::nothrow) qpucuda_q4_0_submission();
    if (submission == nullptr) return QPUCUDA_ALLOCATION_FAILED;
    {
        std::lock_guard<std::mutex> guard(linear->mutex);
        if (linear->busy) {
            delete submission;
            return QPUCUDA_INTERNAL_ERROR;
        }
        linear->busy = true;
    }
    qpucuda_context *context = linear->context;
    std::lock_guard<std::mutex> lock(context->mutex);
    DeviceGuard guard(context->device);
    submission->complete_start = monotonic_ns();
    submission->input_access_end = submission->complete_start;
    const uint8_t *source = static_cast<const uint8_t *>(execution->activation) + execution->activation_offset;
    std::memcpy(linear->h_activation, source, activation_bytes);
    submission->input_pack_end = monotonic_ns();
    qpucuda_status status = begin_submit(context);
    cudaError_t error = cudaSuccess;
    if (status == QPUCUDA_OK) {
        error = cudaMemcpyAsync(linear->d_activation, linear->h_activation, activation_bytes, cudaMemcpyHostToDevice,
                                context->stream);
        submission->input_copy_end = monotonic_ns();
        submission->submit_start = submission->input_copy_end;
        const uint32_t local_start = execution->column_start - linear->resident_column_start;
        if (error == cudaSuccess) {
            error = launch_linear(linear, linear->d_activation, nullptr, 0, rows, execution->activation_interleave,
                                  linear->d_output, linear->resident_column_count, local_start, local_start,
                                  execution->column_count);
        }
        if (error == cudaSuccess) {
            // Only the requested window crosses back to the host.
            error = cudaMemcpy2DAsync(linear->h_output, execution->column_count * sizeof(float),
                                      linear->d_output + local_start, linear->resident_column_count * sizeof(float),
                                      execution->column_count * sizeof(float), rows, cudaMemcpyDeviceToHost,
                                      context->stream);
        }
        if (error != cudaSuccess) status = cuda_fail(context, error, "submit Q4_0 linear");
    }
    if (status != QPUCUDA_OK) {
        release(linear);
        delete submission;
        return status;
    }
    submission->submit_end = monotonic_ns();
    submission->linear = linear;
    submission->destination = static_cast<uint8_t *>(execution->destination);
    submission->destination_offset = execution->destination_offset;
    submission->rows = rows;
    submission->column_start = execution->column_start;
    submission->column_count = execution->column_count;
    submission->active = true;
    *result = submission;
    return QPUCUDA_OK;
}

qpucuda_status qpucuda_q4_0_submission_wait(qpucuda_q4_0_submission *submission, qpucuda_q4_0_timing *timing) {
    if (submission == nullptr || !submission->active || submission->linear == nullptr) {
        return QPUCUDA_INVALID_ARGUMENT;
    }
    qpucuda_q4_0_linear *linear = submission->linear;
    qpucuda_context *context = linear->context;
    const uint64_t wait_start = monotonic_ns();
    qpucuda_status status;
    {
        std::lock_guard<std::mutex> lock(context->mutex);
        DeviceGuard guard(context->device);
        status = wait_stream(context);
    }
    const uint64_t wait_end = monotonic_ns();
    uint64_t copy_end = wait_end;
    if (status == QPUCUDA_OK) {
        uint8_t *destination = submission->destination + submission->destination_offset;
        for (uint32_t row = 0; row < submission->rows; ++row) {
            const size_t offset =
                (static_cast<size_t>(row) * linear->output_columns + submission->column_start) * sizeof(float);
            std::memcpy(destination + offset, linear->h_output + static_cast<size_t>(row) * submission->column_count,
                        static_cast<size_t>(submission->column_count) * sizeof(float));
        }
        copy_end = monotonic_ns();
    }
    if (timing != nullptr) {
        timing->input_access_ns = submission->input_access_end - submission->complete_start;
        timing->input_pack_ns = submission->input_pack_end - submission->input_access_end;
        timing->input_sync_ns = submission->input_copy_end - submission->input_pack_end;
        timing->input_copy_ns = submission->input_copy_end - submission->complete_start;
        timing->submit_ns = submission->submit_end - submission->submit_start;
        timing->wait_ns = wait_end - wait_start;
        timing->submit_wait_ns = wait_end - submission->submit_start;
        timing->output_sync_ns = 0;
        timing->output_copy_ns = copy_end - wait_end;
        timing->complete_ns = copy_end - submission->complete_start;
    }
    submission->active = false;
    release(linear);
    return status;
}

qpucuda_status qpucuda_q4_0_submission_cpu_fallback(qpucuda_q4_0_submission *submission) {
    // The reference rejects this for every non-MX linear (qpu_llama_q4_0.c:836-839) and computes MX
    // linears on the host; this library has no host compute path.
    if (submission != nullptr && submission->linear != nullptr && submission->linear->rows > kMaxRows) {
        return fail(submission->linear->context, QPUCUDA_CAPABILITY_MISSING, "Q4_0 linear: no CPU path in this library");
    }
    return QPUCUDA_INVALID_ARGUMENT;
}

void qpucuda_q4_0_submission_destroy(qpucuda_q4_0_submission *submission) {
    if (submission == nullptr) return;
    if (submission->active) (void)qpucuda_q4_0_submission_wait(submission, nullptr);
    delete submission;
}

qpucuda_status qpucuda_q4_0_linear_execute(qpucuda_q4_0_linear *linear, const qpucuda_q4_0_execution *execution,
                                           qpucuda_q4_0_timing *timing) {
    qpucuda_q4_0_submission *submission = nullptr;
    qpucuda_status status = qpucuda_q4_0_linear_submit(linear, execution, &submission);
    if (status == QPUCUDA_OK) status = qpucuda_q4_0_submission_wait(submission, timing);
    qpucuda_q4_0_submission_destroy(submission);
    return status;
}

qpucuda_status qpucuda_q4_0_linear_execute_device(qpucuda_q4_0_linear *linear, const void *activation, uint32_t rows,
                                                  float *destination, size_t destination_stride,
                                                  uint32_t column_start, uint32_t column_count,
                                                  uint32_t output_column_start) {
    if (linear == nullptr) return QPUCUDA_INVALID_ARGUMENT;
    qpucuda_context *context = linear->context;
    const uint32_t local_start = column_start - linear->resident_column_start;
    if (activation == nullptr || destination == nullptr || rows == 0 || rows > linear->rows ||
        !window_ok(linear, column_start, column_count) ||
        destination_stride < static_cast<size_t>(output_column_start) + column_count) {
        return fail(context, QPUCUDA_INVALID_ARGUMENT, "Q4_0 linear: invalid device execution");
    }
    std::lock_guard<std::mutex> lock(context->mutex);
    qpucuda_status status = begin_submit(context);
    if (status != QPUCUDA_OK) return status;
    DeviceGuard guard(context->device);
    const cudaError_t error = launch_linear(linear, static_cast<const uint8_t *>(activation), nullptr, 0, rows, 0,
                                            destination, destination_stride, local_start, output_column_start,
                                            column_count);
    if (error != cudaSuccess) return cuda_fail(context, error, "launch Q4_0 linear");
    return QPUCUDA_OK;
}

qpucuda_status qpucuda_q4_0_linear_execute_f32_device(qpucuda_q4_0_linear *linear, const float *source,
                                                      size_t source_stride, uint32_t rows, float *destination,
                                                      size_t destination_stride, uint32_t column_start,
                                                      uint32_t column_count, uint32_t output_column_start) {
    if (linear == nullptr) return QPUCUDA_INVALID_ARGUMENT;
    qpucuda_context *context = linear->context;
    const uint32_t k = linear->blocks * kBlockElements;
    const uint32_t local_start = column_start - linear->resident_column_start;
    if (source == nullptr || destination == nullptr || rows == 0 || rows > linear->rows || source_stride < k ||
        !window_ok(linear, column_start, column_count) ||
        destination_stride < static_cast<size_t>(output_column_start) + column_count) {
        return fail(context, QPUCUDA_INVALID_ARGUMENT, "Q4_0 linear: invalid device execution");
    }
    std::lock_guard<std::mutex> lock(context->mutex);
    qpucuda_status status = begin_submit(context);
    if (status != QPUCUDA_OK) return status;
    DeviceGuard guard(context->device);
    // One launch: each CTA quantizes the fp32 blocks to Q8_0 as it stages them (the same
    // arithmetic as qpucuda_quantize_q8_0, so the result is that of quantize-then-execute).
    const cudaError_t error = launch_linear(linear, nullptr, source, source_stride, rows, 0, destination,
                                            destination_stride, local_start, output_column_start, column_count);
    if (error != cudaSuccess) return cuda_fail(context, error, "launch Q4_0 linear");
    return QPUCUDA_OK;
}

}  // extern "C"
