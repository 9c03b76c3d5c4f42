// Single-kernel C entry points (include/qpucuda_kernels.h): argument checks,
// the context's submission rules, then one launch on the context stream.
#include <climits>

#include "qpucuda_internal.h"
#include "qpucuda_kernels.h"

using namespace qpucuda;

namespace {

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

qpucuda_status launched(qpucuda_context *context, cudaError_t error, const char *what) {
    if (error == cudaErrorInvalidValue) return cuda_fail(context, error, what, QPUCUDA_INVALID_ARGUMENT);
    if (error != cudaSuccess) return cuda_fail(context, error, what, QPUCUDA_SUBMISSION_FAILED);
    return QPUCUDA_OK;
}

// gemm_int8.py:298: K * 127 * 127 must fit in int32.
bool accumulation_fits(uint32_t k) { return static_cast<uint64_t>(k) * 127u * 127u <= static_cast<uint64_t>(INT32_MAX); }

qpucuda_status gemm_common(qpucuda_context *context, const int8_t *a, size_t a_stride, const int8_t *w,
                           size_t w_stride, uint32_t m, uint32_t n, uint32_t k, const GemmEpilogue &epilogue,
                           const char *what) {
    if (context == nullptr) return QPUCUDA_INVALID_ARGUMENT;
    if (a == nullptr || w == nullptr || epilogue.out == nullptr || k == 0 || !accumulation_fits(k) ||
        a_stride < k || w_stride < k || epilogue.out_stride < n || !aligned16(a) || !aligned16(w) ||
        a_stride % 16 != 0 || w_stride % 16 != 0) {
        return fail(context, QPUCUDA_INVALID_ARGUMENT,
                    "%s: int8 operands need 16-byte aligned rows, K * 127^2 <= INT32_MAX and in-range strides", what);
    }
    if (epilogue.mode != EpilogueMode::kStoreS32 && (epilogue.row_scales == nullptr || epilogue.col_scales == nullptr)) {
        return fail(context, QPUCUDA_INVALID_ARGUMENT, "%s: dequantization needs row and column scales", what);
    }
    if (m == 0 || n == 0) return QPUCUDA_OK;
    std::lock_guard<std::mutex> lock(context->mutex);
    qpucuda_status status = begin_submit(context);
    if (status != QPUCUDA_OK) return status;
    if (!(context->cc_major == 10 && context->cc_minor == 0)) {
        return fail(context, QPUCUDA_CAPABILITY_MISSING, "%s: the tcgen05 int8 GEMM needs an sm_100 device", what);
    }
    DeviceGuard guard(context->device);
    return launched(context,
                    run_w8a8_gemm(a, a_stride, w, w_stride, m, n, k, epilogue, context->d_error, context->sm_count,
                                  context->stream),
                    what);
}

}  // namespace

extern "C" {

qpucuda_status qpucuda_quantize_rows_int8(qpucuda_context *context, const float *x, size_t x_stride, uint32_t rows,
                                          uint32_t cols, uint32_t padded_cols, int8_t *q, size_t q_stride,
                                          float *scales) {
    if (context == nullptr) return QPUCUDA_INVALID_ARGUMENT;
    if (x == nullptr || q == nullptr || scales == nullptr || cols == 0 || padded_cols < cols || x_stride < cols ||
        q_stride < padded_cols) {
        return fail(context, QPUCUDA_INVALID_ARGUMENT, "quantize_rows_int8: invalid pointers or extents");
    }
    if (rows == 0) return QPUCUDA_OK;
    std::lock_guard<std::mutex> lock(context->mutex);
    qpucuda_status status = begin_submit(context);
    if (status != QPUCUDA_OK) return status;
    DeviceGuard guard(context->device);
    return launched(context,
                    launch_quantize_rows_int8(x, x_stride, rows, cols, padded_cols, q, q_stride, scales,
                                              context->d_error, context->stream),
                    "quantize_rows_int8");
}

qpucuda_status qpucuda_w8a8_gemm_s32(qpucuda_context *context, const int8_t *a, size_t a_stride, const int8_t *w,
                                     size_t w_stride, uint32_t m, uint32_t n, uint32_t k, int32_t *acc,
                                     size_t acc_stride) {
    GemmEpilogue epilogue;
    epilogue.mode = EpilogueMode::kStoreS32;
    epilogue.out = acc;
    epilogue.out_stride = acc_stride;
    return gemm_common(context, a, a_stride, w, w_stride, m, n, k, epilogue, "w8a8_gemm_s32");
}

qpucuda_status qpucuda_w8a8_gemm_dequantize(qpucuda_context *context, const int8_t *a, size_t a_stride,
                                            const int8_t *w, size_t w_stride, uint32_t m, uint32_t n, uint32_t k,
                                            const float *row_scales, const float *col_scales, const float *bias,
                                            float *out, size_t out_stride) {
    GemmEpilogue epilogue;
    epilogue.mode = bias != nullptr ? EpilogueMode::kDequantizeBias : EpilogueMode::kDequantize;
    epilogue.row_scales = row_scales;
    epilogue.col_scales = col_scales;
    epilogue.bias = bias;
    epilogue.out = out;
    epilogue.out_stride = out_stride;
    return gemm_common(context, a, a_stride, w, w_stride, m, n, k, epilogue, "w8a8_gemm_dequantize");
}

qpucuda_status qpucuda_w8a8_dequantize(qpucuda_context *context, const int32_t *acc, size_t acc_stride, uint32_t m,
                                       uint32_t n, const float *row_scales, const float *col_scales,
                                       const float *bias, float *out, size_t out_stride) {
    if (context == nullptr) return QPUCUDA_INVALID_ARGUMENT;
    if (acc == nullptr || row_scales == nullptr || col_scales == nullptr || out == nullptr || acc_stride < n ||
        out_stride < n) {
        return fail(context, QPUCUDA_INVALID_ARGUMENT, "w8a8_dequantize: invalid pointers or strides");
    }
    if (m == 0 || n == 0) return QPUCUDA_OK;
    std::lock_guard<std::mutex> lock(context->mutex);
    qpucuda_status status = begin_submit(context);
    if (status != QPUCUDA_OK) return status;
    DeviceGuard guard(context->device);
    GemmEpilogue epilogue;
    epilogue.mode = bias != nullptr ? EpilogueMode::kDequantizeBias : EpilogueMode::kDequantize;
    epilogue.row_scales = row_scales;
    epilogue.col_scales = col_scales;
    epilogue.bias = bias;
    epilogue.out = out;
    epilogue.out_stride = out_stride;
    return launched(context, launch_w8a8_dequantize(acc, acc_stride, m, n, epilogue, context->stream),
                    "w8a8_dequantize");
}

qpucuda_status qpucuda_w8a8_gemv(qpucuda_context *context, const int8_t *a, size_t a_stride, const int8_t *w,
                                 size_t w_stride, uint32_t m, uint32_t n, uint32_t k, int32_t *acc, size_t acc_stride,
                                 const float *row_scales, const float *col_scales, const float *bias, float *out,
                                 size_t out_stride) {
    if (context == nullptr) return QPUCUDA_INVALID_ARGUMENT;
    const bool dequantize = out != nullptr;
    if (a == nullptr || w == nullptr || k == 0 || k % 16 != 0 || m > 8 || !accumulation_fits(k) ||
        a_stride < k || w_stride < k || !aligned16(a) || !aligned16(w) || a_stride % 16 != 0 ||
        w_stride % 16 != 0 || (dequantize && (row_scales == nullptr || col_scales == nullptr || out_stride < n)) ||
        (!dequantize && (acc == nullptr || acc_stride < n))) {
        return fail(context, QPUCUDA_INVALID_ARGUMENT,
                    "w8a8_gemv: m <= 8, K a multiple of 16 with 16-byte aligned rows, and an output are required");
    }
    if (m == 0 || n == 0) return QPUCUDA_OK;
    std::lock_guard<std::mutex> lock(context->mutex);
    qpucuda_status status = begin_submit(context);
    if (status != QPUCUDA_OK) return status;
    DeviceGuard guard(context->device);
    GemmEpilogue epilogue;
    if (dequantize) {
        epilogue.mode = bias != nullptr ? EpilogueMode::kDequantizeBias : EpilogueMode::kDequantize;
        epilogue.row_scales = row_scales;
        epilogue.col_scales = col_scales;
        epilogue.bias = bias;
        epilogue.out = out;
        epilogue.out_stride = out_stride;
    } else {
        epilogue.mode = EpilogueMode::kStoreS32;
        epilogue.out = acc;
        epilogue.out_stride = acc_stride;
    }
    return launched(context,
                    launch_w8a8_gemv(a, a_stride, w, w_stride, m, n, k, epilogue, context->sm_count, context->stream),
                    "w8a8_gemv");
}

qpucuda_status qpucuda_ggml_q4_0_q8_0_linear(qpucuda_context *context, const uint8_t *activation, uint32_t rows,
                                             uint32_t blocks, const uint8_t *weight, uint32_t weight_outputs,
                                             float *destination, size_t destination_stride,
                                             uint32_t weight_column_start, uint32_t output_column_start,
                                             uint32_t column_count) {
    if (context == nullptr) return QPUCUDA_INVALID_ARGUMENT;
    // Contract of supports_ggml_q4_0_q8_0_linear (ggml_q4_0.py:725-761) for the small-M kernel.
    if (activation == nullptr || weight == nullptr || destination == nullptr || rows == 0 || rows > 4 ||
        blocks == 0 || weight_column_start % 16 != 0 || output_column_start % 16 != 0 || column_count == 0 ||
        column_count % 16 != 0 || static_cast<uint64_t>(weight_column_start) + column_count > weight_outputs ||
        static_cast<uint64_t>(output_column_start) + column_count > destination_stride) {
        return fail(context, QPUCUDA_INVALID_ARGUMENT,
                    "ggml_q4_0_q8_0_linear: rows 1..4 and 16-aligned column windows inside both matrices");
    }
    std::lock_guard<std::mutex> lock(context->mutex);
    qpucuda_status status = begin_submit(context);
    if (status != QPUCUDA_OK) return status;
    DeviceGuard guard(context->device);
    return launched(context,
                    launch_q4_0_q8_0_gemv_native(activation, rows, blocks, weight, destination, destination_stride,
                                                 weight_column_start, output_column_start, column_count,
                                                 context->sm_count, context->stream),
                    "ggml_q4_0_q8_0_linear");
}

qpucuda_status qpucuda_quantize_q8_0(qpucuda_context *context, const float *x, size_t x_stride, uint32_t rows,
                                     uint32_t cols, uint8_t *blocks) {
    if (context == nullptr) return QPUCUDA_INVALID_ARGUMENT;
    if (x == nullptr || blocks == nullptr || cols == 0 || cols % 32 != 0 || x_stride < cols) {
        return fail(context, QPUCUDA_INVALID_ARGUMENT, "quantize_q8_0: K must be a positive multiple of 32");
    }
    if (rows == 0) return QPUCUDA_OK;
    std::lock_guard<std::mutex> lock(context->mutex);
    qpucuda_status status = begin_submit(context);
    if (status != QPUCUDA_OK) return status;
    DeviceGuard guard(context->device);
    return launched(context, launch_quantize_q8_0(x, x_stride, rows, cols, blocks, context->stream), "quantize_q8_0");
}

qpucuda_status qpucuda_quantize_q4_0(qpucuda_context *context, const float *x, size_t x_stride, uint32_t rows,
                                     uint32_t cols, uint8_t *blocks) {
    if (context == nullptr) return QPUCUDA_INVALID_ARGUMENT;
    if (x == nullptr || blocks == nullptr || cols == 0 || cols % 32 != 0 || x_stride < cols) {
        return fail(context, QPUCUDA_INVALID_ARGUMENT, "quantize_q4_0: K must be a positive multiple of 32");
    }
    if (rows == 0) return QPUCUDA_OK;
    std::lock_guard<std::mutex> lock(context->mutex);
    qpucuda_status status = begin_submit(context);
    if (status != QPUCUDA_OK) return status;
    DeviceGuard guard(context->device);
    return launched(context, launch_quantize_q4_0(x, x_stride, rows, cols, blocks, context->stream), "quantize_q4_0");
}

qpucuda_status qpucuda_im2col_nchw_f32(qpucuda_context *context, const float *source, uint32_t batch, uint32_t channels,
                                       uint32_t height, uint32_t width, uint32_t channel_offset,
                                       uint32_t group_channels, uint32_t kernel_height, uint32_t kernel_width,
                                       uint32_t stride_h, uint32_t stride_w, uint32_t pad_h, uint32_t pad_w,
                                       uint32_t dilation_h, uint32_t dilation_w, float *destination,
                                       size_t destination_stride) {
    if (context == nullptr) return QPUCUDA_INVALID_ARGUMENT;
    const uint64_t span_h = static_cast<uint64_t>(dilation_h) * (kernel_height == 0 ? 0 : kernel_height - 1) + 1;
    const uint64_t span_w = static_cast<uint64_t>(dilation_w) * (kernel_width == 0 ? 0 : kernel_width - 1) + 1;
    if (source == nullptr || destination == nullptr || batch == 0 || channels == 0 || height == 0 || width == 0 ||
        group_channels == 0 || kernel_height == 0 || kernel_width == 0 || stride_h == 0 || stride_w == 0 ||
        dilation_h == 0 || dilation_w == 0 || static_cast<uint64_t>(channel_offset) + group_channels > channels ||
        static_cast<uint64_t>(height) + 2ull * pad_h < span_h || static_cast<uint64_t>(width) + 2ull * pad_w < span_w) {
        return fail(context, QPUCUDA_INVALID_ARGUMENT, "im2col: invalid convolution shape");
    }
    const uint32_t output_height = static_cast<uint32_t>((height + 2ull * pad_h - span_h) / stride_h + 1);
    const uint32_t output_width = static_cast<uint32_t>((width + 2ull * pad_w - span_w) / stride_w + 1);
    if (destination_stride < static_cast<uint64_t>(group_channels) * kernel_height * kernel_width) {
        return fail(context, QPUCUDA_INVALID_ARGUMENT, "im2col: destination rows are too short");
    }
    std::lock_guard<std::mutex> lock(context->mutex);
    qpucuda_status status = begin_submit(context);
    if (status != QPUCUDA_OK) return status;
    DeviceGuard guard(context->device);
    return launched(context,
                    launch_im2col_nchw_f32(source, batch, channels, height, width, channel_offset, group_channels,
                                           kernel_height, kernel_width, stride_h, stride_w, pad_h, pad_w, dilation_h,
                                           dilation_w, output_height, output_width, destination, destination_stride,
                                           context->stream),
                    "im2col");
}

}  // extern "C"
