/*
 * Single-kernel entry points of the quantized-linear path, device pointers,
 * asynchronous on the context stream. Each one is the CUDA counterpart of one
 * reference kernel handle (the Kernel objects of src/qpu_xla/kernels/), with
 * the reference's shape contract relaxed where the CUDA kernel has no tile
 * restriction (the reference's 16-multiple rule came from its 16-lane QPU).
 *
 * Layouts are row-major. int8 operand rows must start on 16-byte boundaries
 * (row strides a multiple of 16 bytes, 16-byte aligned bases) so that the
 * tensor-memory-accelerator can load them; pad K with zeros to reach that.
 */
#ifndef QPUCUDA_KERNELS_H
#define QPUCUDA_KERNELS_H

#include "qpucuda_runtime.h"

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

/* Per-row symmetric int8 quantization (quantization.py:156-171, :1085-1092):
 * scales[r] = max(max|x[r,:cols]| / 127, 1/127); q[r, c] = clip(rint(x/scale), -127, 127)
 * for c < cols and q[r, c] = 0 for cols <= c < padded_cols.
 * x: fp32 with row stride x_stride elements; q: int8 with row stride
 * q_stride bytes (>= padded_cols); scales: fp32 [rows]. */
qpucuda_status qpucuda_quantize_rows_int8(
    qpucuda_context *context,
    const float *x, size_t x_stride,
    uint32_t rows, uint32_t cols, uint32_t padded_cols,
    int8_t *q, size_t q_stride,
    float *scales);

/* vc7.tiled_w8a8_gemm (src/qpu_xla/kernels/gemm_int8.py:43-204, :285-320):
 * acc[m, n] = sum_k a[m, k] * w[n, k] in exact int32. a: int8 [M][K] row
 * stride a_stride bytes; w: int8 [N][K] (the weight's output-channel rows,
 * K contiguous) row stride w_stride bytes; acc row stride acc_stride elements.
 * Requires K * 127 * 127 <= INT32_MAX (gemm_int8.py:298). */
qpucuda_status qpucuda_w8a8_gemm_s32(
    qpucuda_context *context,
    const int8_t *a, size_t a_stride,
    const int8_t *w, size_t w_stride,
    uint32_t m, uint32_t n, uint32_t k,
    int32_t *acc, size_t acc_stride);

/* vc7.tiled_w8a8_gemm_dequantize (gemm_int8.py:166-184, :323-373) with the
 * bias fused: out[m, n] = ((float)acc * row_scales[m]) * col_scales[n]
 * (+ bias[n] when bias != NULL), fp32, row stride out_stride elements. */
qpucuda_status qpucuda_w8a8_gemm_dequantize(
    qpucuda_context *context,
    const int8_t *a, size_t a_stride,
    const int8_t *w, size_t w_stride,
    uint32_t m, uint32_t n, uint32_t k,
    const float *row_scales, const float *col_scales, const float *bias,
    float *out, size_t out_stride);

/* vc7.w8a8_dequantize (src/qpu_xla/kernels/w8a8_epilogue.py:20-96):
 * out = ((float)acc * row_scales[m]) * col_scales[n] (+ bias[n]). */
qpucuda_status qpucuda_w8a8_dequantize(
    qpucuda_context *context,
    const int32_t *acc, size_t acc_stride,
    uint32_t m, uint32_t n,
    const float *row_scales, const float *col_scales, const float *bias,
    float *out, size_t out_stride);

/* vc7.w8a8_gemv (src/qpu_xla/kernels/gemv_int8.py:20-153), generalised to
 * m <= 8 rows: exact int32 acc[m, n] with the int8 dot-product units.
 * When out != NULL the fused dequant (+bias) epilogue writes fp32 instead
 * of acc (acc may then be NULL). */
qpucuda_status qpucuda_w8a8_gemv(
    qpucuda_context *context,
    const int8_t *a, size_t a_stride,
    const int8_t *w, size_t w_stride,
    uint32_t m, uint32_t n, uint32_t k,
    int32_t *acc, size_t acc_stride,
    const float *row_scales, const float *col_scales, const float *bias,
    float *out, size_t out_stride);

/* vc7.ggml_q4_0_q8_0_linear (src/qpu_xla/kernels/ggml_q4_0.py:551-712,
 * :783-841) over native blocks: activation [rows][blocks][34], weight
 * [weight_outputs][blocks][18]; writes destination[r][output_column_start + j]
 * = sum_b ((float)dot * d_w) * d_a for weight column weight_column_start + j,
 * j < column_count; other destination columns are untouched.
 * rows 1..4. The fp32 block sum is reduced in a different order from the
 * reference, so results agree to ~1e-6 relative, not bit for bit. */
qpucuda_status qpucuda_ggml_q4_0_q8_0_linear(
    qpucuda_context *context,
    const uint8_t *activation, uint32_t rows, uint32_t blocks,
    const uint8_t *weight, uint32_t weight_outputs,
    float *destination, size_t destination_stride,
    uint32_t weight_column_start, uint32_t output_column_start, uint32_t column_count);

/* fp32 rows -> native block_q8_0 [rows][cols/32][34]
 * (examples/benchmark_llama_cpp_qpu_persistent_q4.py:42-54). cols % 32 == 0. */
qpucuda_status qpucuda_quantize_q8_0(
    qpucuda_context *context,
    const float *x, size_t x_stride, uint32_t rows, uint32_t cols,
    uint8_t *blocks);

/* im2col of one channel group of an NCHW fp32 tensor for a convolution, as the
 * reference's _im2col_nchw (src/qpu_xla/ops/conv2d.py:47-79): row (b, oh, ow) of the
 * [batch * output_height * output_width][group_channels * kernel_height * kernel_width]
 * destination holds, at column (c * kernel_height + i) * kernel_width + j, the source
 * value at channel channel_offset + c, row oh * stride_h - pad_h + i * dilation_h,
 * column ow * stride_w - pad_w + j * dilation_w, or 0 inside the padding. */
qpucuda_status qpucuda_im2col_nchw_f32(
    qpucuda_context *context,
    const float *source, uint32_t batch, uint32_t channels, uint32_t height, uint32_t width,
    uint32_t channel_offset, uint32_t group_channels, uint32_t kernel_height, uint32_t kernel_width,
    uint32_t stride_h, uint32_t stride_w, uint32_t pad_h, uint32_t pad_w, uint32_t dilation_h,
    uint32_t dilation_w, float *destination, size_t destination_stride);

/* fp32 rows -> native block_q4_0 [rows][cols/32][18] (ggml's published
 * quantize_row_q4_0_ref: d = signed max-magnitude / -8, codes min(15, trunc(x/d + 8.5))). */
qpucuda_status qpucuda_quantize_q4_0(
    qpucuda_context *context,
    const float *x, size_t x_stride, uint32_t rows, uint32_t cols,
    uint8_t *blocks);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif
#ifdef __cplusplus
}
#endif

#endif
