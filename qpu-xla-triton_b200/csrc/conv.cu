// Convolution lowering for the W8A8 convolution plan (src/qpu_xla/ops/conv2d_w8a8.py:22-137).
//
// im2col of an NCHW fp32 tensor, as the reference's _im2col_nchw (src/qpu_xla/ops/conv2d.py:47-79):
// row (b, oh, ow) of the [batch * OH * OW][group_channels * KH * KW] matrix holds, at column
// (c * KH + i) * KW + j, source[b, channel_offset + c, oh * sh - ph + i * dh, ow * sw - pw + j * dw],
// or 0 where that position lies in the padding. Pointwise 1x1 convolutions skip this: the
// row quantizer reads NCHW pixels in place (launch_quantize_rows_int8_layout).
//
// One thread per output element; consecutive threads take consecutive columns of a row, so
// the writes are coalesced and the reads of one kernel row are contiguous in the source.
#include "qpucuda_internal.h"

namespace qpucuda {
namespace {

struct Im2colParams {
    const float *source;
    uint32_t channels, height, width;
    uint32_t channel_offset, group_channels;
    uint32_t kernel_height, kernel_width;
    uint32_t stride_h, stride_w, pad_h, pad_w, dilation_h, dilation_w;
    uint32_t output_height, output_width;
    uint64_t rows, cols;
    float *destination;
    size_t destination_stride;
};

__global__ void __launch_bounds__(256) im2col_nchw_kernel(const Im2colParams p) {
    const uint64_t total = p.rows * p.cols;
    for (uint64_t index = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; index < total;
         index += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        const uint64_t row = index / p.cols;
        const uint32_t col = static_cast<uint32_t>(index % p.cols);
        const uint32_t pixels = p.output_height * p.output_width;
        const uint32_t b = static_cast<uint32_t>(row / pixels);
        const uint32_t pixel = static_cast<uint32_t>(row % pixels);
        const uint32_t oh = pixel / p.output_width;
        const uint32_t ow = pixel % p.output_width;
        const uint32_t taps = p.kernel_height * p.kernel_width;
        const uint32_t c = col / taps;
        const uint32_t i = (col % taps) / p.kernel_width;
        const uint32_t j = col % p.kernel_width;
        const int64_t y = static_cast<int64_t>(oh) * p.stride_h - p.pad_h + static_cast<int64_t>(i) * p.dilation_h;
        const int64_t x = static_cast<int64_t>(ow) * p.stride_w - p.pad_w + static_cast<int64_t>(j) * p.dilation_w;
        float value = 0.0f;
        if (y >= 0 && y < p.height && x >= 0 && x < p.width) {
            const size_t offset = ((static_cast<size_t>(b) * p.channels + p.channel_offset + c) * p.height + y) * p.width + x;
            value = __ldg(p.source + offset);
        }
        p.destination[row * p.destination_stride + col] = value;
    }
}

}  // namespace

cudaError_t launch_im2col_nchw_f32(const float *source, uint32_t batch, uint32_t channels, uint32_t height,
                                   uint32_t width, uint32_t channel_offset, uint32_t group_channels,
                                   uint32_t kernel_height, uint32_t kernel_width, uint32_t stride_h,
                                   uint32_t stride_w, uint32_t pad_h, uint32_t pad_w, uint32_t dilation_h,
                                   uint32_t dilation_w, uint32_t output_height, uint32_t output_width,
                                   float *destination, size_t destination_stride, cudaStream_t stream) {
    Im2colParams p{};
    p.source = source;
    p.channels = channels;
    p.height = height;
    p.width = width;
    p.channel_offset = channel_offset;
    p.group_channels = group_channels;
    p.kernel_height = kernel_height;
    p.kernel_width = kernel_width;
    p.stride_h = stride_h;
    p.stride_w = stride_w;
    p.pad_h = pad_h;
    p.pad_w = pad_w;
    p.dilation_h = dilation_h;
    p.dilation_w = dilation_w;
    p.output_height = output_height;
    p.output_width = output_width;
    p.rows = static_cast<uint64_t>(batch) * output_height * output_width;
    p.cols = static_cast<uint64_t>(group_channels) * kernel_height * kernel_width;
    p.destination = destination;
    p.destination_stride = destination_stride;
    const uint64_t total = p.rows * p.cols;
    if (total == 0) return cudaSuccess;
    const uint64_t blocks = (total + 255) / 256;
    const uint32_t grid = static_cast<uint32_t>(blocks < 148ull * 64ull ? blocks : 148ull * 64ull);
    im2col_nchw_kernel<<<grid, 256, 0, stream>>>(p);
    return cudaGetLastError();
}

}  // namespace qpucuda
