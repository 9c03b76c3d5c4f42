// Small-M W8A8 kernels (HBM-bound on the weight, no tensor cores).
//
//  * w8a8_gemv: acc[m, n] = sum_k a[m, k] * w[n, k] for m <= 8 rows, exact int32.
//    Replaces vc7.w8a8_gemv (src/qpu_xla/kernels/gemv_int8.py:20-153), which the
//    reference selects for batch == 1 (src/qpu_xla/models/tinyllama/quantization.py:184).
//    One warp per output column n; each lane streams 16-byte chunks of the weight
//    row (a warp reads 512 contiguous bytes per step), multiplies them with
//    four dp4a per activation row and the warp reduces with shuffles. Integer
//    addition is associative, so the int32 result is exact in any order, and the
//    fused epilogue is the same ((float)acc * s_a) * s_w (+ bias) as the GEMM.
//  * w8a8_dequantize: the standalone vc7.w8a8_dequantize epilogue
//    (src/qpu_xla/kernels/w8a8_epilogue.py:20-96), elementwise.
#include "qpucuda_internal.h"

namespace qpucuda {
namespace {

struct GemvParams {
    const int8_t *a;
    size_t a_stride;
    const int8_t *w;
    size_t w_stride;
    uint32_t m, n, k;
    int mode;
    const float *row_scales;
    const float *col_scales;
    const float *bias;
    void *out;
    size_t out_stride;
};

__device__ __forceinline__ uint4 load_weight_chunk(const int8_t *p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ float dequant_value(int acc, float row_scale, float col_scale) {
    return __fmul_rn(__fmul_rn(__int2float_rn(acc), row_scale), col_scale);
}

template <int ROWS>
__global__ void __launch_bounds__(256) w8a8_gemv_kernel(const GemvParams p) {
    const uint32_t lane = threadIdx.x & 31;
    const uint32_t warps_total = gridDim.x * (blockDim.x / 32);
    const uint32_t chunks = p.k / 16;  // k is a multiple of 16 (rows are zero padded)
    for (uint32_t n = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5); n < p.n; n += warps_total) {
        const int8_t *w_row = p.w + static_cast<size_t>(n) * p.w_stride;
        int acc[ROWS];
#pragma unroll
        for (int r = 0; r < ROWS; ++r) acc[r] = 0;
        uint32_t c = lane;
        // Four independent 16-byte weight loads in flight per lane.
        for (; c + 96 < chunks; c += 128) {
            uint4 wv[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) wv[u] = load_weight_chunk(w_row + static_cast<size_t>(c + 32 * u) * 16);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
#pragma unroll
                for (int r = 0; r < ROWS; ++r) {
                    if (static_cast<uint32_t>(r) >= p.m) break;  // uniform across the warp
                    const uint4 av =
                        __ldg(reinterpret_cast<const uint4 *>(p.a + static_cast<size_t>(r) * p.a_stride) + c + 32 * u);
                    acc[r] = __dp4a(static_cast<int>(wv[u].x), static_cast<int>(av.x), acc[r]);
                    acc[r] = __dp4a(static_cast<int>(wv[u].y), static_cast<int>(av.y), acc[r]);
                    acc[r] = __dp4a(static_cast<int>(wv[u].z), static_cast<int>(av.z), acc[r]);
                    acc[r] = __dp4a(static_cast<int>(wv[u].w), static_cast<int>(av.w), acc[r]);
                }
            }
        }
        for (; c < chunks; c += 32) {
            const uint4 wv = load_weight_chunk(w_row + static_cast<size_t>(c) * 16);
#pragma unroll
            for (int r = 0; r < ROWS; ++r) {
                if (static_cast<uint32_t>(r) >= p.m) break;  // uniform across the warp
                const uint4 av = __ldg(reinterpret_cast<const uint4 *>(p.a + static_cast<size_t>(r) * p.a_stride) + c);
                acc[r] = __dp4a(static_cast<int>(wv.x), static_cast<int>(av.x), acc[r]);
                acc[r] = __dp4a(static_cast<int>(wv.y), static_cast<int>(av.y), acc[r]);
                acc[r] = __dp4a(static_cast<int>(wv.z), static_cast<int>(av.z), acc[r]);
                acc[r] = __dp4a(static_cast<int>(wv.w), static_cast<int>(av.w), acc[r]);
            }
        }
#pragma unroll
        for (int r = 0; r < ROWS; ++r) {
#pragma unroll
            for (int offset = 16; offset > 0; offset >>= 1) acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], offset);
        }
        if (lane < static_cast<uint32_t>(ROWS) && lane < p.m) {
            int value = acc[0];
#pragma unroll
            for (int r = 1; r < ROWS; ++r)
                if (lane == static_cast<uint32_t>(r)) value = acc[r];
            const size_t index = static_cast<size_t>(lane) * p.out_stride + n;
            if (p.mode == static_cast<int>(EpilogueMode::kStoreS32)) {
                static_cast<int32_t *>(p.out)[index] = value;
            } else {
                float v = dequant_value(value, p.row_scales[lane], p.col_scales[n]);
                if (p.mode == static_cast<int>(EpilogueMode::kDequantizeBias)) v = __fadd_rn(v, p.bias[n]);
                static_cast<float *>(p.out)[index] = v;
            }
        }
    }
}

__global__ void __launch_bounds__(256) w8a8_dequantize_kernel(const int32_t *__restrict__ acc, size_t acc_stride,
                                                              uint32_t m, uint32_t n, int mode,
                                                              const float *__restrict__ row_scales,
                                                              const float *__restrict__ col_scales,
                                                              const float *__restrict__ bias, float *__restrict__ out,
                                                              size_t out_stride) {
    const size_t total = static_cast<size_t>(m) * n;
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const size_t row = i / n;
        const size_t col = i % n;
        float v = dequant_value(acc[row * acc_stride + col], row_scales[row], col_scales[col]);
        if (mode == static_cast<int>(EpilogueMode::kDequantizeBias)) v = __fadd_rn(v, bias[col]);
        out[row * out_stride + col] = v;
    }
}

template <int ROWS>
cudaError_t launch_rows(const GemvParams &p, int sm_count, cudaStream_t stream) {
    const uint32_t warps_per_block = 8;
    uint32_t grid = (p.n + warps_per_block - 1) / warps_per_block;
    const uint32_t cap = static_cast<uint32_t>(sm_count) * 8u;
    if (grid > cap) grid = cap;
    w8a8_gemv_kernel<ROWS><<<grid, 256, 0, stream>>>(p);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_w8a8_gemv(const int8_t *a, size_t a_stride, const int8_t *w, size_t w_stride, uint32_t m,
                             uint32_t n, uint32_t k, const GemmEpilogue &epilogue, int sm_count,
                             cudaStream_t stream) {
    if (m == 0 || n == 0) return cudaSuccess;
    if (m > 8 || k % 16 != 0 || a_stride % 16 != 0 || w_stride % 16 != 0 ||
        (reinterpret_cast<uintptr_t>(a) & 15u) != 0 || (reinterpret_cast<uintptr_t>(w) & 15u) != 0) {
        return cudaErrorInvalidValue;
    }
    GemvParams p;
    p.a = a;
    p.a_stride = a_stride;
    p.w = w;
    p.w_stride = w_stride;
    p.m = m;
    p.n = n;
    p.k = k;
    p.mode = static_cast<int>(epilogue.mode);
    p.row_scales = epilogue.row_scales;
    p.col_scales = epilogue.col_scales;
    p.bias = epilogue.bias;
    p.out = epilogue.out;
    p.out_stride = epilogue.out_stride;
    switch (m) {
        case 1: return launch_rows<1>(p, sm_count, stream);
        case 2: return launch_rows<2>(p, sm_count, stream);
        case 3:
        case 4: return launch_rows<4>(p, sm_count, stream);
        default: return launch_rows<8>(p, sm_count, stream);
    }
}

cudaError_t launch_w8a8_dequantize(const int32_t *acc, size_t acc_stride, uint32_t m, uint32_t n,
                                   const GemmEpilogue &epilogue, cudaStream_t stream) {
    const size_t total = static_cast<size_t>(m) * n;
    if (total == 0) return cudaSuccess;
    size_t grid = (total + 255) / 256;
    if (grid > 148u * 32u) grid = 148u * 32u;
    w8a8_dequantize_kernel<<<static_cast<uint32_t>(grid), 256, 0, stream>>>(
        acc, acc_stride, m, n, static_cast<int>(epilogue.mode), epilogue.row_scales, epilogue.col_scales,
        epilogue.bias, static_cast<float *>(epilogue.out), epilogue.out_stride);
    return cudaGetLastError();
}

}  // namespace qpucuda
