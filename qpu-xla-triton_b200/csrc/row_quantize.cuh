// Per-row symmetric int8 quantization, element by element: the arithmetic shared by the row
// quantizer kernels (quantize.cu) and the one-row GEMV that quantizes its own activation
// (w8a8_gemv.cu), so both produce the same bytes and scale for a row.
// s = max(RN(max|x| / 127), RN(1/127)), q = clamp(rint(x / s), -127, 127), round-half-even
// (src/qpu_xla/models/tinyllama/quantization.py:156-171).
#pragma once

#include <cstdint>

namespace qpucuda {

// np.float32(1.0 / 127.0), the scale floor of every per-row quantizer (quantization.py:165).
__device__ __forceinline__ float scale_floor() { return __uint_as_float(0x3c010204u); }

__device__ __forceinline__ float row_scale_of(float amax) { return fmaxf(__fdiv_rn(amax, 127.0f), scale_floor()); }

__device__ __forceinline__ int quantize_value(float x, float scale) {
    const int v = __float2int_rn(__fdiv_rn(x, scale));
    return v < -127 ? -127 : (v > 127 ? 127 : v);
}

// Same result as quantize_value without a division per element: p = x * RN(1/scale) is within
// 3 * 2^-24 * |x/scale| < 2.3e-5 of RN(x/scale) (|x/scale| < 128, as |x| <= amax and
// scale >= RN(amax/127)). So when p lies farther than 2^-15 from every half-integer, RN(x/scale)
// sits strictly on the same side of it and rounds to the same integer; otherwise (about 6e-5 of
// the elements) the exact IEEE division decides. NaN and infinite inputs give 0 on both paths.
__device__ __forceinline__ int quantize_value_fast(float x, float scale, float inverse) {
    const float p = __fmul_rn(x, inverse);
    if (fabsf(p - rintf(p)) > 0.5f - 3.0517578125e-05f) return quantize_value(x, scale);
    const int v = __float2int_rn(p);
    return v < -127 ? -127 : (v > 127 ? 127 : v);
}

__device__ __forceinline__ uint32_t pack4(int a, int b, int c, int d) {
    return (static_cast<uint32_t>(a) & 0xffu) | ((static_cast<uint32_t>(b) & 0xffu) << 8) |
           ((static_cast<uint32_t>(c) & 0xffu) << 16) | ((static_cast<uint32_t>(d) & 0xffu) << 24);
}

__device__ __forceinline__ uint32_t quantize4(float4 v, float scale, float inverse) {
    return pack4(quantize_value_fast(v.x, scale, inverse), quantize_value_fast(v.y, scale, inverse),
                 quantize_value_fast(v.z, scale, inverse), quantize_value_fast(v.w, scale, inverse));
}

__device__ __forceinline__ float abs_max4(float amax, float4 v) {
    return fmaxf(amax, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
}

// Maximum over the CTA (every thread gets it); scratch holds one float per warp.
template <int THREADS>
__device__ __forceinline__ float block_max(float value, float *scratch) {
#pragma unroll
    for (int offset = 16; offset > 0; offset >>= 1) value = fmaxf(value, __shfl_xor_sync(0xffffffffu, value, offset));
    constexpr int kWarps = THREADS / 32;
    if constexpr (kWarps > 1) {
        const int warp = threadIdx.x >> 5;
        const int lane = threadIdx.x & 31;
        __syncthreads();  // scratch reuse across rows
        if (lane == 0) scratch[warp] = value;
        __syncthreads();
        value = lane < kWarps ? scratch[lane] : 0.0f;
#pragma unroll
        for (int offset = 16; offset > 0; offset >>= 1)
            value = fmaxf(value, __shfl_xor_sync(0xffffffffu, value, offset));
    }
    return value;
}

}  // namespace qpucuda
