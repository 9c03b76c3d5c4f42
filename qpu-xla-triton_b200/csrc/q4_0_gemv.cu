// GGML Q4_0 x Q8_0 linear for M = 1..4 rows (HBM-bound on the 4-bit weight).
//
// Replaces the reference's vc7.ggml_q4_0_q8_0_linear QPU program
// (src/qpu_xla/kernels/ggml_q4_0.py:551-712, executor :783-841) and its native
// C operator (integrations/llama_cpp/src/qpu_llama_q4_0.c). Per output
// (m, n): y = sum over blocks b of ((float)dot_b * d_w[n, b]) * d_a[m, b], with
// dot_b the exact int32 dot of the 32 weight codes (code - 8) and the 32 int8
// activations (ggml_q4_0.py:81-100). Each block contribution is rounded exactly
// as the reference rounds it; the fp32 sum over blocks is a per-lane sum
// followed by a warp tree, a different order from the reference's sequential
// sum, so the result agrees to ~1e-6 relative rather than bit for bit.
//
// Prepared weight layout (made once at prepare, same bytes per block as the
// native 18-byte block): nibbles [columns][blocks][16] (16-byte aligned) and
// fp16 scales [columns][blocks]. One warp per output column (SPLIT = 2 or 4 warps for
// long reductions, their partials added in a fixed order); lane l takes blocks
// l, l + 32 * SPLIT, ..., so a warp reads 512 contiguous bytes of nibbles per load,
// eight loads in flight per lane.
// Weight codes stay packed: dp4a(nibbles & 0x0F0F0F0F, a[0..3]) and
// dp4a((nibbles >> 4) & 0x0F0F0F0F, a[16..19]) etc., and the -8 offset is one
// subtraction of 8 * sum(a) per block, precomputed when the activation is staged.
// The activation (rows x K bytes) is staged once per CTA in shared memory as
// 16-byte aligned int8 rows, fp32 block scales and block sums; CTAs are
// persistent over columns.
#include <cuda_fp16.h>

#include "qpucuda_internal.h"

namespace qpucuda {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kUnroll = 8;

struct ActivationView {
    const uint8_t *base;
    uint32_t rows;
    uint32_t blocks;
    uint32_t interleave;  // 0 native; 4 / 8 CPU_REPACK block_q8_0x4 groups
};

// Address of the fp16 scale and of value `index` of (row, block), following the
// reference's q8_0_source_block / q8_0_source_value (qpu_llama_q4_0.c:153-190):
// rows below rows - rows % 4 are stored as block_q8_0x4 groups when interleaved.
__device__ __forceinline__ void activation_block(const ActivationView &view, uint32_t row, uint32_t block,
                                                 const uint8_t **scale, const uint8_t **values) {
    const size_t row_bytes = static_cast<size_t>(view.blocks) * 34;
    const uint32_t interleaved_rows = view.interleave == 0 ? 0 : view.rows - view.rows % 4;
    if (row < interleaved_rows) {
        const uint8_t *group = view.base + static_cast<size_t>(row / 4) * 4 * row_bytes + static_cast<size_t>(block) * 4 * 34;
        *scale = group + (row % 4) * 2;
        *values = group + 8;
        return;
    }
    const uint8_t *native = view.base + static_cast<size_t>(row) * row_bytes + static_cast<size_t>(block) * 34;
    *scale = native;
    *values = native + 2;
}

__device__ __forceinline__ int8_t activation_value(const ActivationView &view, const uint8_t *values, uint32_t row,
                                                   uint32_t index) {
    const uint32_t interleaved_rows = view.interleave == 0 ? 0 : view.rows - view.rows % 4;
    if (row >= interleaved_rows) return static_cast<int8_t>(values[index]);
    const uint32_t il = view.interleave;
    return static_cast<int8_t>(values[(index / il) * 4 * il + (row % 4) * il + index % il]);
}

// Shared memory: q [rows][blocks * 32] int8, d [rows][blocks] fp32, sum8 [rows][blocks] int32.
// One thread per (row, block): a native block is read with independent 16-bit loads (blocks
// start on even bytes), so staging costs one round trip to L2 rather than one per block.
__device__ __forceinline__ void stage_activation(const ActivationView &view, int8_t *q, float *d, int *sum8) {
    const uint32_t total = view.rows * view.blocks;
    const uint32_t interleaved_rows = view.interleave == 0 ? 0 : view.rows - view.rows % 4;
    for (uint32_t item = threadIdx.x; item < total; item += blockDim.x) {
        const uint32_t row = item / view.blocks;
        const uint32_t block = item % view.blocks;
        const uint8_t *scale_bytes;
        const uint8_t *values;
        activation_block(view, row, block, &scale_bytes, &values);
        uint32_t words[8];
        if (row >= interleaved_rows) {
            const uint16_t *halves = reinterpret_cast<const uint16_t *>(values);
#pragma unroll
            for (int i = 0; i < 8; ++i)
                words[i] = static_cast<uint32_t>(halves[2 * i]) | (static_cast<uint32_t>(halves[2 * i + 1]) << 16);
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                uint32_t word = 0;
#pragma unroll
                for (int byte = 0; byte < 4; ++byte)
                    word |= static_cast<uint32_t>(static_cast<uint8_t>(activation_value(view, values, row, 4 * i + byte)))
                            << (8 * byte);
                words[i] = word;
            }
        }
        int sum = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) sum = __dp4a(static_cast<int>(words[i]), 0x01010101, sum);
        uint4 *destination = reinterpret_cast<uint4 *>(q + static_cast<size_t>(item) * 32);
        destination[0] = make_uint4(words[0], words[1], words[2], words[3]);
        destination[1] = make_uint4(words[4], words[5], words[6], words[7]);
        d[item] = __half2float(__ushort_as_half(*reinterpret_cast<const unsigned short *>(scale_bytes)));
        sum8[item] = 8 * sum;
    }
}

__device__ __forceinline__ uint4 load_stream_u4(const void *p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ int block_dot(uint4 w, const int8_t *a) {
    const int4 lo = *reinterpret_cast<const int4 *>(a);       // activation values 0..15
    const int4 hi = *reinterpret_cast<const int4 *>(a + 16);  // activation values 16..31
    int dot = 0;
    dot = __dp4a(static_cast<int>(w.x & 0x0F0F0F0Fu), lo.x, dot);
    dot = __dp4a(static_cast<int>((w.x >> 4) & 0x0F0F0F0Fu), hi.x, dot);
    dot = __dp4a(static_cast<int>(w.y & 0x0F0F0F0Fu), lo.y, dot);
    dot = __dp4a(static_cast<int>((w.y >> 4) & 0x0F0F0F0Fu), hi.y, dot);
    dot = __dp4a(static_cast<int>(w.z & 0x0F0F0F0Fu), lo.z, dot);
    dot = __dp4a(static_cast<int>((w.z >> 4) & 0x0F0F0F0Fu), hi.z, dot);
    dot = __dp4a(static_cast<int>(w.w & 0x0F0F0F0Fu), lo.w, dot);
    dot = __dp4a(static_cast<int>((w.w >> 4) & 0x0F0F0F0Fu), hi.w, dot);
    return dot;
}

template <int ROWS>
__device__ __forceinline__ void accumulate_block(uint4 w, uint16_t w_scale_bits, uint32_t block, uint32_t blocks,
                                                 const int8_t *q, const float *d, const int *sum8, float (&acc)[ROWS]) {
    const float dw = __half2float(__ushort_as_half(w_scale_bits));
#pragma unroll
    for (int r = 0; r < ROWS; ++r) {
        const size_t item = static_cast<size_t>(r) * blocks + block;
        const int dot = block_dot(w, q + item * 32) - sum8[item];
        acc[r] = __fadd_rn(acc[r], __fmul_rn(__fmul_rn(__int2float_rn(dot), dw), d[item]));
    }
}

// SPLIT warps share one column: warp part p takes blocks p*32 + lane + i*32*SPLIT, and
// the SPLIT partial sums are added in part order through shared memory (deterministic).
template <int ROWS, bool NATIVE, int SPLIT>
__global__ void __launch_bounds__(kThreads) q4_0_gemv_kernel(const uint8_t *__restrict__ nibbles,
                                                             const uint16_t *__restrict__ scales,
                                                             const uint8_t *__restrict__ native, uint32_t blocks,
                                                             ActivationView view, float *__restrict__ destination,
                                                             size_t destination_stride, uint32_t col0,
                                                             uint32_t out_col0, uint32_t count) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ float partial[kWarps][ROWS];
    int8_t *q = reinterpret_cast<int8_t *>(smem);
    float *d = reinterpret_cast<float *>(smem + static_cast<size_t>(ROWS) * blocks * 32);
    int *sum8 = reinterpret_cast<int *>(d + static_cast<size_t>(ROWS) * blocks);
    stage_activation(view, q, d, sum8);
    __syncthreads();

    constexpr uint32_t kSlots = kWarps / SPLIT;
    constexpr uint32_t kStride = 32 * SPLIT;  // blocks between a lane's consecutive blocks
    const uint32_t warp = threadIdx.x >> 5;
    const uint32_t lane = threadIdx.x & 31;
    const uint32_t part = warp % SPLIT;
    const uint32_t slot = warp / SPLIT;
    const uint32_t first = part * 32 + lane;
    for (uint32_t j = blockIdx.x * kSlots + slot; j < count; j += gridDim.x * kSlots) {
        const size_t column = col0 + j;
        float acc[ROWS];
#pragma unroll
        for (int r = 0; r < ROWS; ++r) acc[r] = 0.0f;
        if constexpr (NATIVE) {
            // Native 18-byte blocks: 2-byte aligned, read as nine 16-bit words.
            for (uint32_t b = first; b < blocks; b += kStride) {
                const uint16_t *src = reinterpret_cast<const uint16_t *>(native + (column * blocks + b) * 18);
                uint4 w;
                w.x = static_cast<uint32_t>(src[1]) | (static_cast<uint32_t>(src[2]) << 16);
                w.y = static_cast<uint32_t>(src[3]) | (static_cast<uint32_t>(src[4]) << 16);
                w.z = static_cast<uint32_t>(src[5]) | (static_cast<uint32_t>(src[6]) << 16);
                w.w = static_cast<uint32_t>(src[7]) | (static_cast<uint32_t>(src[8]) << 16);
                accumulate_block<ROWS>(w, src[0], b, blocks, q, d, sum8, acc);
            }
        } else {
            const uint8_t *w_col = nibbles + column * blocks * 16;
            const uint16_t *s_col = scales + column * blocks;
            uint32_t b = first;
            // Eight independent 16-byte loads in flight per lane (4 KB per warp).
            for (; b + kStride * (kUnroll - 1) < blocks; b += kStride * kUnroll) {
                uint4 w[kUnroll];
                uint16_t s[kUnroll];
#pragma unroll
                for (int u = 0; u < kUnroll; ++u) {
                    w[u] = load_stream_u4(w_col + static_cast<size_t>(b + kStride * u) * 16);
                    s[u] = __ldg(s_col + b + kStride * u);
                }
#pragma unroll
                for (int u = 0; u < kUnroll; ++u) accumulate_block<ROWS>(w[u], s[u], b + kStride * u, blocks, q, d, sum8, acc);
            }
            for (; b < blocks; b += kStride) {
                const uint4 w = load_stream_u4(w_col + static_cast<size_t>(b) * 16);
                accumulate_block<ROWS>(w, __ldg(s_col + b), b, blocks, q, d, sum8, acc);
            }
        }
#pragma unroll
        for (int r = 0; r < ROWS; ++r) {
#pragma unroll
            for (int offset = 16; offset > 0; offset >>= 1) acc[r] = __fadd_rn(acc[r], __shfl_xor_sync(0xffffffffu, acc[r], offset));
        }
        if constexpr (SPLIT > 1) {
            // The SPLIT warps of this slot run the same trip count, so the named barrier is safe.
            if (lane == 0) {
#pragma unroll
                for (int r = 0; r < ROWS; ++r) partial[warp][r] = acc[r];
            }
            asm volatile("bar.sync %0, %1;" ::"r"(1 + slot), "r"(32 * SPLIT) : "memory");
            if (part == 0 && lane < static_cast<uint32_t>(ROWS)) {
                float value = partial[slot * SPLIT][lane];
#pragma unroll
                for (int p = 1; p < SPLIT; ++p) value = __fadd_rn(value, partial[slot * SPLIT + p][lane]);
                destination[static_cast<size_t>(lane) * destination_stride + out_col0 + j] = value;
            }
            asm volatile("bar.sync %0, %1;" ::"r"(1 + slot), "r"(32 * SPLIT) : "memory");
        } else if (lane < static_cast<uint32_t>(ROWS)) {
            float value = acc[0];
#pragma unroll
            for (int r = 1; r < ROWS; ++r)
                if (lane == static_cast<uint32_t>(r)) value = acc[r];
            destination[static_cast<size_t>(lane) * destination_stride + out_col0 + j] = value;
        }
    }
}

size_t smem_bytes(uint32_t rows, uint32_t blocks) { return static_cast<size_t>(rows) * blocks * (32 + 4 + 4); }

struct LaunchArgs {
    const uint8_t *nibbles;
    const uint16_t *scales;
    const uint8_t *native;
    uint32_t blocks;
    ActivationView view;
    float *destination;
    size_t destination_stride;
    uint32_t col0;
    uint32_t out_col0;
    uint32_t count;
    int sm_count;
    cudaStream_t stream;
};

template <int ROWS, bool NATIVE, int SPLIT>
cudaError_t launch_split(const LaunchArgs &a) {
    const size_t smem = smem_bytes(ROWS, a.blocks);
    if (smem > 200u * 1024u) return cudaErrorInvalidValue;
    auto kernel = q4_0_gemv_kernel<ROWS, NATIVE, SPLIT>;
    if (smem > 48u * 1024u) {
        const cudaError_t error =
            cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (error != cudaSuccess) return error;
    }
    // Persistent CTAs filling the SM's real residency (each stages the activation once); the
    // grid is balanced so every column slot runs the same number of rounds (no straggling tail).
    int per_sm = 0;
    cudaError_t error = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kThreads, smem);
    if (error != cudaSuccess) return error;
    if (per_sm < 1) per_sm = 1;
    constexpr uint32_t kSlots = kWarps / SPLIT;
    const uint64_t capacity = static_cast<uint64_t>(a.sm_count) * static_cast<uint64_t>(per_sm);
    const uint64_t rounds = (a.count + capacity * kSlots - 1) / (capacity * kSlots);
    const uint32_t grid = static_cast<uint32_t>((a.count + kSlots * rounds - 1) / (kSlots * rounds));
    kernel<<<grid, kThreads, smem, a.stream>>>(a.nibbles, a.scales, a.native, a.blocks, a.view, a.destination,
                                               a.destination_stride, a.col0, a.out_col0, a.count);
    return cudaGetLastError();
}

template <int ROWS, bool NATIVE>
cudaError_t launch_rows(const LaunchArgs &a) {
    // Columns with many blocks are split over 2 or 4 warps so there are enough independent
    // units to keep every SM busy without a long last round.
    if (a.blocks >= 2048) return launch_split<ROWS, NATIVE, 4>(a);
    if (a.blocks >= 512) return launch_split<ROWS, NATIVE, 2>(a);
    return launch_split<ROWS, NATIVE, 1>(a);
}

template <bool NATIVE>
cudaError_t dispatch_rows(const LaunchArgs &a) {
    switch (a.view.rows) {
        case 1: return launch_rows<1, NATIVE>(a);
        case 2: return launch_rows<2, NATIVE>(a);
        case 3: return launch_rows<3, NATIVE>(a);
        case 4: return launch_rows<4, NATIVE>(a);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace

cudaError_t launch_q4_0_q8_0_gemv(const Q40Weights &weights, const uint8_t *activation, uint32_t rows,
                                  uint32_t interleave, float *destination, size_t destination_stride, uint32_t col0,
                                  uint32_t out_col0, uint32_t count, int sm_count, cudaStream_t stream) {
    if (count == 0 || rows == 0) return cudaSuccess;
    if ((reinterpret_cast<uintptr_t>(weights.nibbles) & 15u) != 0 || (reinterpret_cast<uintptr_t>(activation) & 1u) != 0) {
        return cudaErrorInvalidValue;
    }
    const LaunchArgs args{weights.nibbles, weights.scales, nullptr, weights.blocks,
                          ActivationView{activation, rows, weights.blocks, interleave},
                          destination, destination_stride, col0, out_col0, count, sm_count, stream};
    return dispatch_rows<false>(args);
}

cudaError_t launch_q4_0_q8_0_gemv_native(const uint8_t *activation, uint32_t rows, uint32_t blocks,
                                         const uint8_t *weight, float *destination, size_t destination_stride,
                                         uint32_t col0, uint32_t out_col0, uint32_t count, int sm_count,
                                         cudaStream_t stream) {
    if (count == 0 || rows == 0) return cudaSuccess;
    if ((reinterpret_cast<uintptr_t>(weight) & 1u) != 0 || (reinterpret_cast<uintptr_t>(activation) & 1u) != 0) {
        return cudaErrorInvalidValue;
    }
    const LaunchArgs args{nullptr, nullptr, weight, blocks, ActivationView{activation, rows, blocks, 0},
                          destination, destination_stride, col0, out_col0, count, sm_count, stream};
    return dispatch_rows<true>(args);
}

}  // namespace qpucuda
