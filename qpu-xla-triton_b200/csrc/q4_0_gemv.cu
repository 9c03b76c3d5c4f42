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
// Two kernels:
//  * q4_0_direct_kernel (prepared weights, the operator's path). Prepared layout,
//    made once at prepare with the same 18 bytes per block as the native format:
//    nibbles [columns][blocks][16] and fp16 scales [columns][scale_stride]
//    (scale_stride = blocks rounded up to 8). One warp per output column (2 or 4
//    warps for long reductions, partials added in a fixed order); lane l takes
//    blocks l, l + 32, ..., a warp reads 512 contiguous bytes per 16-byte load,
//    eight loads in flight per lane; persistent CTAs sized from the occupancy
//    API with a balanced number of rounds.
//  * q4_0_native_kernel (single-kernel entry point over native 18-byte blocks,
//    which are only 2-byte aligned): lanes read each block as nine 16-bit loads.
// Both keep the weight codes packed: dp4a(nibbles & 0x0F0F0F0F, a[0..3]) and
// dp4a((nibbles >> 4) & 0x0F0F0F0F, a[16..19]) etc.; the -8 offset is one
// subtraction of 8 * sum(a) per block, precomputed when the activation (rows x K
// bytes, 16-byte aligned rows + fp32 block scales + block sums) is staged in
// shared memory once per CTA.
#include <cuda_fp16.h>

#include "qpucuda_internal.h"

namespace qpucuda {
namespace {


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
__device__ __forceinline__ void stage_activation(const ActivationView &view, int8_t *q, float *d, int *sum8,
                                                 uint32_t thread, uint32_t threads) {
    const uint32_t total = view.rows * view.blocks;
    const uint32_t interleaved_rows = view.interleave == 0 ? 0 : view.rows - view.rows % 4;
    for (uint32_t item = thread; item < total; item += threads) {
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

template <int ROWS>
__device__ __forceinline__ void warp_sum(float (&acc)[ROWS]) {
#pragma unroll
    for (int r = 0; r < ROWS; ++r) {
#pragma unroll
        for (int offset = 16; offset > 0; offset >>= 1) acc[r] = __fadd_rn(acc[r], __shfl_xor_sync(0xffffffffu, acc[r], offset));
    }
}

template <int ROWS>
__device__ __forceinline__ void store_rows(const float (&acc)[ROWS], uint32_t lane, float *destination,
                                           size_t destination_stride, size_t column) {
    if (lane < static_cast<uint32_t>(ROWS)) {
        float value = acc[0];
#pragma unroll
        for (int r = 1; r < ROWS; ++r)
            if (lane == static_cast<uint32_t>(r)) value = acc[r];
        destination[static_cast<size_t>(lane) * destination_stride + column] = value;
    }
}

size_t activation_bytes(uint32_t rows, uint32_t blocks) { return static_cast<size_t>(rows) * blocks * (32 + 4 + 4); }

// ---- direct-load kernel over the prepared layout -------------------------------------------

constexpr size_t kSmemBudget = 200u * 1024u;
constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kUnroll = 8;

__device__ __forceinline__ uint4 load_stream_u4(const void *p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

struct DirectParams {
    const uint8_t *nibbles;
    const uint16_t *scales;
    uint32_t blocks;
    uint32_t scale_stride;
    ActivationView view;
    float *destination;
    size_t destination_stride;
    uint32_t col0;      // first weight column (resident-relative)
    uint32_t out_col0;  // destination column of weight column col0
    uint32_t count;
};

// One warp per column; SPLIT warps share a column for long reductions: warp part p takes
// blocks p*32 + lane + i*32*SPLIT and the SPLIT partial sums are added in part order
// through shared memory (deterministic). Eight independent 16-byte loads per lane are in
// flight before any of them is consumed.
template <int ROWS, int SPLIT>
__global__ void __launch_bounds__(kThreads) q4_0_direct_kernel(const DirectParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ float partial[kWarps][ROWS];
    int8_t *q = reinterpret_cast<int8_t *>(smem);
    float *d = reinterpret_cast<float *>(smem + static_cast<size_t>(ROWS) * p.blocks * 32);
    int *sum8 = reinterpret_cast<int *>(d + static_cast<size_t>(ROWS) * p.blocks);
    stage_activation(p.view, q, d, sum8, threadIdx.x, blockDim.x);
    __syncthreads();

    constexpr uint32_t kSlots = kWarps / SPLIT;
    constexpr uint32_t kStride = 32 * SPLIT;  // blocks between a lane's consecutive blocks
    const uint32_t warp = threadIdx.x >> 5;
    const uint32_t lane = threadIdx.x & 31;
    const uint32_t part = warp % SPLIT;
    const uint32_t slot = warp / SPLIT;
    const uint32_t first = part * 32 + lane;
    for (uint32_t j = blockIdx.x * kSlots + slot; j < p.count; j += gridDim.x * kSlots) {
        const size_t column = p.col0 + j;
        const uint8_t *w_col = p.nibbles + column * p.blocks * 16;
        const uint16_t *s_col = p.scales + column * p.scale_stride;
        float acc[ROWS];
#pragma unroll
        for (int r = 0; r < ROWS; ++r) acc[r] = 0.0f;
        uint32_t b = first;
        for (; b + kStride * (kUnroll - 1) < p.blocks; b += kStride * kUnroll) {
            uint4 w[kUnroll];
            uint16_t s[kUnroll];
#pragma unroll
            for (int u = 0; u < kUnroll; ++u) {
                w[u] = load_stream_u4(w_col + static_cast<size_t>(b + kStride * u) * 16);
                s[u] = __ldg(s_col + b + kStride * u);
            }
#pragma unroll
            for (int u = 0; u < kUnroll; ++u) accumulate_block<ROWS>(w[u], s[u], b + kStride * u, p.blocks, q, d, sum8, acc);
        }
        for (; b < p.blocks; b += kStride) {
            accumulate_block<ROWS>(load_stream_u4(w_col + static_cast<size_t>(b) * 16), __ldg(s_col + b), b, p.blocks, q, d,
                                   sum8, acc);
        }
        warp_sum<ROWS>(acc);
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
                for (int q_part = 1; q_part < SPLIT; ++q_part) value = __fadd_rn(value, partial[slot * SPLIT + q_part][lane]);
                p.destination[static_cast<size_t>(lane) * p.destination_stride + p.out_col0 + j] = value;
            }
            asm volatile("bar.sync %0, %1;" ::"r"(1 + slot), "r"(32 * SPLIT) : "memory");
        } else {
            store_rows<ROWS>(acc, lane, p.destination, p.destination_stride, p.out_col0 + j);
        }
    }
}

// ---- native-block kernel (single-kernel entry point) --------------------------------------

constexpr int kNativeThreads = 256;
constexpr int kNativeWarps = kNativeThreads / 32;

struct NativeParams {
    const uint8_t *weight;  // [columns][blocks][18]
    uint32_t blocks;
    ActivationView view;
    float *destination;
    size_t destination_stride;
    uint32_t col0;
    uint32_t out_col0;
    uint32_t count;
};

template <int ROWS>
__global__ void __launch_bounds__(kNativeThreads) q4_0_native_kernel(const NativeParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    int8_t *q = reinterpret_cast<int8_t *>(smem);
    float *d = reinterpret_cast<float *>(smem + static_cast<size_t>(ROWS) * p.blocks * 32);
    int *sum8 = reinterpret_cast<int *>(d + static_cast<size_t>(ROWS) * p.blocks);
    stage_activation(p.view, q, d, sum8, threadIdx.x, blockDim.x);
    __syncthreads();
    const uint32_t lane = threadIdx.x & 31;
    for (uint32_t j = blockIdx.x * kNativeWarps + (threadIdx.x >> 5); j < p.count; j += gridDim.x * kNativeWarps) {
        const size_t column = p.col0 + j;
        float acc[ROWS];
#pragma unroll
        for (int r = 0; r < ROWS; ++r) acc[r] = 0.0f;
        for (uint32_t b = lane; b < p.blocks; b += 32) {
            // Native 18-byte blocks are 2-byte aligned: nine 16-bit loads.
            const uint16_t *src = reinterpret_cast<const uint16_t *>(p.weight + (column * p.blocks + b) * 18);
            uint4 w;
            w.x = static_cast<uint32_t>(src[1]) | (static_cast<uint32_t>(src[2]) << 16);
            w.y = static_cast<uint32_t>(src[3]) | (static_cast<uint32_t>(src[4]) << 16);
            w.z = static_cast<uint32_t>(src[5]) | (static_cast<uint32_t>(src[6]) << 16);
            w.w = static_cast<uint32_t>(src[7]) | (static_cast<uint32_t>(src[8]) << 16);
            accumulate_block<ROWS>(w, src[0], b, p.blocks, q, d, sum8, acc);
        }
        warp_sum<ROWS>(acc);
        store_rows<ROWS>(acc, lane, p.destination, p.destination_stride, p.out_col0 + j);
    }
}

template <int ROWS, int SPLIT>
cudaError_t launch_direct(const DirectParams &p, int sm_count, cudaStream_t stream) {
    const size_t smem = activation_bytes(ROWS, p.blocks);
    if (smem > kSmemBudget) return cudaErrorInvalidValue;
    auto kernel = q4_0_direct_kernel<ROWS, SPLIT>;
    if (smem > 48u * 1024u) {
        const cudaError_t error =
            cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (error != cudaSuccess) return error;
    }
    // Persistent CTAs filling the SM's real residency (each stages the activation once); the
    // grid is balanced so every column slot runs the same number of rounds (no straggling tail).
    int per_sm = 0;
    const cudaError_t error = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kThreads, smem);
    if (error != cudaSuccess) return error;
    if (per_sm < 1) per_sm = 1;
    constexpr uint32_t kSlots = kWarps / SPLIT;
    const uint64_t capacity = static_cast<uint64_t>(sm_count) * static_cast<uint64_t>(per_sm);
    const uint64_t rounds = (p.count + capacity * kSlots - 1) / (capacity * kSlots);
    const uint32_t grid = static_cast<uint32_t>((p.count + kSlots * rounds - 1) / (kSlots * rounds));
    kernel<<<grid, kThreads, smem, stream>>>(p);
    return cudaGetLastError();
}

template <int ROWS>
cudaError_t launch_rows(const DirectParams &p, int sm_count, cudaStream_t stream) {
    // Columns with many blocks are split over 2 or 4 warps so there are enough independent
    // units to keep every SM busy without a long last round.
    if (p.blocks >= 2048) return launch_direct<ROWS, 4>(p, sm_count, stream);
    if (p.blocks >= 512) return launch_direct<ROWS, 2>(p, sm_count, stream);
    return launch_direct<ROWS, 1>(p, sm_count, stream);
}

template <int ROWS>
cudaError_t launch_native(const NativeParams &p, int sm_count, cudaStream_t stream) {
    const size_t smem = activation_bytes(ROWS, p.blocks);
    if (smem > kSmemBudget) return cudaErrorInvalidValue;
    auto kernel = q4_0_native_kernel<ROWS>;
    if (smem > 48u * 1024u) {
        const cudaError_t error =
            cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (error != cudaSuccess) return error;
    }
    uint32_t grid = (p.count + kNativeWarps - 1) / kNativeWarps;
    const uint32_t cap = static_cast<uint32_t>(sm_count) * 4u;
    if (grid > cap) grid = cap;
    kernel<<<grid, kNativeThreads, smem, stream>>>(p);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_q4_0_q8_0_gemv(const Q40Weights &weights, const uint8_t *activation, uint32_t rows,
                                  uint32_t interleave, float *destination, size_t destination_stride, uint32_t col0,
                                  uint32_t out_col0, uint32_t count, unsigned int *error_word, int sm_count,
                                  cudaStream_t stream) {
    if (count == 0 || rows == 0) return cudaSuccess;
    if ((reinterpret_cast<uintptr_t>(weights.nibbles) & 15u) != 0 || (reinterpret_cast<uintptr_t>(weights.scales) & 15u) != 0 ||
        (reinterpret_cast<uintptr_t>(activation) & 1u) != 0 || weights.scale_stride % 8 != 0 ||
        weights.scale_stride < weights.blocks) {
        return cudaErrorInvalidValue;
    }
    DirectParams p{};
    p.nibbles = weights.nibbles;
    p.scales = weights.scales;
    p.blocks = weights.blocks;
    p.scale_stride = weights.scale_stride;
    p.view = ActivationView{activation, rows, weights.blocks, interleave};
    p.destination = destination;
    p.destination_stride = destination_stride;
    p.col0 = col0;
    p.out_col0 = out_col0;
    p.count = count;
    (void)error_word;  // the direct kernel has no barrier waits to bound
    switch (rows) {
        case 1: return launch_rows<1>(p, sm_count, stream);
        case 2: return launch_rows<2>(p, sm_count, stream);
        case 3: return launch_rows<3>(p, sm_count, stream);
        case 4: return launch_rows<4>(p, sm_count, stream);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_q4_0_q8_0_gemv_native(const uint8_t *activation, uint32_t rows, uint32_t blocks,
                                         const uint8_t *weight, float *destination, size_t destination_stride,
                                         uint32_t col0, uint32_t out_col0, uint32_t count, int sm_count,
                                         cudaStream_t stream) {
    if (count == 0 || rows == 0) return cudaSuccess;
    if ((reinterpret_cast<uintptr_t>(weight) & 1u) != 0 || (reinterpret_cast<uintptr_t>(activation) & 1u) != 0) {
        return cudaErrorInvalidValue;
    }
    const NativeParams p{weight, blocks, ActivationView{activation, rows, blocks, 0}, destination, destination_stride,
                         col0, out_col0, count};
    switch (rows) {
        case 1: return launch_native<1>(p, sm_count, stream);
        case 2: return launch_native<2>(p, sm_count, stream);
        case 3: return launch_native<3>(p, sm_count, stream);
        case 4: return launch_native<4>(p, sm_count, stream);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace qpucuda
