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
//  * q4_0_stream_kernel (prepared weights, the operator's path). Prepared layout,
//    made once at prepare with the same 18 bytes per block as the native format:
//    nibbles [columns][blocks][16] and fp16 scales [columns][scale_stride]
//    (scale_stride = blocks rounded up to 8, so every column's scales are a
//    16-byte multiple). One persistent CTA per SM owns a contiguous column
//    range; a producer thread streams each column's nibbles and scales into a
//    ring of shared-memory slots with 1D TMA bulk copies (cp.async.bulk +
//    mbarrier complete_tx), keeping ~100-160 KB per SM in flight with no register
//    cost; consumer warps take one column each from the ring (lane l reads
//    blocks l, l + 32, ... from shared memory) and release the slot.
//  * q4_0_native_kernel (single-kernel entry point over native 18-byte blocks,
//    which are only 2-byte aligned): lanes read each block as nine 16-bit loads.
// Both keep the weight codes packed: dp4a(nibbles & 0x0F0F0F0F, a[0..3]) and
// dp4a((nibbles >> 4) & 0x0F0F0F0F, a[16..19]) etc.; the -8 offset is one
// subtraction of 8 * sum(a) per block, precomputed when the activation (rows x K
// bytes, 16-byte aligned rows + fp32 block scales + block sums) is staged in
// shared memory once per CTA.
#include <cuda_fp16.h>

#include "qpucuda_internal.h"
#include "sm100_sync.cuh"

namespace qpucuda {
namespace {

using namespace sm100;

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

// ---- streaming kernel over the prepared layout ------------------------------------------

constexpr int kMaxSlots = 32;
constexpr size_t kSmemBudget = 200u * 1024u;

struct StreamParams {
    const uint8_t *nibbles;
    const uint16_t *scales;
    uint32_t blocks;
    uint32_t scale_stride;  // fp16 scales per column row (blocks rounded up to 8)
    ActivationView view;
    float *destination;
    size_t destination_stride;
    uint32_t col0;      // first weight column (resident-relative)
    uint32_t out_col0;  // destination column of weight column col0
    uint32_t count;
    uint32_t slots;
    uint32_t slot_bytes;
    uint32_t act_bytes;  // activation area, 128-aligned
    unsigned int *error_word;
};

template <int ROWS, int CONSUMERS>
__global__ void __launch_bounds__(32 * (CONSUMERS + 1), 1) q4_0_stream_kernel(const StreamParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint64_t full_bar[kMaxSlots];
    __shared__ uint64_t empty_bar[kMaxSlots];
    __shared__ volatile int abort_flag;
    int8_t *q = reinterpret_cast<int8_t *>(smem);
    float *d = reinterpret_cast<float *>(smem + static_cast<size_t>(ROWS) * p.blocks * 32);
    int *sum8 = reinterpret_cast<int *>(d + static_cast<size_t>(ROWS) * p.blocks);
    uint8_t *ring = smem + p.act_bytes;

    // This CTA's contiguous column range, balanced to within one column.
    const uint32_t per = p.count / gridDim.x;
    const uint32_t extra = p.count % gridDim.x;
    const uint32_t begin = blockIdx.x * per + (blockIdx.x < extra ? blockIdx.x : extra);
    const uint32_t columns = per + (blockIdx.x < extra ? 1u : 0u);
    const uint32_t nibble_bytes = p.blocks * 16;
    const uint32_t scale_bytes = p.scale_stride * 2;

    const uint32_t warp = threadIdx.x >> 5;
    const uint32_t lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < p.slots; ++s) {
            mbar_init(smem_u32(&full_bar[s]), 1);
            mbar_init(smem_u32(&empty_bar[s]), 1);
        }
        abort_flag = 0;
        mbar_init_fence();
    }
    __syncthreads();

    if (warp == CONSUMERS) {
        // ---- producer: one thread streams every column of the range through the ring ----
        if (lane == 0) {
            bool ok = true;
            uint32_t issued = 0;
            for (uint32_t i = 0; i < columns; ++i) {
                const uint32_t slot = i % p.slots;
                const uint32_t round = i / p.slots;
                if (round > 0 && !wait_bounded(smem_u32(&empty_bar[slot]), (round - 1) & 1u, &abort_flag, p.error_word)) {
                    ok = false;
                    break;
                }
                const uint32_t bar = smem_u32(&full_bar[slot]);
                const size_t column = p.col0 + begin + i;
                uint8_t *destination = ring + static_cast<size_t>(slot) * p.slot_bytes;
                mbar_expect_tx(bar, nibble_bytes + scale_bytes);
                bulk_load(smem_u32(destination), p.nibbles + column * nibble_bytes, nibble_bytes, bar);
                bulk_load(smem_u32(destination + nibble_bytes), p.scales + column * p.scale_stride, scale_bytes, bar);
                issued = i + 1;
            }
            if (!ok) {
                // Abort path: let this thread's copies land before the CTA exits.
                for (uint32_t i = issued > p.slots ? issued - p.slots : 0; i < issued; ++i) {
                    wait_drain(smem_u32(&full_bar[i % p.slots]), (i / p.slots) & 1u);
                }
            }
        }
        __syncwarp();  // reconverge before the CTA barrier below
    } else {
        // ---- consumers: stage the activation, then one column per warp from the ring ----
        stage_activation(p.view, q, d, sum8, threadIdx.x, 32 * CONSUMERS);
        asm volatile("bar.sync 1, %0;" ::"r"(32 * CONSUMERS) : "memory");
        for (uint32_t i = warp; i < columns; i += CONSUMERS) {
            const uint32_t slot = i % p.slots;
            bool ok = true;
            if (lane == 0) ok = wait_bounded(smem_u32(&full_bar[slot]), (i / p.slots) & 1u, &abort_flag, p.error_word);
            if (__shfl_sync(0xffffffffu, ok ? 1 : 0, 0) == 0) break;
            const uint8_t *slot_base = ring + static_cast<size_t>(slot) * p.slot_bytes;
            const uint4 *w = reinterpret_cast<const uint4 *>(slot_base);
            const uint16_t *s = reinterpret_cast<const uint16_t *>(slot_base + nibble_bytes);
            float acc[ROWS];
#pragma unroll
            for (int r = 0; r < ROWS; ++r) acc[r] = 0.0f;
#pragma unroll 4
            for (uint32_t b = lane; b < p.blocks; b += 32) accumulate_block<ROWS>(w[b], s[b], b, p.blocks, q, d, sum8, acc);
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&empty_bar[slot]));
            warp_sum<ROWS>(acc);
            store_rows<ROWS>(acc, lane, p.destination, p.destination_stride, p.out_col0 + begin + i);
        }
    }
    __syncthreads();
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

template <int ROWS, int CONSUMERS>
cudaError_t launch_stream(StreamParams p, int sm_count, cudaStream_t stream) {
    const size_t act = (activation_bytes(ROWS, p.blocks) + 127) & ~static_cast<size_t>(127);
    const size_t slot = (static_cast<size_t>(p.blocks) * 16 + static_cast<size_t>(p.scale_stride) * 2 + 127) &
                        ~static_cast<size_t>(127);
    if (act + slot > kSmemBudget) return cudaErrorInvalidValue;
    size_t slots = (kSmemBudget - act) / slot;
    if (slots > static_cast<size_t>(kMaxSlots)) slots = kMaxSlots;
    const size_t smem = act + slots * slot;
    auto kernel = q4_0_stream_kernel<ROWS, CONSUMERS>;
    cudaError_t error = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (error != cudaSuccess) return error;
    p.slots = static_cast<uint32_t>(slots);
    p.slot_bytes = static_cast<uint32_t>(slot);
    p.act_bytes = static_cast<uint32_t>(act);
    const uint32_t grid = p.count < static_cast<uint32_t>(sm_count) ? p.count : static_cast<uint32_t>(sm_count);
    kernel<<<grid, 32 * (CONSUMERS + 1), smem, stream>>>(p);
    return cudaGetLastError();
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
    StreamParams p{};
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
    p.error_word = error_word;
    switch (rows) {
        case 1: return launch_stream<1, 8>(p, sm_count, stream);
        case 2: return launch_stream<2, 8>(p, sm_count, stream);
        case 3: return launch_stream<3, 16>(p, sm_count, stream);
        case 4: return launch_stream<4, 16>(p, sm_count, stream);
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
