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
//    (scale_stride = blocks rounded up to 8). A warp owns two adjacent columns; lane l
//    takes blocks l, l + 32, ..., so a warp reads 512 contiguous bytes of each column per
//    16-byte load, with eight such loads in flight per lane; persistent CTAs sized from the
//    occupancy API with a balanced number of rounds.
//  * q4_0_native_kernel (single-kernel entry point over native 18-byte blocks,
//    which are only 2-byte aligned): lanes read each block as nine 16-bit loads.
// Both keep the weight codes packed: dp4a(nibbles & 0x0F0F0F0F, a[0..3]) and
// dp4a((nibbles >> 4) & 0x0F0F0F0F, a[16..19]) etc.; the -8 offset seeds each block's
// dp4a chain with -8 * sum(a), precomputed when the activation (rows x K bytes + fp32
// block scales + block sums) is staged in shared memory once per CTA.
#include <cuda_fp16.h>

#include "qpucuda_internal.h"

namespace qpucuda {
namespace {


struct ActivationView {
    const uint8_t *base;
    uint32_t rows;
    uint32_t blocks;
    uint32_t interleave;  // 0 native; 4 / 8 CPU_REPACK block_q8_0x4 groups
    // fp32 rows instead of Q8_0 blocks: each block is quantized to Q8_0 while it is staged.
    const float *f32;
    size_t f32_stride;  // elements
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

// Shared memory holds the activation in a split layout so that consecutive lanes, which
// take consecutive blocks, read consecutive 16-byte words (no bank conflicts):
//   lo   [rows * blocks] int4  values 0..15 of each (row, block)
//   hi   [rows * blocks] int4  values 16..31
//   meta [rows * blocks] int2  {fp32 bits of the block scale, -8 * sum of the 32 values}
// The -8 * sum seeds the dp4a chain, which turns the unsigned 4-bit codes (0..15) into
// code - 8 without unpacking them to signed bytes.
struct StagedActivation {
    int4 *lo;
    int4 *hi;
    int2 *meta;
};

__device__ __forceinline__ StagedActivation staged_activation(uint8_t *smem, uint32_t items) {
    int4 *lo = reinterpret_cast<int4 *>(smem);
    int4 *hi = lo + items;
    return StagedActivation{lo, hi, reinterpret_cast<int2 *>(hi + items)};
}

size_t activation_bytes(uint32_t rows, uint32_t blocks) { return static_cast<size_t>(rows) * blocks * (16 + 16 + 8); }

// Q8_0 quantization of one block of 32 fp32 values, exactly as quantize_q8_0_kernel (and the
// reference's restatement of ggml's quantize_row_q8_0, examples/benchmark_llama_cpp_qpu_
// persistent_q4.py:42-54): d = amax / 127, q = rint(x * (1/d)) clamped to +-127, fp16(d) kept.
__device__ __forceinline__ void quantize_f32_block(const float *x, bool vector, uint32_t (&words)[8],
                                                   uint16_t &scale_bits) {
    float v[32];
    if (vector) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float4 f = __ldg(reinterpret_cast<const float4 *>(x) + i);
            v[4 * i] = f.x;
            v[4 * i + 1] = f.y;
            v[4 * i + 2] = f.z;
            v[4 * i + 3] = f.w;
        }
    } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = __ldg(x + i);
    }
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
    const float d = __fdiv_rn(amax, 127.0f);
    const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
#pragma unroll
    for (int w = 0; w < 8; ++w) {
        uint32_t word = 0;
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            int q = __float2int_rn(__fmul_rn(v[4 * w + b], id));
            q = q < -127 ? -127 : (q > 127 ? 127 : q);
            word |= static_cast<uint32_t>(static_cast<uint8_t>(static_cast<int8_t>(q))) << (8 * b);
        }
        words[w] = word;
    }
    scale_bits = __half_as_ushort(__float2half_rn(d));
}

__device__ __forceinline__ void read_activation_item(const ActivationView &view, uint32_t item, uint32_t (&words)[8],
                                                     uint16_t &scale_bits) {
    const uint32_t row = item / view.blocks;
    const uint32_t block = item % view.blocks;
    const uint32_t interleaved_rows = view.interleave == 0 ? 0 : view.rows - view.rows % 4;
    const uint8_t *scale_bytes;
    const uint8_t *values;
    activation_block(view, row, block, &scale_bytes, &values);
    scale_bits = *reinterpret_cast<const uint16_t *>(scale_bytes);
    if (row >= interleaved_rows) {
        // Native blocks start on even bytes: sixteen independent 16-bit loads.
        const uint16_t *halves = reinterpret_cast<const uint16_t *>(values);
#pragma unroll
        for (int i = 0; i < 8; ++i)
            words[i] = static_cast<uint32_t>(halves[2 * i]) | (static_cast<uint32_t>(halves[2 * i + 1]) << 16);
        return;
    }
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

__device__ __forceinline__ void write_activation_item(const StagedActivation &staged, uint32_t item,
                                                      const uint32_t (&words)[8], uint16_t scale_bits) {
    int sum = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) sum = __dp4a(static_cast<int>(words[i]), 0x01010101, sum);
    staged.lo[item] = make_int4(words[0], words[1], words[2], words[3]);
    staged.hi[item] = make_int4(words[4], words[5], words[6], words[7]);
    staged.meta[item] = make_int2(__float_as_int(__half2float(__ushort_as_half(scale_bits))), -8 * sum);
}

// One thread per (row, block) item, two items per trip so two L2 round trips overlap. With
// F32, the items are quantized from fp32 rows (one per trip: 32 values in registers each).
template <bool F32>
__device__ __forceinline__ void stage_activation(const ActivationView &view, const StagedActivation &staged,
                                                 uint32_t thread, uint32_t threads) {
    const uint32_t total = view.rows * view.blocks;
    if constexpr (F32) {
        const bool vector = (reinterpret_cast<uintptr_t>(view.f32) & 15u) == 0 && (view.f32_stride & 3u) == 0;
        for (uint32_t item = thread; item < total; item += threads) {
            const uint32_t row = item / view.blocks;
            const uint32_t block = item % view.blocks;
            uint32_t words[8];
            uint16_t scale;
            quantize_f32_block(view.f32 + static_cast<size_t>(row) * view.f32_stride + static_cast<size_t>(block) * 32,
                               vector, words, scale);
            write_activation_item(staged, item, words, scale);
        }
        return;
    }
    for (uint32_t item = thread; item < total; item += 2 * threads) {
        uint32_t words0[8], words1[8];
        uint16_t scale0, scale1 = 0;
        const bool second = item + threads < total;
        read_activation_item(view, item, words0, scale0);
        if (second) read_activation_item(view, item + threads, words1, scale1);
        write_activation_item(staged, item, words0, scale0);
        if (second) write_activation_item(staged, item + threads, words1, scale1);
    }
}

// Exact int32 dot of one block: sum of (code - 8) * a over the 32 values. Weight word i holds
// codes i*4..i*4+3 in its low nibbles and codes 16+i*4.. in its high nibbles (GGML order).
__device__ __forceinline__ int block_dot(uint4 w, int4 lo, int4 hi, int seed) {
    int dot = seed;
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

// acc[r][c] += ((float)dot * d_w[c]) * d_a[r], rounded step by step as the reference rounds
// each block term (ggml_q4_0.py:81-100).
template <int ROWS, int COLS>
__device__ __forceinline__ void accumulate_block(const uint4 (&w)[COLS], const float (&dw)[COLS], uint32_t item,
                                                 uint32_t blocks, const StagedActivation &staged,
                                                 float (&acc)[ROWS][COLS]) {
#pragma unroll
    for (int r = 0; r < ROWS; ++r) {
        const uint32_t at = static_cast<uint32_t>(r) * blocks + item;
        const int4 lo = staged.lo[at];
        const int4 hi = staged.hi[at];
        const int2 meta = staged.meta[at];
        const float da = __int_as_float(meta.x);
#pragma unroll
        for (int c = 0; c < COLS; ++c)
            acc[r][c] = __fadd_rn(acc[r][c], __fmul_rn(__fmul_rn(__int2float_rn(block_dot(w[c], lo, hi, meta.y)), dw[c]), da));
    }
}

template <int N>
__device__ __forceinline__ void warp_sum(float (&values)[N]) {
#pragma unroll
    for (int i = 0; i < N; ++i) {
#pragma unroll
        for (int offset = 16; offset > 0; offset >>= 1)
            values[i] = __fadd_rn(values[i], __shfl_xor_sync(0xffffffffu, values[i], offset));
    }
}

// ---- direct-load kernel over the prepared layout -------------------------------------------

constexpr size_t kSmemBudget = 200u * 1024u;
constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;

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

// A warp owns COLS adjacent columns (a "group"); SPLIT warps share a group for long
// reductions. Lane l of part q takes blocks q*32 + l + i*32*SPLIT; each trip loads UNROLL such
// blocks of every column of the group (UNROLL * COLS independent 16-byte loads in flight per
// lane) before any is consumed, and each staged activation word read from shared memory
// serves COLS weight blocks. The first trip of a warp's first group is loaded before the
// activation is staged, and the first trip of its next group before the warp reduces the
// current one, so the weight stream does not stop for either. Partial sums of a group's
// SPLIT warps are added in part order through shared memory (deterministic). Registers per
// thread are capped so that MIN_BLOCKS CTAs of 256 threads fit on an SM.
template <int ROWS, int SPLIT, int COLS, int UNROLL, int MIN_BLOCKS, bool F32>
__global__ void __launch_bounds__(kThreads, MIN_BLOCKS) q4_0_direct_kernel(const DirectParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ float partial[kWarps][ROWS * COLS];
    constexpr uint32_t kSlots = kWarps / SPLIT;
    constexpr uint32_t kStride = 32 * SPLIT;  // blocks between a lane's consecutive blocks
    constexpr uint32_t kTrip = kStride * UNROLL;
    const uint32_t warp = threadIdx.x >> 5;
    const uint32_t lane = threadIdx.x & 31;
    const uint32_t part = warp % SPLIT;
    const uint32_t slot = warp / SPLIT;
    const uint32_t first = part * 32 + lane;
    const uint32_t blocks = p.blocks;
    const uint32_t groups = (p.count + COLS - 1) / COLS;
    const size_t column_bytes = static_cast<size_t>(blocks) * 16;

    uint4 w[UNROLL][COLS];
    uint16_t s[UNROLL][COLS];
    auto load_trip = [&](uint32_t group, uint32_t b) {
        const uint32_t j0 = group * COLS;
        const uint32_t valid = min(static_cast<uint32_t>(COLS), p.count - j0);
        const uint8_t *wp = p.nibbles + static_cast<size_t>(p.col0 + j0) * column_bytes + static_cast<size_t>(b) * 16;
        const uint16_t *sp = p.scales + static_cast<size_t>(p.col0 + j0) * p.scale_stride + b;
        if (valid == static_cast<uint32_t>(COLS) && b + kStride * (UNROLL - 1) < blocks) {
#pragma unroll
            for (int u = 0; u < UNROLL; ++u) {
#pragma unroll
                for (int c = 0; c < COLS; ++c) {
                    w[u][c] = load_stream_u4(wp + c * column_bytes + static_cast<size_t>(u) * kStride * 16);
                    s[u][c] = __ldg(sp + static_cast<size_t>(c) * p.scale_stride + u * kStride);
                }
            }
            return;
        }
#pragma unroll
        for (int u = 0; u < UNROLL; ++u) {
#pragma unroll
            for (int c = 0; c < COLS; ++c) {
                if (b + u * kStride < blocks && static_cast<uint32_t>(c) < valid) {
                    w[u][c] = load_stream_u4(wp + c * column_bytes + static_cast<size_t>(u) * kStride * 16);
                    s[u][c] = __ldg(sp + static_cast<size_t>(c) * p.scale_stride + u * kStride);
                } else {
                    w[u][c] = make_uint4(0, 0, 0, 0);
                    s[u][c] = 0;
                }
            }
        }
    };

    uint32_t group = blockIdx.x * kSlots + slot;
    if (group < groups) load_trip(group, first);
    // Programmatic dependent launch: the kernel may start while the previous kernel on the
    // stream drains. The prepared weights are immutable once prepare has returned, so the first
    // trip above is issued before the wait; the activation may be the previous kernel's output
    // and is read only after it. Every CTA of this grid is resident (persistent grid), so the
    // next kernel may be scheduled into the SMs' free slots right away.
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const StagedActivation staged = staged_activation(smem, ROWS * blocks);
    stage_activation<F32>(p.view, staged, threadIdx.x, blockDim.x);
    __syncthreads();

    for (; group < groups; group += gridDim.x * kSlots) {
        const uint32_t j0 = group * COLS;
        const uint32_t valid = min(static_cast<uint32_t>(COLS), p.count - j0);
        float acc[ROWS][COLS];
#pragma unroll
        for (int r = 0; r < ROWS; ++r) {
#pragma unroll
            for (int c = 0; c < COLS; ++c) acc[r][c] = 0.0f;
        }
        for (uint32_t b = first; b < blocks; b += kTrip) {
            if (b != first) load_trip(group, b);
#pragma unroll
            for (int u = 0; u < UNROLL; ++u) {
                if (b + u * kStride < blocks) {
                    float dw[COLS];
#pragma unroll
                    for (int c = 0; c < COLS; ++c) dw[c] = __half2float(__ushort_as_half(s[u][c]));
                    accumulate_block<ROWS, COLS>(w[u], dw, b + u * kStride, blocks, staged, acc);
                }
            }
        }
        const uint32_t next = group + gridDim.x * kSlots;
        if (next < groups) load_trip(next, first);

        float sums[ROWS * COLS];
#pragma unroll
        for (int r = 0; r < ROWS; ++r) {
#pragma unroll
            for (int c = 0; c < COLS; ++c) sums[r * COLS + c] = acc[r][c];
        }
        warp_sum<ROWS * COLS>(sums);
        float mine = sums[0];  // lane r * COLS + c keeps output (r, c)
#pragma unroll
        for (int i = 1; i < ROWS * COLS; ++i)
            if (lane == static_cast<uint32_t>(i)) mine = sums[i];
        const uint32_t out_row = lane / COLS;
        const uint32_t out_col = lane % COLS;
        const bool writer = lane < static_cast<uint32_t>(ROWS * COLS) && out_col < valid;
        if constexpr (SPLIT > 1) {
            // The SPLIT warps of this slot run the same groups, so the named barrier is safe.
            if (lane < static_cast<uint32_t>(ROWS * COLS)) partial[warp][lane] = mine;
            asm volatile("bar.sync %0, %1;" ::"r"(1 + slot), "r"(32 * SPLIT) : "memory");
            if (part == 0 && writer) {
                float value = partial[slot * SPLIT][lane];
#pragma unroll
                for (int q = 1; q < SPLIT; ++q) value = __fadd_rn(value, partial[slot * SPLIT + q][lane]);
                p.destination[static_cast<size_t>(out_row) * p.destination_stride + p.out_col0 + j0 + out_col] = value;
            }
            asm volatile("bar.sync %0, %1;" ::"r"(1 + slot), "r"(32 * SPLIT) : "memory");
        } else if (writer) {
            p.destination[static_cast<size_t>(out_row) * p.destination_stride + p.out_col0 + j0 + out_col] = mine;
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
    const StagedActivation staged = staged_activation(smem, ROWS * p.blocks);
    stage_activation<false>(p.view, staged, threadIdx.x, blockDim.x);
    __syncthreads();
    const uint32_t lane = threadIdx.x & 31;
    for (uint32_t j = blockIdx.x * kNativeWarps + (threadIdx.x >> 5); j < p.count; j += gridDim.x * kNativeWarps) {
        const size_t column = p.col0 + j;
        float acc[ROWS][1];
#pragma unroll
        for (int r = 0; r < ROWS; ++r) acc[r][0] = 0.0f;
        for (uint32_t b = lane; b < p.blocks; b += 32) {
            // Native 18-byte blocks are 2-byte aligned: nine 16-bit loads.
            const uint16_t *src = reinterpret_cast<const uint16_t *>(p.weight + (column * p.blocks + b) * 18);
            uint4 w[1];
            w[0].x = static_cast<uint32_t>(src[1]) | (static_cast<uint32_t>(src[2]) << 16);
            w[0].y = static_cast<uint32_t>(src[3]) | (static_cast<uint32_t>(src[4]) << 16);
            w[0].z = static_cast<uint32_t>(src[5]) | (static_cast<uint32_t>(src[6]) << 16);
            w[0].w = static_cast<uint32_t>(src[7]) | (static_cast<uint32_t>(src[8]) << 16);
            const float dw[1] = {__half2float(__ushort_as_half(src[0]))};
            accumulate_block<ROWS, 1>(w, dw, b, p.blocks, staged, acc);
        }
        float sums[ROWS];
#pragma unroll
        for (int r = 0; r < ROWS; ++r) sums[r] = acc[r][0];
        warp_sum<ROWS>(sums);
        float mine = sums[0];
#pragma unroll
        for (int r = 1; r < ROWS; ++r)
            if (lane == static_cast<uint32_t>(r)) mine = sums[r];
        if (lane < static_cast<uint32_t>(ROWS)) p.destination[static_cast<size_t>(lane) * p.destination_stride + p.out_col0 + j] = mine;
    }
}

template <int ROWS, int SPLIT, int COLS, int UNROLL, int MIN_BLOCKS, bool F32>
cudaError_t launch_direct(const DirectParams &p, int sm_count, cudaStream_t stream) {
    const size_t smem = activation_bytes(ROWS, p.blocks);
    if (smem > kSmemBudget) return cudaErrorInvalidValue;
    auto kernel = q4_0_direct_kernel<ROWS, SPLIT, COLS, UNROLL, MIN_BLOCKS, F32>;
    if (smem > 48u * 1024u) {
        const cudaError_t error =
            cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (error != cudaSuccess) return error;
    }
    // Persistent CTAs filling the SM's real residency (each stages the activation once); the
    // grid is balanced so every group slot runs the same number of rounds (no straggling tail).
    int per_sm = 0;
    const cudaError_t error = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kThreads, smem);
    if (error != cudaSuccess) return error;
    if (per_sm < 1) per_sm = 1;
    constexpr uint32_t kSlots = kWarps / SPLIT;
    const uint64_t groups = (static_cast<uint64_t>(p.count) + COLS - 1) / COLS;
    const uint64_t capacity = static_cast<uint64_t>(sm_count) * static_cast<uint64_t>(per_sm);
    const uint64_t rounds = (groups + capacity * kSlots - 1) / (capacity * kSlots);
    const uint32_t grid = static_cast<uint32_t>((groups + kSlots * rounds - 1) / (kSlots * rounds));
    cudaLaunchAttribute attribute{};
    attribute.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attribute.val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t config{};
    config.gridDim = dim3(grid);
    config.blockDim = dim3(kThreads);
    config.dynamicSmemBytes = smem;
    config.stream = stream;
    config.attrs = &attribute;
    config.numAttrs = 1;
    return cudaLaunchKernelEx(&config, kernel, p);
}

template <int ROWS, bool F32 = false>
cudaError_t launch_rows(const DirectParams &p, int sm_count, cudaStream_t stream) {
    // Two columns per warp halve the shared-memory reads per weight byte. One row: four blocks
    // of each column in flight per lane within 80 registers (3 CTAs per SM). Two rows: two
    // blocks at the same budget. Three or four rows are closer to issue-bound and keep four
    // blocks in flight at 128 registers (2 CTAs per SM), which measured faster than either
    // more CTAs or more columns per warp.
    // Long single-row reductions (>= 640 blocks, e.g. the 70B down projection with 896) are
    // split over 4 warps with seven blocks per lane and column in one trip: four times the
    // independent groups of the unsplit kernel, so the grid fills the SMs even when the matrix
    // is narrow (a column shard), and 14 loads in flight per lane within 128 registers.
    if constexpr (ROWS == 1) {
        if (p.blocks >= 640) return launch_direct<ROWS, 4, 2, 7, 2, F32>(p, sm_count, stream);
        return launch_direct<ROWS, 1, 2, 4, 3, F32>(p, sm_count, stream);
    } else if constexpr (ROWS == 2) {
        return launch_direct<ROWS, 1, 2, 2, 3, F32>(p, sm_count, stream);
    } else {
        return launch_direct<ROWS, 1, 2, 4, 2, F32>(p, sm_count, stream);
    }
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
    p.view = ActivationView{activation, rows, weights.blocks, interleave, nullptr, 0};
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

cudaError_t launch_q4_0_f32_gemv(const Q40Weights &weights, const float *source, size_t source_stride, uint32_t rows,
                                 float *destination, size_t destination_stride, uint32_t col0, uint32_t out_col0,
                                 uint32_t count, int sm_count, cudaStream_t stream) {
    if (count == 0 || rows == 0) return cudaSuccess;
    if ((reinterpret_cast<uintptr_t>(weights.nibbles) & 15u) != 0 || (reinterpret_cast<uintptr_t>(weights.scales) & 15u) != 0 ||
        (reinterpret_cast<uintptr_t>(source) & 3u) != 0 || weights.scale_stride % 8 != 0 ||
        weights.scale_stride < weights.blocks || source_stride < static_cast<size_t>(weights.blocks) * 32) {
        return cudaErrorInvalidValue;
    }
    DirectParams p{};
    p.nibbles = weights.nibbles;
    p.scales = weights.scales;
    p.blocks = weights.blocks;
    p.scale_stride = weights.scale_stride;
    p.view = ActivationView{nullptr, rows, weights.blocks, 0, source, source_stride};
    p.destination = destination;
    p.destination_stride = destination_stride;
    p.col0 = col0;
    p.out_col0 = out_col0;
    p.count = count;
    switch (rows) {
        case 1: return launch_rows<1, true>(p, sm_count, stream);
        case 2: return launch_rows<2, true>(p, sm_count, stream);
        case 3: return launch_rows<3, true>(p, sm_count, stream);
        case 4: return launch_rows<4, true>(p, sm_count, stream);
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
    const NativeParams p{weight, blocks, ActivationView{activation, rows, blocks, 0, nullptr, 0}, destination,
                         destination_stride, col0, out_col0, count};
    switch (rows) {
        case 1: return launch_native<1>(p, sm_count, stream);
        case 2: return launch_native<2>(p, sm_count, stream);
        case 3: return launch_native<3>(p, sm_count, stream);
        case 4: return launch_native<4>(p, sm_count, stream);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace qpucuda
