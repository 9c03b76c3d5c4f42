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
// Kernels:
//  * q4_0_direct_kernel (prepared weights, the operator's path). Prepared layout,
//    made once at prepare with the same 18 bytes per block as the native format:
//    nibbles [columns][blocks][16] and fp16 scales [columns][scale_stride]
//    (scale_stride = blocks rounded up to 8). A warp owns two adjacent columns; lane l
//    takes blocks l, l + 32, ..., so a warp reads 512 contiguous bytes of each column per
//    16-byte load, with eight such loads in flight per lane; persistent CTAs sized from the
//    occupancy API with a balanced number of rounds.
//  * q4_0_native_kernel (single-kernel entry point over native 18-byte blocks,
//    which are only 2-byte aligned): lanes read each block as nine 16-bit loads.
//  * q4_0_mx_kernel (rows > 4, the reference's MX path): int8 tensor-core MMAs per
//    32-value block with the exact per-block scaling of the reference program (see below).
// The two matvec kernels keep the weight codes packed: dp4a(nibbles & 0x0F0F0F0F, a[0..3]) and
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

constexpr int kFloatMagic = 0x4B400000;  // bits of 1.5 * 2^23 = 12582912.0f

// Packed fp32 pairs (sm_100 add/mul .f32x2): each lane rounds to nearest exactly as
// __fadd_rn / __fmul_rn, two values per instruction.
__device__ __forceinline__ unsigned long long pack2(float lo, float hi) {
    return static_cast<unsigned long long>(__float_as_uint(lo)) | (static_cast<unsigned long long>(__float_as_uint(hi)) << 32);
}
__device__ __forceinline__ unsigned long long add2(unsigned long long a, unsigned long long b) {
    unsigned long long d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ unsigned long long mul2(unsigned long long a, unsigned long long b) {
    unsigned long long d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}

__device__ __forceinline__ void write_activation_item(const StagedActivation &staged, uint32_t item,
                                                      const uint32_t (&words)[8], uint16_t scale_bits) {
    int sum = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) sum = __dp4a(static_cast<int>(words[i]), 0x01010101, sum);
    staged.lo[item] = make_int4(words[0], words[1], words[2], words[3]);
    staged.hi[item] = make_int4(words[4], words[5], words[6], words[7]);
    // The dp4a seed also carries the float magic, so a block's dot comes out as the bits of
    // 1.5 * 2^23 + dot (|dot| <= 32 * 127 * 8 < 2^22): one exact subtraction gives (float)dot.
    staged.meta[item] = make_int2(__float_as_int(__half2float(__ushort_as_half(scale_bits))), kFloatMagic - 8 * sum);
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
// each block term (ggml_q4_0.py:81-100). (float)dot is exact (the magic in the seed, one
// subtraction), the two products of a column pair share packed multiplies, and the accumulate
// stays a scalar __fadd_rn so nothing can be contracted into a fused multiply-add.
template <int ROWS, int COLS>
__device__ __forceinline__ void accumulate_block(const uint4 (&w)[COLS], const float (&dw)[COLS], uint32_t item,
                                                 uint32_t blocks, const StagedActivation &staged,
                                                 float (&acc)[ROWS][COLS]) {
    const unsigned long long unbias = pack2(-12582912.0f, -12582912.0f);
#pragma unroll
    for (int r = 0; r < ROWS; ++r) {
        const uint32_t at = static_cast<uint32_t>(r) * blocks + item;
        const int4 lo = staged.lo[at];
        const int4 hi = staged.hi[at];
        const int2 meta = staged.meta[at];
        const float da = __int_as_float(meta.x);
        const unsigned long long da2 = pack2(da, da);
#pragma unroll
        for (int c = 0; c + 1 < COLS; c += 2) {
            const int bits0 = block_dot(w[c], lo, hi, meta.y);
            const int bits1 = block_dot(w[c + 1], lo, hi, meta.y);
            unsigned long long v = add2(pack2(__int_as_float(bits0), __int_as_float(bits1)), unbias);
            v = mul2(v, pack2(dw[c], dw[c + 1]));
            v = mul2(v, da2);
            acc[r][c] = __fadd_rn(acc[r][c], __uint_as_float(static_cast<uint32_t>(v)));
            acc[r][c + 1] = __fadd_rn(acc[r][c + 1], __uint_as_float(static_cast<uint32_t>(v >> 32)));
        }
        if constexpr (COLS % 2 == 1) {
            const float x = __fadd_rn(__int_as_float(block_dot(w[COLS - 1], lo, hi, meta.y)), -12582912.0f);
            acc[r][COLS - 1] = __fadd_rn(acc[r][COLS - 1], __fmul_rn(__fmul_rn(x, dw[COLS - 1]), da));
        }
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
// thread are capped so that MIN_BLOCKS CTAs of 256 threads fit on an SM. With PIPE, a trip's
// weights are copied and the next trip's loads (or the next group's first) are issued before
// the trip is computed, so a warp's loads stay in flight during its own arithmetic (the
// several-row kernels, whose arithmetic per byte is several times the single row's).
template <int ROWS, int SPLIT, int COLS, int UNROLL, int MIN_BLOCKS, bool F32, bool PIPE = false>
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
        const uint32_t next = group + gridDim.x * kSlots;
        for (uint32_t b = first; b < blocks; b += kTrip) {
            uint4 wc[UNROLL][COLS];
            uint16_t sc[UNROLL][COLS];
            if constexpr (PIPE) {
#pragma unroll
                for (int u = 0; u < UNROLL; ++u) {
#pragma unroll
                    for (int c = 0; c < COLS; ++c) {
                        wc[u][c] = w[u][c];
                        sc[u][c] = s[u][c];
                    }
                }
                if (b + kTrip < blocks) {
                    load_trip(group, b + kTrip);
                } else if (next < groups) {
                    load_trip(next, first);
                }
            } else if (b != first) {
                load_trip(group, b);
            }
            const auto &wt = PIPE ? wc : w;
            const auto &st = PIPE ? sc : s;
#pragma unroll
            for (int u = 0; u < UNROLL; ++u) {
                if (b + u * kStride < blocks) {
                    float dw[COLS];
#pragma unroll
                    for (int c = 0; c < COLS; ++c) dw[c] = __half2float(__ushort_as_half(st[u][c]));
                    accumulate_block<ROWS, COLS>(wt[u], dw, b + u * kStride, blocks, staged, acc);
                }
            }
        }
        if (!PIPE && next < groups) load_trip(next, first);

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

template <int ROWS, int SPLIT, int COLS, int UNROLL, int MIN_BLOCKS, bool F32, bool PIPE = false>
cudaError_t launch_direct(const DirectParams &p, int sm_count, cudaStream_t stream) {
    const size_t smem = activation_bytes(ROWS, p.blocks);
    if (smem > kSmemBudget) return cudaErrorInvalidValue;
    auto kernel = q4_0_direct_kernel<ROWS, SPLIT, COLS, UNROLL, MIN_BLOCKS, F32, PIPE>;
    if (smem > 48u * 1024u) {
        const cudaError_t error =
            cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (error != cudaSuccess) return error;
    }
    // Persistent CTAs filling every resident slot of every SM (each stages the activation once),
    // so each SM carries the same share of the column groups. A grid trimmed so that every CTA ran
    // the same number of rounds left SMs with one CTA beside SMs with two (M = 4 on the 70B gate:
    // 256 CTAs for 296 slots) and measured slower: decode FFN at M = 4 126.0 against 119.9 us.
    int per_sm = 0;
    const cudaError_t error = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kThreads, smem);
    if (error != cudaSuccess) return error;
    if (per_sm < 1) per_sm = 1;
    constexpr uint32_t kSlots = kWarps / SPLIT;
    const uint64_t groups = (static_cast<uint64_t>(p.count) + COLS - 1) / COLS;
    const uint64_t capacity = static_cast<uint64_t>(sm_count) * static_cast<uint64_t>(per_sm);
    const uint64_t wanted = (groups + kSlots - 1) / kSlots;
    const uint32_t grid = static_cast<uint32_t>(wanted < capacity ? wanted : capacity);
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
    // Two rows, and four rows over long reductions, overlap each warp's next loads with its
    // arithmetic (PIPE); measured on B200 with L2 flushed (70B FFN shapes): two rows
    // 34.8 -> 32.8 us (K = 8192) and 41.0 -> 34.8 us (K = 28672), four rows at K = 28672
    // 59.4 -> 51.2 us; four rows at K = 8192 and the single row gained nothing from it, and three
    // rows at K = 28672 lost (45.1 -> 49.2 us).
    // A small matrix (a few MB, so one launch is mostly latency) whose reduction needs more than
    // one four-block trip: six blocks per lane and column take each warp's whole group in one
    // trip, loaded before the dependency wait. Measured on B200 (TinyLlama down 5632 -> 2048,
    // 16 weight copies back to back, L2 flushed): 4.03 -> 3.13 us per launch at M = 1 and
    // 6.08 -> 5.62 us at M = 4. Four columns per warp for the 64-block up projection measured
    // the same at M = 1 and slower at M = 4 (5.04 against 4.80 us), so it is not used.
    const uint64_t weight_bytes = static_cast<uint64_t>(p.count) * p.blocks * 18u;
    if (weight_bytes <= (16u << 20) && p.blocks > 128 && p.blocks <= 192) {
        return launch_direct<ROWS, 1, 2, 6, 2, F32>(p, sm_count, stream);
    }
    // One row over 193-512 blocks: eight blocks per lane and column per trip (two trips instead
    // of three for the 7B down projection's 344, one instead of two for the 70B gate's 256):
    // decode FFN at M = 1 25.6 -> 23.6 us on the 7B shapes, 74.8 -> 72.8 us on the 70B shapes.
    // At M = 4 the same measured slower (7B: 39.9 against 38.0 us) and is not used.
    if constexpr (ROWS == 1) {
        if (p.blocks > 192 && p.blocks <= 512) return launch_direct<ROWS, 1, 2, 8, 2, F32>(p, sm_count, stream);
        if (p.blocks >= 640) return launch_direct<ROWS, 4, 2, 7, 2, F32>(p, sm_count, stream);
        return launch_direct<ROWS, 1, 2, 4, 3, F32>(p, sm_count, stream);
    } else if constexpr (ROWS == 2) {
        return launch_direct<ROWS, 1, 2, 2, 2, F32, true>(p, sm_count, stream);
    } else {
        if (ROWS == 4 && p.blocks >= 640) return launch_direct<ROWS, 1, 2, 4, 2, F32, true>(p, sm_count, stream);
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

// ---- MX path: rows > 4 on the tensor cores -------------------------------------------------
//
// The reference's tiled Q4_0 x Q8_0 program (src/qpu_xla/kernels/ggml_q4_0.py:310-547, prepared
// by qpu_llama_q4_0.c:238-290 for rows > 4, EXACT weight mode) computes, for every output, one
// fp32 accumulator over the blocks in order: acc += ((float)dot_b * d_a[m, b]) * d_w[n, b]
// (itof, fmul by the activation scale, fmul by the weight scale, fadd; :506-513). Here each
// block's exact int32 dots come from mma.sync m16n8k32 (s8 x s8 -> s32) with a fresh accumulator
// per block, and each thread applies those three roundings and the add to the outputs it owns,
// in block order, so the result follows the reference program's arithmetic exactly.
//
// GGML's nibble order is already the m16n8k32 B-fragment order: word t of a block holds codes
// 4t..4t+3 in its low nibbles and 16+4t.. in its high nibbles, which are exactly the two B
// registers of the lane with threadID_in_group t. The codes enter the MMA as unsigned 0..15;
// the -8 offset is removed by subtracting 8 * sum(q) of the activation block.
//
// Activation (split once per call by q4_0_mx_split_kernel, rows and blocks zero-padded):
//   q    int8 [rows_pad][blocks_pad * 32]
//   meta int2 [rows_pad][blocks_pad]   {fp32 bits of d_a, 8 * sum of the block's 32 values}
constexpr int kMxKB = 4;        // Q4_0 blocks per pipeline stage (128 bytes of K)
constexpr int kMxThreads = 256; // 8 warps
constexpr int kMxRowAlign = 64; // the split activation is padded to the largest row tile
constexpr int kMxAPitch = 144;  // bytes per staged activation row (128 + 16: conflict-free fragments)
constexpr int kMxBPitch = 80;   // bytes per staged weight column (64 + 16)
// BM rows x BN columns per CTA. Small row counts take narrow column tiles so that a narrow
// matrix still gives every SM work (each output's block sum stays in one thread, in order, so
// K is never split), and deeper pipelines since their stages are small.
template <int BM>
struct MxTile {
    static constexpr int kBN = BM >= 64 ? 128 : 64;
    static constexpr int kStages = BM >= 64 ? 4 : 6;
    static constexpr int kWarpsM = BM >= 64 ? 2 : 1;             // warps along rows
    static constexpr int kWarpsN = 8 / kWarpsM;                  // warps along columns
    static constexpr int kM16 = BM / kWarpsM / 16;               // m16 tiles per warp
    static constexpr int kN8 = kBN / kWarpsN / 8;                // n8 tiles per warp
    static constexpr int kStageA = BM * kMxAPitch;
    static constexpr int kStageMeta = BM * kMxKB * 8;
    static constexpr int kStageB = kBN * kMxBPitch;
    static constexpr int kStageScale = kBN * kMxKB * 2;
    static constexpr int kStageBytes = kStageA + kStageMeta + kStageB + kStageScale;
    static constexpr int kSmemBytes = kStages * kStageBytes;
};

uint32_t mx_rows_pad(uint32_t rows) { return (rows + kMxRowAlign - 1) / kMxRowAlign * kMxRowAlign; }
uint32_t mx_blocks_pad(uint32_t blocks) { return (blocks + kMxKB - 1) / kMxKB * kMxKB; }

struct MxSplitParams {
    ActivationView view;  // Q8_0 blocks, or fp32 rows when view.f32 is set
    uint32_t rows_pad, blocks_pad;
    int8_t *q;
    int2 *meta;
    float *da_t;  // tcgen05 path: the block scales again, block-major [blocks_pad][rows_pad]; or null
};

// One thread per (row, block) of the padded split activation; padding is written as zeros.
__global__ void __launch_bounds__(256) q4_0_mx_split_kernel(const MxSplitParams p) {
    const uint64_t total = static_cast<uint64_t>(p.rows_pad) * p.blocks_pad;
    const bool vector = p.view.f32 != nullptr && (reinterpret_cast<uintptr_t>(p.view.f32) & 15u) == 0 &&
                        (p.view.f32_stride & 3u) == 0;
    for (uint64_t item = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; item < total;
         item += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        const uint32_t row = static_cast<uint32_t>(item / p.blocks_pad);
        const uint32_t block = static_cast<uint32_t>(item % p.blocks_pad);
        uint32_t words[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        float d = 0.0f;
        int sum = 0;
        if (row < p.view.rows && block < p.view.blocks) {
            uint16_t scale_bits;
            if (p.view.f32 != nullptr) {
                quantize_f32_block(p.view.f32 + static_cast<size_t>(row) * p.view.f32_stride + static_cast<size_t>(block) * 32,
                                   vector, words, scale_bits);
            } else {
                read_activation_item(p.view, row * p.view.blocks + block, words, scale_bits);
            }
            d = __half2float(__ushort_as_half(scale_bits));
#pragma unroll
            for (int i = 0; i < 8; ++i) sum = __dp4a(static_cast<int>(words[i]), 0x01010101, sum);
        }
        uint4 *q = reinterpret_cast<uint4 *>(p.q + (static_cast<size_t>(row) * p.blocks_pad + block) * 32);
        q[0] = make_uint4(words[0], words[1], words[2], words[3]);
        q[1] = make_uint4(words[4], words[5], words[6], words[7]);
        p.meta[static_cast<size_t>(row) * p.blocks_pad + block] = make_int2(__float_as_int(d), 8 * sum);
        if (p.da_t != nullptr) p.da_t[static_cast<size_t>(block) * p.rows_pad + row] = d;
    }
}

struct MxParams {
    const int8_t *q;
    const int2 *meta;
    uint32_t rows, blocks_pad;
    const uint8_t *nibbles;
    const uint16_t *scales;
    uint32_t blocks, scale_stride;
    uint32_t col0, out_col0, count;
    float *destination;
    size_t destination_stride;
};

__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src, uint32_t bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ void cp_async8(uint32_t dst, const void *src, uint32_t bytes) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(dst), "l"(src), "r"(bytes) : "memory");
}

// d = a . b + c (s32). c carries 0x4B400000 - 8 * sum(q) for the row: the MMA then returns the
// bit pattern of the float 1.5 * 2^23 + dot, where dot = sum (code - 8) * q is the block's exact
// integer dot (|dot| < 2^22, so that float is exact with a unit ulp), and one subtraction of
// 1.5 * 2^23 yields (float)dot exactly.
__device__ __forceinline__ void mma_s8(const uint32_t (&a)[4], uint32_t b0, uint32_t b1, int c_lo, int c_hi, int (&d)[4]) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%10, %10, %11, %11};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(c_lo), "r"(c_hi));
}

// BM rows x BN columns per CTA, 8 warps tiled over it (MxTile), kStages stages of 4 blocks.
template <int BM>
__global__ void __launch_bounds__(kMxThreads) q4_0_mx_kernel(const MxParams p) {
    using Tile = MxTile<BM>;
    extern __shared__ __align__(128) uint8_t smem[];
    const uint32_t tid = threadIdx.x;
    const uint32_t warp = tid >> 5, lane = tid & 31;
    const uint32_t group = lane >> 2, tig = lane & 3;
    const uint32_t warp_m = warp / Tile::kWarpsN, warp_n = warp % Tile::kWarpsN;
    const uint32_t warp_row0 = warp_m * (BM / Tile::kWarpsM);
    const uint32_t warp_col0 = warp_n * (Tile::kBN / Tile::kWarpsN);
    const uint32_t m0 = blockIdx.y * BM;
    const uint32_t n0 = blockIdx.x * Tile::kBN;
    const uint32_t chunks = p.blocks_pad / kMxKB;
    const uint32_t k_bytes = p.blocks_pad * 32;

    auto load_stage = [&](uint32_t s, uint32_t chunk) {
        const uint32_t a_smem = static_cast<uint32_t>(__cvta_generic_to_shared(smem + s * Tile::kStageBytes));
        // activation: BM rows x 128 bytes (in bounds: the split buffer is padded to 64 rows)
        for (uint32_t i = tid; i < BM * 8; i += kMxThreads) {
            const uint32_t row = i >> 3, seg = i & 7;
            cp_async16(a_smem + row * kMxAPitch + seg * 16,
                       p.q + static_cast<size_t>(m0 + row) * k_bytes + chunk * 128 + seg * 16, 16);
        }
        const uint32_t meta_smem = a_smem + Tile::kStageA;
        for (uint32_t i = tid; i < BM * 2; i += kMxThreads) {
            const uint32_t row = i >> 1, half = i & 1;
            cp_async16(meta_smem + row * 32 + half * 16,
                       p.meta + static_cast<size_t>(m0 + row) * p.blocks_pad + chunk * kMxKB + half * 2, 16);
        }
        // weights: 128 columns x 4 blocks of 16 bytes; columns or blocks past the end are zero-filled
        const uint32_t b_smem = meta_smem + Tile::kStageMeta;
        for (uint32_t i = tid; i < Tile::kBN * kMxKB; i += kMxThreads) {
            const uint32_t col = i >> 2, blk = i & 3;
            const uint32_t block = chunk * kMxKB + blk;
            const bool valid = n0 + col < p.count && block < p.blocks;
            const uint8_t *src = valid ? p.nibbles + (static_cast<size_t>(p.col0 + n0 + col) * p.blocks + block) * 16 : p.nibbles;
            cp_async16(b_smem + col * kMxBPitch + blk * 16, src, valid ? 16u : 0u);
        }
        const uint32_t scale_smem = b_smem + Tile::kStageB;
        for (uint32_t col = tid; col < Tile::kBN; col += kMxThreads) {
            const bool valid = n0 + col < p.count;
            const uint16_t *src = valid ? p.scales + static_cast<size_t>(p.col0 + n0 + col) * p.scale_stride + chunk * kMxKB : p.scales;
            cp_async8(scale_smem + col * 8, src, valid ? 8u : 0u);
        }
    };

    // acc[mt][nt][h]: the thread's two adjacent columns of row group (h = 0) or group + 8 (h = 1).
    unsigned long long acc[Tile::kM16][Tile::kN8][2];
#pragma unroll
    for (int mt = 0; mt < Tile::kM16; ++mt)
#pragma unroll
        for (int nt = 0; nt < Tile::kN8; ++nt) acc[mt][nt][0] = acc[mt][nt][1] = 0ull;

    // Tile::kStages - 1 chunks in flight ahead of the one being computed. Every iteration commits one
    // group (empty past the end) so that wait_group counts stay uniform.
#pragma unroll
    for (int s = 0; s < Tile::kStages - 1; ++s) {
        if (static_cast<uint32_t>(s) < chunks) load_stage(s, s);
        asm volatile("cp.async.commit_group;" ::: "memory");
    }
    for (uint32_t chunk = 0; chunk < chunks; ++chunk) {
        asm volatile("cp.async.wait_group %0;" ::"n"(Tile::kStages - 2) : "memory");
        __syncthreads();  // chunk's stage is complete for all threads; the stage loaded next was computed last iteration
        const uint32_t next = chunk + Tile::kStages - 1;
        if (next < chunks) load_stage(next % Tile::kStages, next);
        asm volatile("cp.async.commit_group;" ::: "memory");

        const uint8_t *base = smem + (chunk % Tile::kStages) * Tile::kStageBytes;
        const uint8_t *stage_a = base;
        const int2 *stage_meta = reinterpret_cast<const int2 *>(base + Tile::kStageA);
        const uint8_t *stage_b = base + Tile::kStageA + Tile::kStageMeta;
        const uint16_t *stage_scale = reinterpret_cast<const uint16_t *>(stage_b + Tile::kStageB);
        const uint32_t valid_blocks = min(static_cast<uint32_t>(kMxKB), p.blocks - chunk * kMxKB);
        for (uint32_t bb = 0; bb < valid_blocks; ++bb) {
            uint32_t b[Tile::kN8][2];
            unsigned long long dw[Tile::kN8];  // weight scales of the thread's two output columns
#pragma unroll
            for (int nt = 0; nt < Tile::kN8; ++nt) {
                const uint32_t col = warp_col0 + nt * 8 + group;
                const uint32_t w = *reinterpret_cast<const uint32_t *>(stage_b + col * kMxBPitch + bb * 16 + tig * 4);
                b[nt][0] = w & 0x0F0F0F0Fu;
                b[nt][1] = (w >> 4) & 0x0F0F0F0Fu;
                const uint32_t out_col = warp_col0 + nt * 8 + tig * 2;
                dw[nt] = pack2(__half2float(__ushort_as_half(stage_scale[out_col * kMxKB + bb])),
                               __half2float(__ushort_as_half(stage_scale[(out_col + 1) * kMxKB + bb])));
            }
#pragma unroll
            for (int mt = 0; mt < Tile::kM16; ++mt) {
                const uint32_t row_lo = warp_row0 + mt * 16 + group;
                const uint8_t *a_lo = stage_a + row_lo * kMxAPitch + bb * 32 + tig * 4;
                const uint8_t *a_hi = a_lo + 8 * kMxAPitch;
                const uint32_t a[4] = {*reinterpret_cast<const uint32_t *>(a_lo), *reinterpret_cast<const uint32_t *>(a_hi),
                                       *reinterpret_cast<const uint32_t *>(a_lo + 16), *reinterpret_cast<const uint32_t *>(a_hi + 16)};
                const int2 meta_lo = stage_meta[row_lo * kMxKB + bb];
                const int2 meta_hi = stage_meta[(row_lo + 8) * kMxKB + bb];
                const unsigned long long da[2] = {pack2(__int_as_float(meta_lo.x), __int_as_float(meta_lo.x)),
                                                  pack2(__int_as_float(meta_hi.x), __int_as_float(meta_hi.x))};
                const unsigned long long unbias = pack2(-12582912.0f, -12582912.0f);
#pragma unroll
                for (int nt = 0; nt < Tile::kN8; ++nt) {
                    int d[4];
                    mma_s8(a, b[nt][0], b[nt][1], kFloatMagic - meta_lo.y, kFloatMagic - meta_hi.y, d);
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        // ((float)dot * d_a) * d_w, then the add: the reference program's roundings.
                        unsigned long long v = add2(pack2(__int_as_float(d[2 * h]), __int_as_float(d[2 * h + 1])), unbias);
                        v = mul2(v, da[h]);
                        v = mul2(v, dw[nt]);
                        // The accumulate stays scalar: a packed add after a packed multiply may be
                        // contracted into a fused multiply-add, which would drop the product's rounding.
                        const unsigned long long a_pair = acc[mt][nt][h];
                        acc[mt][nt][h] = pack2(__fadd_rn(__uint_as_float(static_cast<uint32_t>(a_pair)), __uint_as_float(static_cast<uint32_t>(v))),
                                               __fadd_rn(__uint_as_float(static_cast<uint32_t>(a_pair >> 32)), __uint_as_float(static_cast<uint32_t>(v >> 32))));
                    }
                }
            }
        }
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");

#pragma unroll
    for (int mt = 0; mt < Tile::kM16; ++mt) {
#pragma unroll
        for (int nt = 0; nt < Tile::kN8; ++nt) {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint32_t row = m0 + warp_row0 + mt * 16 + group + (i < 2 ? 0 : 8);
                const uint32_t col = n0 + warp_col0 + nt * 8 + tig * 2 + (i & 1);
                const unsigned long long pair = acc[mt][nt][i >> 1];
                const float value = __uint_as_float(static_cast<uint32_t>((i & 1) ? pair >> 32 : pair));
                if (row < p.rows && col < p.count)
                    p.destination[static_cast<size_t>(row) * p.destination_stride + p.out_col0 + col] = value;
            }
        }
    }
}

template <int BM>
cudaError_t launch_mx_tiles(const MxParams &p, uint32_t rows_pad, uint32_t count, cudaStream_t stream) {
    static PerDeviceOnce configured;
    const cudaError_t error = configured.run([] {
        return cudaFuncSetAttribute(q4_0_mx_kernel<BM>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    MxTile<BM>::kSmemBytes);
    });
    if (error != cudaSuccess) return error;
    const dim3 grid((count + MxTile<BM>::kBN - 1) / MxTile<BM>::kBN, (p.rows + BM - 1) / BM);
    (void)rows_pad;
    q4_0_mx_kernel<BM><<<grid, kMxThreads, MxTile<BM>::kSmemBytes, stream>>>(p);
    return cudaGetLastError();
}

cudaError_t launch_mx(const Q40Weights &weights, const ActivationView &view, uint8_t *scratch, float *destination,
                      size_t destination_stride, uint32_t col0, uint32_t out_col0, uint32_t count,
                      unsigned int *error_word, int sm_count, cudaStream_t stream) {
    const uint32_t rows_pad = mx_rows_pad(view.rows);
    const uint32_t blocks_pad = mx_blocks_pad(weights.blocks);
    const size_t items_bytes = static_cast<size_t>(rows_pad) * blocks_pad;
    const bool tcgen05 = weights.mx_values != nullptr && weights.mx_scales_t != nullptr &&
                         q4_0_mx_sm100_fills_wave(view.rows, count, sm_count);
    MxSplitParams split{view, rows_pad, blocks_pad, reinterpret_cast<int8_t *>(scratch),
                        reinterpret_cast<int2 *>(scratch + items_bytes * 32),
                        tcgen05 ? reinterpret_cast<float *>(scratch + items_bytes * 40) : nullptr};
    const uint64_t items = static_cast<uint64_t>(rows_pad) * blocks_pad;
    const uint32_t split_grid = static_cast<uint32_t>(items / 256 + 1 < 148ull * 32ull ? items / 256 + 1 : 148ull * 32ull);
    q4_0_mx_split_kernel<<<split_grid, 256, 0, stream>>>(split);
    cudaError_t error = cudaGetLastError();
    if (error != cudaSuccess) return error;
    if (tcgen05) {
        return launch_q4_0_mx_sm100(split.q, split.da_t, view.rows, rows_pad, weights.mx_values, weights.mx_scales_t,
                                    weights.columns, weights.blocks, blocks_pad, destination, destination_stride, col0,
                                    out_col0, count, error_word, sm_count, stream);
    }
    MxParams p{};
    p.q = split.q;
    p.meta = split.meta;
    p.rows = view.rows;
    p.blocks_pad = blocks_pad;
    p.nibbles = weights.nibbles;
    p.scales = weights.scales;
    p.blocks = weights.blocks;
    p.scale_stride = weights.scale_stride;
    p.col0 = col0;
    p.out_col0 = out_col0;
    p.count = count;
    p.destination = destination;
    p.destination_stride = destination_stride;
    // Few rows: the smallest row tile that holds them (fewer padded rows computed, more CTAs);
    // 33..64 rows keep the wide 64 x 128 tiles only when those fill a wave of SMs.
    if (view.rows <= 16) return launch_mx_tiles<16>(p, rows_pad, count, stream);
    const uint64_t wide_ctas = static_cast<uint64_t>((count + MxTile<64>::kBN - 1) / MxTile<64>::kBN) * ((view.rows + 63) / 64);
    if (view.rows <= 32 || (view.rows <= 64 && wide_ctas < static_cast<uint64_t>(sm_count)))
        return launch_mx_tiles<32>(p, rows_pad, count, stream);
    return launch_mx_tiles<64>(p, rows_pad, count, stream);
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

// int8 rows (32 bytes per block), {d_a, 8 * sum} pairs (8), and the block-major d_a copy (4).
size_t q4_0_mx_scratch_bytes(uint32_t rows, uint32_t blocks) {
    return static_cast<size_t>(mx_rows_pad(rows)) * mx_blocks_pad(blocks) * (32 + 8 + 4);
}

uint32_t q4_0_mx_blocks_pad(uint32_t blocks) { return mx_blocks_pad(blocks); }

cudaError_t launch_q4_0_mx(const Q40Weights &weights, const uint8_t *activation, const float *f32_source,
                           size_t f32_stride, uint32_t rows, uint32_t interleave, uint8_t *scratch, float *destination,
                           size_t destination_stride, uint32_t col0, uint32_t out_col0, uint32_t count,
                           unsigned int *error_word, int sm_count, cudaStream_t stream) {
    if (count == 0 || rows == 0) return cudaSuccess;
    if ((reinterpret_cast<uintptr_t>(weights.nibbles) & 15u) != 0 || (reinterpret_cast<uintptr_t>(weights.scales) & 15u) != 0 ||
        (reinterpret_cast<uintptr_t>(scratch) & 15u) != 0 || weights.scale_stride % 8 != 0 ||
        weights.scale_stride < weights.blocks || (activation == nullptr) == (f32_source == nullptr) ||
        (activation != nullptr && (reinterpret_cast<uintptr_t>(activation) & 1u) != 0) ||
        (f32_source != nullptr && ((reinterpret_cast<uintptr_t>(f32_source) & 3u) != 0 ||
                                   f32_stride < static_cast<size_t>(weights.blocks) * 32))) {
        return cudaErrorInvalidValue;
    }
    const ActivationView view{activation, rows, weights.blocks, f32_source != nullptr ? 0u : interleave, f32_source,
                              f32_stride};
    return launch_mx(weights, view, scratch, destination, destination_stride, col0, out_col0, count, error_word, sm_count,
                     stream);
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
