// Small-M W8A8 kernels (HBM-bound on the weight).
//
//  * w8a8_gemv: acc[m, n] = sum_k a[m, k] * w[n, k] for m <= 8 rows, exact int32.
//    Replaces vc7.w8a8_gemv (src/qpu_xla/kernels/gemv_int8.py:20-153), which the
//    reference selects for batch == 1 (src/qpu_xla/models/tinyllama/quantization.py:184).
//    - One row (w8a8_gemv_kernel): one warp, or SPLIT warps of a CTA over disjoint K
//      ranges, per output column n; each lane streams 16-byte chunks of the weight row (a
//      warp reads 512 contiguous bytes per step) into dp4a, the warp reduces with shuffles
//      and split warps add through shared memory.
//    - Two to eight rows (w8a8_gemv_mma_kernel): mma.sync m16n8k32 over 16-column groups,
//      so the weight bytes are read once however many rows there are (dp4a would issue four
//      instructions per row per 16 bytes and re-read the activation chunks per row).
//    - One row with its quantization fused (w8a8_gemv_kernel<1, SPLIT, true>): every CTA
//      quantizes the fp32 row into shared memory itself (the row quantizer's arithmetic,
//      row_quantize.cuh) after streaming in its first weights, so no separate quantizer launch
//      sits between the previous kernel and the GEMV; CTA 0 also writes the int8 row and scale to
//      the plan scratch. Used for rows up to kFusedQuantMaxK columns (an L1-resident re-read).
//    Integer addition is associative, so the int32 result is exact in any order, and the
//    fused epilogue is the same ((float)acc * s_a) * s_w (+ bias) as the GEMM. The grids
//    are persistent, sized from the occupancy API with every CTA running the same number
//    of rounds.
//  * w8a8_dequantize: the standalone vc7.w8a8_dequantize epilogue
//    (src/qpu_xla/kernels/w8a8_epilogue.py:20-96), elementwise.
#include <atomic>

#include "qpucuda_internal.h"
#include "row_quantize.cuh"

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
    // One-row kernel that quantizes its own activation (QUANT): the fp32 row x[0 .. x_cols) and
    // where CTA 0 leaves the int8 row (k bytes, zero padded) and its scale.
    const float *x;
    uint32_t x_cols;
    int8_t *q_out;
    float *scale_out;
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

constexpr int kGemvThreads = 256;
constexpr int kGemvWarps = kGemvThreads / 32;

// SPLIT warps of a CTA share one output column, each over its own range of K (whole 32-chunk
// warp steps); their int32 partial sums meet in shared memory. Integer addition is
// associative, so any split gives the same exact accumulator. The grid is persistent and
// balanced (every column slot runs the same number of rounds), so no partial wave trails.
template <int ROWS, int SPLIT, bool QUANT = false>
__global__ void __launch_bounds__(kGemvThreads) w8a8_gemv_kernel(const GemvParams p) {
    static_assert(!QUANT || ROWS == 1, "the fused quantizer serves one row");
    __shared__ int partial[kGemvWarps][ROWS];
    extern __shared__ __align__(16) uint8_t quantized_row[];  // QUANT: the int8 row, p.k bytes
    constexpr uint32_t kSlots = kGemvWarps / SPLIT;
    // One or two rows are bound by the weight stream: each column's first trip is loaded during
    // the previous column's reduction. More rows are issue-bound and keep those registers for
    // occupancy instead. Measured on B200 (70B FFN shapes, L2 flushed, per call with the row
    // quantizer): M = 1 gate 58.4 -> 52.2 us and down 62.5 -> 50.2 us with the prefetch; M = 8
    // gate 101.4 -> 107.6 us and down 140.3 -> 183.4 us with it.
    constexpr bool kPrefetch = ROWS <= 2;
    const uint32_t warp = threadIdx.x >> 5;
    const uint32_t lane = threadIdx.x & 31;
    const uint32_t part = warp % SPLIT;
    const uint32_t slot = warp / SPLIT;
    const uint32_t chunks = p.k / 16;  // k is a multiple of 16 (rows are zero padded)
    const uint32_t steps = (chunks + 31) / 32;
    const uint32_t part_steps = (steps + SPLIT - 1) / SPLIT;
    const uint32_t c_begin = min(chunks, part * part_steps * 32);
    const uint32_t c_end = min(chunks, c_begin + part_steps * 32);
    const uint32_t stride = gridDim.x * kSlots;
    const uint32_t c_first = c_begin + lane;
    // Whether a lane's K range starts with a whole four-load trip (the same for every column).
    const bool first_wide = c_first + 96 < c_end;
    const bool writer = lane < static_cast<uint32_t>(ROWS) && lane < p.m;
    uint4 wv[4];
    auto load_trip = [&](uint32_t column, uint32_t c) {
        const int8_t *row = p.w + static_cast<size_t>(column) * p.w_stride;
#pragma unroll
        for (int u = 0; u < 4; ++u) wv[u] = load_weight_chunk(row + static_cast<size_t>(c + 32 * u) * 16);
    };
    uint32_t n = blockIdx.x * kSlots + slot;
    if (kPrefetch && n < p.n && first_wide) load_trip(n, c_first);
    // Programmatic dependent launch: the weights are immutable, so the first trip above is issued
    // while the previous kernel (the row quantizer) may still run; the activation rows and their
    // scales are its output and are read only after the wait.
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    float quant_scale = 0.0f;
    if constexpr (QUANT) {
        // The row quantizer's two passes over the fp32 row (the second one hits L1): max|x|
        // over the CTA, then the int8 row into shared memory (and, from CTA 0, the plan scratch).
        __shared__ float reduce_scratch[32];
        const float4 *x4 = reinterpret_cast<const float4 *>(p.x);
        const uint32_t vectors = p.x_cols / 4;
        float amax = 0.0f;
        for (uint32_t i = threadIdx.x; i < vectors; i += kGemvThreads) amax = abs_max4(amax, __ldg(x4 + i));
        amax = block_max<kGemvThreads>(amax, reduce_scratch);
        quant_scale = row_scale_of(amax);
        const float inverse = __frcp_rn(quant_scale);
        uint32_t *row_words = reinterpret_cast<uint32_t *>(quantized_row);
        uint32_t *scratch_words = reinterpret_cast<uint32_t *>(p.q_out);
        const bool keeper = blockIdx.x == 0;
        for (uint32_t i = threadIdx.x; i < vectors; i += kGemvThreads) {
            const uint32_t packed = quantize4(__ldg(x4 + i), quant_scale, inverse);
            row_words[i] = packed;
            if (keeper) scratch_words[i] = packed;
        }
        for (uint32_t i = vectors + threadIdx.x; i < p.k / 4; i += kGemvThreads) {
            row_words[i] = 0u;
            if (keeper) scratch_words[i] = 0u;
        }
        if (keeper && threadIdx.x == 0) *p.scale_out = quant_scale;
        __syncthreads();
    }
    // 16 activation bytes (chunk `index` of row r): from the CTA's own quantized row, or global.
    auto activation = [&](int r, uint32_t index) -> uint4 {
        if constexpr (QUANT) {
            return reinterpret_cast<const uint4 *>(quantized_row)[index];
        } else {
            return __ldg(reinterpret_cast<const uint4 *>(p.a + static_cast<size_t>(r) * p.a_stride) + index);
        }
    };
    const float row_scale = writer && p.mode != static_cast<int>(EpilogueMode::kStoreS32)
                                ? (QUANT ? quant_scale : p.row_scales[lane])
                                : 0.0f;
    for (; n < p.n; n += stride) {
        const int8_t *w_row = p.w + static_cast<size_t>(n) * p.w_stride;
        // The epilogue's per-column operands, loaded now so they arrive with the weights.
        float col_scale = 0.0f, bias = 0.0f;
        if (part == 0 && writer && p.mode != static_cast<int>(EpilogueMode::kStoreS32)) {
            col_scale = p.col_scales[n];
            if (p.mode == static_cast<int>(EpilogueMode::kDequantizeBias)) bias = p.bias[n];
        }
        int acc[ROWS];
#pragma unroll
        for (int r = 0; r < ROWS; ++r) acc[r] = 0;
        uint32_t c = c_first;
        // Four independent 16-byte weight loads in flight per lane (with the prefetch, the
        // column's first trip was loaded during the previous column's reduction).
        for (; c + 96 < c_end; c += 128) {
            if (!kPrefetch || c != c_first) load_trip(n, c);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
#pragma unroll
                for (int r = 0; r < ROWS; ++r) {
                    if (static_cast<uint32_t>(r) >= p.m) break;  // uniform across the warp
                    const uint4 av = activation(r, c + 32 * u);
                    acc[r] = __dp4a(static_cast<int>(wv[u].x), static_cast<int>(av.x), acc[r]);
                    acc[r] = __dp4a(static_cast<int>(wv[u].y), static_cast<int>(av.y), acc[r]);
                    acc[r] = __dp4a(static_cast<int>(wv[u].z), static_cast<int>(av.z), acc[r]);
                    acc[r] = __dp4a(static_cast<int>(wv[u].w), static_cast<int>(av.w), acc[r]);
                }
            }
        }
        // The next column's first trip streams in while this one finishes and reduces.
        if (kPrefetch && first_wide && n + stride < p.n) load_trip(n + stride, c_first);
        for (; c < c_end; c += 32) {
            const uint4 wt = load_weight_chunk(w_row + static_cast<size_t>(c) * 16);
#pragma unroll
            for (int r = 0; r < ROWS; ++r) {
                if (static_cast<uint32_t>(r) >= p.m) break;  // uniform across the warp
                const uint4 av = activation(r, c);
                acc[r] = __dp4a(static_cast<int>(wt.x), static_cast<int>(av.x), acc[r]);
                acc[r] = __dp4a(static_cast<int>(wt.y), static_cast<int>(av.y), acc[r]);
                acc[r] = __dp4a(static_cast<int>(wt.z), static_cast<int>(av.z), acc[r]);
                acc[r] = __dp4a(static_cast<int>(wt.w), static_cast<int>(av.w), acc[r]);
            }
        }
#pragma unroll
        for (int r = 0; r < ROWS; ++r) {
#pragma unroll
            for (int offset = 16; offset > 0; offset >>= 1) acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], offset);
        }
        int value = acc[0];  // lane r keeps row r's sum
#pragma unroll
        for (int r = 1; r < ROWS; ++r)
            if (lane == static_cast<uint32_t>(r)) value = acc[r];
        if constexpr (SPLIT > 1) {
            // The SPLIT warps of this slot run the same columns, so the named barrier is safe.
            if (lane < static_cast<uint32_t>(ROWS)) partial[warp][lane] = value;
            asm volatile("bar.sync %0, %1;" ::"r"(1 + slot), "r"(32 * SPLIT) : "memory");
            if (part == 0 && writer) {
#pragma unroll
                for (int q = 1; q < SPLIT; ++q) value += partial[slot * SPLIT + q][lane];
            }
            asm volatile("bar.sync %0, %1;" ::"r"(1 + slot), "r"(32 * SPLIT) : "memory");
        }
        if (part == 0 && writer) {
            const size_t index = static_cast<size_t>(lane) * p.out_stride + n;
            if (p.mode == static_cast<int>(EpilogueMode::kStoreS32)) {
                static_cast<int32_t *>(p.out)[index] = value;
            } else {
                float v = dequant_value(value, row_scale, col_scale);
                if (p.mode == static_cast<int>(EpilogueMode::kDequantizeBias)) v = __fadd_rn(v, bias);
                static_cast<float *>(p.out)[index] = v;
            }
        }
    }
}

// ---- tensor-core GEMV (M <= 8) ------------------------------------------------------------
// D[16 weight columns][8 rows] += W[16][32] x A[32][8] with mma.sync m16n8k32 (s8 x s8 -> s32),
// the weights as the A operand and the activation rows as B (rows >= m are zero). The K order
// inside an MMA may be any permutation applied to both operands (the dot is a sum), so every lane
// reads whole 16-byte chunks: over a 64-byte K segment, lane (g, t) loads bytes 16t..16t+15 of
// weight columns g and g + 8 and of activation row g; words x, y feed one MMA (as its k = 4t..
// and 16 + 4t.. fragments) and words z, w a second. Each weight byte is loaded once, with no
// per-row re-reads, so the kernel streams the weights instead of issuing 4 dp4a per row and
// 16 bytes. The 8 warps of a CTA take disjoint K slices of the same 16 columns and add their
// int32 partial sums through shared memory (exact in any order); the epilogue is the same
// ((float)acc * s_a) * s_w (+ bias) as the GEMM.
constexpr int kMmaSegments = 4;  // 64-byte K segments loaded per lane before its MMAs

__device__ __forceinline__ void mma_s8_acc(uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1,
                                           int (&d)[4]) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__global__ void __launch_bounds__(kGemvThreads, 4) w8a8_gemv_mma_kernel(const GemvParams p) {
    __shared__ int partial[kGemvWarps][128];
    const uint32_t warp = threadIdx.x >> 5;
    const uint32_t lane = threadIdx.x & 31;
    const uint32_t g = lane >> 2;  // weight columns g and g + 8; activation row g
    const uint32_t t = lane & 3;   // 16-byte chunk t of each 64-byte segment
    const uint32_t segments = (p.k + 63) / 64;
    const uint32_t per_warp = (segments + kGemvWarps - 1) / kGemvWarps;
    const uint32_t s_begin = min(segments, warp * per_warp);
    const uint32_t s_end = min(segments, s_begin + per_warp);
    const uint32_t groups = (p.n + 15) / 16;
    const bool row_live = g < p.m;
    const int8_t *a_row = p.a + static_cast<size_t>(row_live ? g : 0) * p.a_stride;
    uint4 wa[kMmaSegments], wb[kMmaSegments];
    auto load_weights = [&](const int8_t *w0, const int8_t *w1, bool live0, bool live1, uint32_t s) {
#pragma unroll
        for (int u = 0; u < kMmaSegments; ++u) {
            const uint32_t byte = (s + u) * 64 + t * 16;
            const bool in = s + u < s_end && byte < p.k;
            wa[u] = in && live0 ? load_weight_chunk(w0 + byte) : make_uint4(0, 0, 0, 0);
            wb[u] = in && live1 ? load_weight_chunk(w1 + byte) : make_uint4(0, 0, 0, 0);
        }
    };
    // Programmatic dependent launch: the first group's first weight loads are issued while the
    // previous kernel (the row quantizer) may still run; the activation rows and scales are read
    // only after the wait.
    bool primed = false;
    if (blockIdx.x < groups && s_begin < s_end) {
        const uint32_t n0 = blockIdx.x * 16;
        load_weights(p.w + static_cast<size_t>(n0 + g < p.n ? n0 + g : 0) * p.w_stride,
                     p.w + static_cast<size_t>(n0 + g + 8 < p.n ? n0 + g + 8 : 0) * p.w_stride, n0 + g < p.n,
                     n0 + g + 8 < p.n, s_begin);
        primed = true;
    }
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

    for (uint32_t group = blockIdx.x; group < groups; group += gridDim.x) {
        const uint32_t n0 = group * 16;
        const bool live0 = n0 + g < p.n, live1 = n0 + g + 8 < p.n;
        const int8_t *w0 = p.w + static_cast<size_t>(live0 ? n0 + g : 0) * p.w_stride;
        const int8_t *w1 = p.w + static_cast<size_t>(live1 ? n0 + g + 8 : 0) * p.w_stride;
        int d[4] = {0, 0, 0, 0};
        for (uint32_t s = s_begin; s < s_end; s += kMmaSegments) {
            uint4 av[kMmaSegments];
            if (!primed) load_weights(w0, w1, live0, live1, s);
            primed = false;
#pragma unroll
            for (int u = 0; u < kMmaSegments; ++u) {
                const uint32_t byte = (s + u) * 64 + t * 16;
                const bool in = s + u < s_end && byte < p.k;
                av[u] = in && row_live ? __ldg(reinterpret_cast<const uint4 *>(a_row + byte)) : make_uint4(0, 0, 0, 0);
            }
#pragma unroll
            for (int u = 0; u < kMmaSegments; ++u) {
                mma_s8_acc(wa[u].x, wb[u].x, wa[u].y, wb[u].y, av[u].x, av[u].y, d);
                mma_s8_acc(wa[u].z, wb[u].z, wa[u].w, wb[u].w, av[u].z, av[u].w, d);
            }
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) partial[warp][lane * 4 + i] = d[i];
        __syncthreads();
        if (threadIdx.x < 128) {
            // output x: lane x / 4 of every warp holds it in register x % 4
            const uint32_t x = threadIdx.x;
            const uint32_t col = n0 + ((x >> 2) >> 2) + 8 * ((x & 3) >> 1);
            const uint32_t row = 2 * ((x >> 2) & 3) + (x & 1);
            int value = 0;
#pragma unroll
            for (int w = 0; w < kGemvWarps; ++w) value += partial[w][x];
            if (row < p.m && col < p.n) {
                const size_t index = static_cast<size_t>(row) * p.out_stride + col;
                if (p.mode == static_cast<int>(EpilogueMode::kStoreS32)) {
                    static_cast<int32_t *>(p.out)[index] = value;
                } else {
                    float v = dequant_value(value, p.row_scales[row], p.col_scales[col]);
                    if (p.mode == static_cast<int>(EpilogueMode::kDequantizeBias)) v = __fadd_rn(v, p.bias[col]);
                    static_cast<float *>(p.out)[index] = v;
                }
            }
        }
        __syncthreads();
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

// A launch that may begin while the previous kernel on the stream finishes (programmatic stream
// serialization); the kernel's griddepcontrol.wait orders its reads of that kernel's output.
cudaError_t launch_dependent(void (*kernel)(GemvParams), uint32_t grid, const GemvParams &p, cudaStream_t stream,
                             size_t smem = 0) {
    cudaLaunchAttribute attribute{};
    attribute.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attribute.val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t config{};
    config.gridDim = dim3(grid);
    config.blockDim = dim3(kGemvThreads);
    config.dynamicSmemBytes = smem;
    config.stream = stream;
    config.attrs = &attribute;
    config.numAttrs = 1;
    return cudaLaunchKernelEx(&config, kernel, p);
}

// Split-K reduction: out[r][c] = epilogue(sum over slices s of ws[s * R + r][c]), R = m rounded up
// to kGemmBlockM, four
// columns per thread with 16-byte loads. Integer sums are exact in any order, so the result equals
// the unsplit GEMM's bit for bit. Launched as a programmatic dependent of the split GEMM.
__global__ void __launch_bounds__(256) w8a8_splitk_reduce_kernel(const int32_t *__restrict__ ws, uint32_t splits,
                                                                 uint32_t m, uint32_t n, int mode,
                                                                 const float *__restrict__ row_scales,
                                                                 const float *__restrict__ col_scales,
                                                                 const float *__restrict__ bias, float *__restrict__ out,
                                                                 size_t out_stride) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const uint32_t quads = n / 4;
    const size_t slice = static_cast<size_t>((m + kGemmBlockM - 1) / kGemmBlockM * kGemmBlockM) * n;
    const bool vector_out = (reinterpret_cast<uintptr_t>(out) & 15u) == 0 && (out_stride & 3u) == 0;
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < static_cast<size_t>(m) * quads;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const uint32_t row = static_cast<uint32_t>(i / quads);
        const uint32_t col = static_cast<uint32_t>(i % quads) * 4;
        const int32_t *src = ws + static_cast<size_t>(row) * n + col;
        int4 acc = __ldg(reinterpret_cast<const int4 *>(src));
        for (uint32_t s = 1; s < splits; ++s) {
            const int4 part = __ldg(reinterpret_cast<const int4 *>(src + s * slice));
            acc.x += part.x;
            acc.y += part.y;
            acc.z += part.z;
            acc.w += part.w;
        }
        const int values[4] = {acc.x, acc.y, acc.z, acc.w};
        float result[4];
        const float row_scale = row_scales[row];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            float v = dequant_value(values[j], row_scale, col_scales[col + j]);
            if (mode == static_cast<int>(EpilogueMode::kDequantizeBias)) v = __fadd_rn(v, bias[col + j]);
            result[j] = v;
        }
        float *dst = out + static_cast<size_t>(row) * out_stride + col;
        if (vector_out) {
            *reinterpret_cast<float4 *>(dst) = make_float4(result[0], result[1], result[2], result[3]);
        } else {
#pragma unroll
            for (int j = 0; j < 4; ++j) dst[j] = result[j];
        }
    }
}

// Longest row the one-row GEMV quantizes itself (32 KB of fp32, re-read from L1); its int8 copy
// is the kernel's dynamic shared memory.
constexpr uint32_t kFusedQuantMaxK = 8192;

// CTAs of one instantiation resident per SM, from the occupancy API, cached per device (the
// fused-quantizer variants with the largest shared-memory row they take).
template <int ROWS, int SPLIT, bool QUANT = false>
int resident_ctas() {
    static std::atomic<int> cached[64] = {};
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= 64) return 1;
    const int known = cached[device].load(std::memory_order_relaxed);
    if (known > 0) return known;
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, w8a8_gemv_kernel<ROWS, SPLIT, QUANT>, kGemvThreads,
                                                      QUANT ? kFusedQuantMaxK : 0) != cudaSuccess ||
        per_sm < 1) {
        (void)cudaGetLastError();
        return 1;
    }
    cached[device].store(per_sm, std::memory_order_relaxed);
    return per_sm;
}

// Balanced persistent grid for one split: the rounds every column slot runs, the CTAs that
// gives, and the share of the SMs' resident CTA slots it occupies.
struct GemvShape {
    uint32_t grid = 0;
    double occupied = 0.0;
};

template <int ROWS, int SPLIT, bool QUANT = false>
GemvShape gemv_shape(uint32_t n, int sm_count) {
    constexpr uint64_t kSlots = kGemvWarps / SPLIT;
    const uint64_t capacity =
        static_cast<uint64_t>(sm_count) * static_cast<uint64_t>(resident_ctas<ROWS, SPLIT, QUANT>());
    const uint64_t rounds = (n + capacity * kSlots - 1) / (capacity * kSlots);
    GemvShape shape;
    shape.grid = static_cast<uint32_t>((n + kSlots * rounds - 1) / (kSlots * rounds));
    shape.occupied = static_cast<double>(shape.grid) / static_cast<double>(capacity);
    return shape;
}

// The smallest split that keeps at least three quarters of the resident CTA slots busy (so
// enough weight loads are in flight to stream HBM), among splits that leave every warp at
// least four 32-chunk steps of K; else the split that occupies the most. Wide matrices take
// one warp per column; narrow ones (a column shard, or the down projection's few long
// columns) spread each column over 2, 4 or 8 warps.
template <int ROWS, bool QUANT = false>
cudaError_t launch_rows(const GemvParams &p, int sm_count, cudaStream_t stream) {
    const uint32_t steps = (p.k / 16 + 31) / 32;
    const GemvShape shapes[4] = {gemv_shape<ROWS, 1, QUANT>(p.n, sm_count), gemv_shape<ROWS, 2, QUANT>(p.n, sm_count),
                                 gemv_shape<ROWS, 4, QUANT>(p.n, sm_count), gemv_shape<ROWS, 8, QUANT>(p.n, sm_count)};
    int choice = 0;
    for (int i = 0; i < 4; ++i) {
        if (i > 0 && steps < 4u * (1u << i)) break;
        if (shapes[i].occupied >= 0.75) {
            choice = i;
            break;
        }
        if (shapes[i].occupied > shapes[choice].occupied) choice = i;
    }
    const uint32_t grid = shapes[choice].grid;
    const size_t smem = QUANT ? p.k : 0;
    switch (choice) {
        case 0: return launch_dependent(w8a8_gemv_kernel<ROWS, 1, QUANT>, grid, p, stream, smem);
        case 1: return launch_dependent(w8a8_gemv_kernel<ROWS, 2, QUANT>, grid, p, stream, smem);
        case 2: return launch_dependent(w8a8_gemv_kernel<ROWS, 4, QUANT>, grid, p, stream, smem);
        default: return launch_dependent(w8a8_gemv_kernel<ROWS, 8, QUANT>, grid, p, stream, smem);
    }
}

int mma_resident_ctas() {
    static std::atomic<int> cached[64] = {};
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= 64) return 1;
    const int known = cached[device].load(std::memory_order_relaxed);
    if (known > 0) return known;
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, w8a8_gemv_mma_kernel, kGemvThreads, 0) != cudaSuccess ||
        per_sm < 1) {
        (void)cudaGetLastError();
        return 1;
    }
    cached[device].store(per_sm, std::memory_order_relaxed);
    return per_sm;
}

// Persistent grid filling every resident slot, so each SM carries the same share of the 16-column
// groups (a grid trimmed to equal rounds per CTA put a fourth CTA on a few SMs: 70B gate at M = 8
// 52.3 against 48.2 us with the quantizer).
cudaError_t launch_mma(const GemvParams &p, int sm_count, cudaStream_t stream) {
    const uint64_t groups = (p.n + 15) / 16;
    const uint64_t capacity = static_cast<uint64_t>(sm_count) * static_cast<uint64_t>(mma_resident_ctas());
    const uint32_t grid = static_cast<uint32_t>(groups < capacity ? groups : capacity);
    return launch_dependent(w8a8_gemv_mma_kernel, grid, p, stream);
}

template <int ROWS, bool QUANT = false>
cudaError_t preload_rows() {
    cudaFuncAttributes attributes;
    cudaError_t error = cudaFuncGetAttributes(&attributes, w8a8_gemv_kernel<ROWS, 1, QUANT>);
    if (error == cudaSuccess) error = cudaFuncGetAttributes(&attributes, w8a8_gemv_kernel<ROWS, 2, QUANT>);
    if (error == cudaSuccess) error = cudaFuncGetAttributes(&attributes, w8a8_gemv_kernel<ROWS, 4, QUANT>);
    if (error == cudaSuccess) error = cudaFuncGetAttributes(&attributes, w8a8_gemv_kernel<ROWS, 8, QUANT>);
    (void)resident_ctas<ROWS, 1, QUANT>();
    (void)resident_ctas<ROWS, 2, QUANT>();
    (void)resident_ctas<ROWS, 4, QUANT>();
    (void)resident_ctas<ROWS, 8, QUANT>();
    return error;
}

}  // namespace

cudaError_t preload_w8a8_gemv() {
    cudaFuncAttributes attributes;
    cudaError_t error = cudaFuncGetAttributes(&attributes, w8a8_gemv_mma_kernel);
    (void)mma_resident_ctas();
    if (error == cudaSuccess) error = preload_rows<1>();
    if (error == cudaSuccess) error = preload_rows<1, true>();
    return error;
}

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
    // One row streams the weights best with dp4a and the cross-column prefetch; two or more rows
    // go to the tensor-core kernel, whose time does not grow with the rows. Measured on B200
    // (prepared plan, row quantizer included, L2 flushed): 70B gate 8192 -> 28672 at M = 1 50.2 us
    // (dp4a) against 52.4 (MMA); at M = 4 68.6 against 54.2, at M = 8 103.5 against 54.3; 70B down
    // 28672 -> 8192 at M = 8 140.3 against 52.2.
    if (m == 1) return launch_rows<1>(p, sm_count, stream);
    return launch_mma(p, sm_count, stream);
}

cudaError_t launch_w8a8_gemv_quantize(const float *x, uint32_t cols, int8_t *q_out, float *scale_out, const int8_t *w,
                                      size_t w_stride, uint32_t n, uint32_t k, const GemmEpilogue &epilogue,
                                      int sm_count, cudaStream_t stream) {
    if (n == 0) return cudaSuccess;
    if (x == nullptr || q_out == nullptr || scale_out == nullptr || cols == 0 || cols % 4 != 0 || k < cols ||
        k % 16 != 0 || k > kFusedQuantMaxK || w_stride % 16 != 0 || (reinterpret_cast<uintptr_t>(x) & 15u) != 0 ||
        (reinterpret_cast<uintptr_t>(q_out) & 3u) != 0 || (reinterpret_cast<uintptr_t>(w) & 15u) != 0 ||
        epilogue.mode == EpilogueMode::kStoreS32) {
        return cudaErrorNotSupported;
    }
    GemvParams p{};
    p.a = q_out;
    p.a_stride = k;
    p.w = w;
    p.w_stride = w_stride;
    p.m = 1;
    p.n = n;
    p.k = k;
    p.mode = static_cast<int>(epilogue.mode);
    p.row_scales = scale_out;
    p.col_scales = epilogue.col_scales;
    p.bias = epilogue.bias;
    p.out = epilogue.out;
    p.out_stride = epilogue.out_stride;
    p.x = x;
    p.x_cols = cols;
    p.q_out = q_out;
    p.scale_out = scale_out;
    return launch_rows<1, true>(p, sm_count, stream);
}

cudaError_t launch_w8a8_splitk_reduce(const int32_t *workspace, uint32_t splits, uint32_t m, uint32_t n,
                                      const GemmEpilogue &epilogue, int sm_count, cudaStream_t stream) {
    if (m == 0 || n == 0) return cudaSuccess;
    if (n % 4 != 0 || epilogue.mode == EpilogueMode::kStoreS32) return cudaErrorInvalidValue;
    const uint64_t items = static_cast<uint64_t>(m) * (n / 4);
    uint64_t grid = (items + 255) / 256;
    const uint64_t cap = static_cast<uint64_t>(sm_count) * 8u;
    if (grid > cap) grid = cap;
    cudaLaunchAttribute attribute{};
    attribute.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attribute.val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t config{};
    config.gridDim = dim3(static_cast<uint32_t>(grid));
    config.blockDim = dim3(256);
    config.stream = stream;
    config.attrs = &attribute;
    config.numAttrs = 1;
    return cudaLaunchKernelEx(&config, w8a8_splitk_reduce_kernel, workspace, splits, m, n, static_cast<int>(epilogue.mode),
                              epilogue.row_scales, epilogue.col_scales, epilogue.bias, static_cast<float *>(epilogue.out),
                              epilogue.out_stride);
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
