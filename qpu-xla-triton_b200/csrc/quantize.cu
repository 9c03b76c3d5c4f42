// Quantizer kernels of the quantized-linear path (all HBM-bound, no tensor cores).
//
//  * quantize_rows_int8: per-row symmetric int8 (src/qpu_xla/models/tinyllama/quantization.py:156-171,
//    :1065-1071 for activations, :1085-1092 for weights). One CTA per row; the row is read once with
//    128-bit loads into registers, reduced to max|x| with warp shuffles, then quantized from registers.
//    Rows longer than ~14.5K columns stream through shared memory instead (bulk copies, two stages).
//    Bit-exact with NumPy: the quotient x / scale is the IEEE one (a reciprocal product where it
//    provably rounds the same, __fdiv_rn elsewhere; never fast-math), round-half-even, clamp +-127.
//  * quantize_q8_0: fp32 -> native block_q8_0 (examples/benchmark_llama_cpp_qpu_persistent_q4.py:42-54).
//  * quantize_q4_0: fp32 -> native block_q4_0, ggml's published quantize_row_q4_0_ref.
//  * q4_0_repack: native 18-byte Q4_0 blocks -> the prepared layout (16-byte nibble blocks + fp16 scales).
#include <cuda_fp16.h>

#include "qpucuda_internal.h"
#include "row_quantize.cuh"
#include "sm100_sync.cuh"

namespace qpucuda {
namespace {

__device__ __forceinline__ float4 load_stream(const float4 *p) {
    float4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(p));
    return v;
}

// Vector path: cols % 4 == 0, 16-byte aligned rows; VEC float4 per thread cached in registers.
template <int THREADS, int VEC>
__global__ void __launch_bounds__(THREADS) quantize_rows_int8_vec(const float *__restrict__ x, size_t x_stride,
                                                                  uint32_t rows, uint32_t cols, uint32_t padded_cols,
                                                                  int8_t *__restrict__ q, size_t q_stride,
                                                                  float *__restrict__ scales) {
    __shared__ float scratch[32];
    const uint32_t vectors = cols / 4;
    // Launched as a programmatic dependent of the previous kernel on the stream: wait for it
    // (its writes may be this kernel's source, or it may still read this kernel's destination)
    // before touching memory, then let the next kernel (the GEMV that reads these rows) launch
    // and start streaming its weights while the rows are quantized.
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    for (uint32_t row = blockIdx.x; row < rows; row += gridDim.x) {
        const float4 *source = reinterpret_cast<const float4 *>(x + static_cast<size_t>(row) * x_stride);
        float4 cache[VEC];
        float amax = 0.0f;
#pragma unroll
        for (int v = 0; v < VEC; ++v) {
            const uint32_t index = threadIdx.x + v * THREADS;
            if (index < vectors) {
                cache[v] = load_stream(source + index);
                amax = fmaxf(amax, fmaxf(fmaxf(fabsf(cache[v].x), fabsf(cache[v].y)),
                                         fmaxf(fabsf(cache[v].z), fabsf(cache[v].w))));
            }
        }
        amax = block_max<THREADS>(amax, scratch);
        const float scale = fmaxf(__fdiv_rn(amax, 127.0f), scale_floor());
        const float inverse = __frcp_rn(scale);
        uint32_t *destination = reinterpret_cast<uint32_t *>(q + static_cast<size_t>(row) * q_stride);
#pragma unroll
        for (int v = 0; v < VEC; ++v) {
            const uint32_t index = threadIdx.x + v * THREADS;
            if (index < vectors) {
                destination[index] = pack4(
                    quantize_value_fast(cache[v].x, scale, inverse), quantize_value_fast(cache[v].y, scale, inverse),
                    quantize_value_fast(cache[v].z, scale, inverse), quantize_value_fast(cache[v].w, scale, inverse));
            }
        }
        int8_t *row_q = q + static_cast<size_t>(row) * q_stride;
        for (uint32_t c = cols + threadIdx.x; c < padded_cols; c += THREADS) row_q[c] = 0;
        if (threadIdx.x == 0) scales[row] = scale;
    }
}

// Staged path for many long rows: a persistent CTA walks rows blockIdx.x, + gridDim.x, ... with
// STAGES row buffers in shared memory, each filled by one 1D bulk copy (TMA engine, completing on
// the stage's mbarrier) issued by thread 0 as soon as the CTA has finished the row that held it.
// Up to STAGES rows per CTA are in flight while the CTA reduces and quantizes the current one,
// so the SM keeps streaming instead of alternating load and compute phases. Waits are bounded
// (error word + abort); an aborting CTA drains its own outstanding copies before it exits.
template <int THREADS, int STAGES>
__global__ void __launch_bounds__(THREADS) quantize_rows_int8_bulk(const float *__restrict__ x, size_t x_stride,
                                                                   uint32_t rows, uint32_t cols, uint32_t padded_cols,
                                                                   int8_t *__restrict__ q, size_t q_stride,
                                                                   float *__restrict__ scales,
                                                                   unsigned int *error_word) {
    extern __shared__ __align__(128) float4 staged[];  // [STAGES][cols / 4]
    __shared__ __align__(8) uint64_t full[STAGES];
    __shared__ float scratch[32];
    __shared__ int abort_flag;
    const uint32_t vectors = cols / 4;
    const uint32_t row_bytes = cols * 4u;
    const uint32_t step = gridDim.x;
    auto refill = [&](uint32_t row, uint32_t stage) {
        const uint32_t bar = sm100::smem_u32(&full[stage]);
        sm100::mbar_expect_tx(bar, row_bytes);
        sm100::bulk_load(sm100::smem_u32(staged + static_cast<size_t>(stage) * vectors),
                         x + static_cast<size_t>(row) * x_stride, row_bytes, bar);
    };
    if (threadIdx.x == 0) {
        abort_flag = 0;
#pragma unroll
        for (int s = 0; s < STAGES; ++s) sm100::mbar_init(sm100::smem_u32(&full[s]), 1);
        sm100::mbar_init_fence();
#pragma unroll
        for (int s = 0; s < STAGES; ++s) {
            const uint32_t row = blockIdx.x + s * step;
            if (row < rows) refill(row, s);
        }
    }
    __syncthreads();
    uint32_t iteration = 0;
    for (uint32_t row = blockIdx.x; row < rows; row += step, ++iteration) {
        const uint32_t stage = iteration % STAGES;
        const uint32_t parity = (iteration / STAGES) & 1u;
        const bool landed = sm100::wait_bounded(sm100::smem_u32(&full[stage]), parity, &abort_flag, error_word);
        if (!__syncthreads_and(landed)) {
            if (threadIdx.x == 0) {  // let this CTA's copies in flight land before it exits
                for (uint32_t k = 0; k < STAGES; ++k) {
                    if (row + k * step < rows) {
                        sm100::wait_drain(sm100::smem_u32(&full[(iteration + k) % STAGES]),
                                          ((iteration + k) / STAGES) & 1u);
                    }
                }
            }
            return;
        }
        const float4 *slots = staged + static_cast<size_t>(stage) * vectors;
        float amax = 0.0f;
        for (uint32_t i = threadIdx.x; i < vectors; i += THREADS) {
            const float4 v = slots[i];
            amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
        }
        amax = block_max<THREADS>(amax, scratch);
        const float scale = fmaxf(__fdiv_rn(amax, 127.0f), scale_floor());
        const float inverse = __frcp_rn(scale);
        int8_t *row_q = q + static_cast<size_t>(row) * q_stride;
        uint32_t *destination = reinterpret_cast<uint32_t *>(row_q);
        for (uint32_t i = threadIdx.x; i < vectors; i += THREADS) {
            const float4 v = slots[i];
            destination[i] = pack4(quantize_value_fast(v.x, scale, inverse), quantize_value_fast(v.y, scale, inverse),
                                   quantize_value_fast(v.z, scale, inverse), quantize_value_fast(v.w, scale, inverse));
        }
        for (uint32_t c = cols + threadIdx.x; c < padded_cols; c += THREADS) row_q[c] = 0;
        if (threadIdx.x == 0) scales[row] = scale;
        __syncthreads();  // every thread is done with this stage
        if (threadIdx.x == 0 && row + STAGES * step < rows) refill(row + STAGES * step, stage);
    }
}

// Generic path: any alignment / column count; the second pass re-reads the row (an L2 hit).
__global__ void __launch_bounds__(256) quantize_rows_int8_generic(const float *__restrict__ x, size_t x_stride,
                                                                  uint32_t rows, uint32_t cols, uint32_t padded_cols,
                                                                  int8_t *__restrict__ q, size_t q_stride,
                                                                  float *__restrict__ scales) {
    __shared__ float scratch[32];
    for (uint32_t row = blockIdx.x; row < rows; row += gridDim.x) {
        const float *source = x + static_cast<size_t>(row) * x_stride;
        float amax = 0.0f;
        for (uint32_t c = threadIdx.x; c < cols; c += 256) amax = fmaxf(amax, fabsf(source[c]));
        amax = block_max<256>(amax, scratch);
        const float scale = fmaxf(__fdiv_rn(amax, 127.0f), scale_floor());
        int8_t *row_q = q + static_cast<size_t>(row) * q_stride;
        for (uint32_t c = threadIdx.x; c < padded_cols; c += 256) {
            row_q[c] = c < cols ? static_cast<int8_t>(quantize_value(source[c], scale)) : static_cast<int8_t>(0);
        }
        if (threadIdx.x == 0) scales[row] = scale;
    }
}

template <int THREADS, int VEC>
cudaError_t launch_vec(const float *x, size_t x_stride, uint32_t rows, uint32_t cols, uint32_t padded_cols, int8_t *q,
                       size_t q_stride, float *scales, cudaStream_t stream) {
    const uint32_t grid = rows < 65535u * 4u ? rows : 65535u * 4u;
    cudaLaunchAttribute attribute{};
    attribute.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attribute.val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t config{};
    config.gridDim = dim3(grid);
    config.blockDim = dim3(THREADS);
    config.stream = stream;
    config.attrs = &attribute;
    config.numAttrs = 1;
    return cudaLaunchKernelEx(&config, quantize_rows_int8_vec<THREADS, VEC>, x, x_stride, rows, cols, padded_cols, q,
                              q_stride, scales);
}

// Layout path: one thread per row; consecutive threads take consecutive rows, so for NCHW
// pixels (row step 1, element = channel, element stride H*W) every channel read is coalesced
// across the warp. Two passes over the row (max, then quantize; the second hits L1/L2); the
// int8 row is written four bytes at a time, zero-padded to padded_cols (a multiple of 4).
__global__ void __launch_bounds__(256) quantize_rows_int8_layout_kernel(
    const float *__restrict__ x, uint32_t rows, uint32_t cols, uint32_t padded_cols, uint32_t rows_per_batch,
    size_t batch_stride, size_t row_stride, size_t col_stride, int8_t *__restrict__ q, size_t q_stride,
    float *__restrict__ scales) {
    const uint32_t row = blockIdx.x * blockDim.x + threadIdx.x;
    if (row >= rows) return;
    const float *source = x + static_cast<size_t>(row / rows_per_batch) * batch_stride +
                          static_cast<size_t>(row % rows_per_batch) * row_stride;
    float amax = 0.0f;
    for (uint32_t c = 0; c < cols; ++c) amax = fmaxf(amax, fabsf(__ldg(source + c * col_stride)));
    const float scale = fmaxf(__fdiv_rn(amax, 127.0f), scale_floor());
    uint32_t *destination = reinterpret_cast<uint32_t *>(q + static_cast<size_t>(row) * q_stride);
    for (uint32_t c = 0; c < padded_cols; c += 4) {
        int v[4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
            v[i] = c + i < cols ? quantize_value(__ldg(source + (c + i) * col_stride), scale) : 0;
        destination[c / 4] = pack4(v[0], v[1], v[2], v[3]);
    }
    scales[row] = scale;
}

// ---- Q8_0 -------------------------------------------------------------------------------

// One warp per 32-element block: d = amax / 127 (fp32), id = 1/d (0 when d == 0),
// q = clip(rint(x * id), -127, 127), stored scale fp16(d) (round to nearest even).
__global__ void __launch_bounds__(256) quantize_q8_0_kernel(const float *__restrict__ x, size_t x_stride,
                                                            uint32_t rows, uint32_t blocks_per_row,
                                                            uint8_t *__restrict__ out) {
    const uint32_t lane = threadIdx.x & 31;
    const size_t total = static_cast<size_t>(rows) * blocks_per_row;
    for (size_t block = (static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x) / 32; block < total;
         block += static_cast<size_t>(gridDim.x) * blockDim.x / 32) {
        const size_t row = block / blocks_per_row;
        const size_t column_block = block % blocks_per_row;
        const float value = x[row * x_stride + column_block * 32 + lane];
        float amax = fabsf(value);
#pragma unroll
        for (int offset = 16; offset > 0; offset >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, offset));
        const float d = __fdiv_rn(amax, 127.0f);
        const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
        int v = __float2int_rn(__fmul_rn(value, id));
        v = v < -127 ? -127 : (v > 127 ? 127 : v);
        uint8_t *destination = out + block * 34;  // blocks start on even bytes
        if (lane == 0) *reinterpret_cast<unsigned short *>(destination) = __half_as_ushort(__float2half_rn(d));
        destination[2 + lane] = static_cast<uint8_t>(static_cast<int8_t>(v));
    }
}

// ---- Q4_0 -------------------------------------------------------------------------------

// One warp per block. max = the signed value of largest magnitude, first index on ties
// (ggml compares amax < |v| in index order); d = max / -8; id = 1/d (0 when d == 0);
// code = min(15, trunc(x * id + 8.5)); byte j = code j | code j+16 << 4.
__global__ void __launch_bounds__(256) quantize_q4_0_kernel(const float *__restrict__ x, size_t x_stride,
                                                            uint32_t rows, uint32_t blocks_per_row,
                                                            uint8_t *__restrict__ out) {
    const uint32_t lane = threadIdx.x & 31;
    const size_t total = static_cast<size_t>(rows) * blocks_per_row;
    for (size_t block = (static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x) / 32; block < total;
         block += static_cast<size_t>(gridDim.x) * blockDim.x / 32) {
        const size_t row = block / blocks_per_row;
        const size_t column_block = block % blocks_per_row;
        const float value = x[row * x_stride + column_block * 32 + lane];
        float best_abs = fabsf(value);
        uint32_t best_lane = lane;
#pragma unroll
        for (int offset = 16; offset > 0; offset >>= 1) {
            const float other_abs = __shfl_xor_sync(0xffffffffu, best_abs, offset);
            const uint32_t other_lane = __shfl_xor_sync(0xffffffffu, best_lane, offset);
            if (other_abs > best_abs || (other_abs == best_abs && other_lane < best_lane)) {
                best_abs = other_abs;
                best_lane = other_lane;
            }
        }
        const float maximum = __shfl_sync(0xffffffffu, value, best_lane);
        const float d = __fdiv_rn(maximum, -8.0f);
        const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
        int code = __float2int_rz(__fadd_rn(__fmul_rn(value, id), 8.5f));
        code = code > 15 ? 15 : (code < 0 ? 0 : code);
        const int high = __shfl_down_sync(0xffffffffu, code, 16);
        uint8_t *destination = out + block * 18;  // blocks start on even bytes
        if (lane == 0) *reinterpret_cast<unsigned short *>(destination) = __half_as_ushort(__float2half_rn(d));
        if (lane < 16) destination[2 + lane] = static_cast<uint8_t>(code | (high << 4));
    }
}

// Native [columns][blocks][18] -> nibbles [columns][blocks][16] + scales [columns][scale_stride].
__global__ void __launch_bounds__(256) q4_0_repack_kernel(const uint8_t *__restrict__ native, size_t total_blocks,
                                                          uint32_t blocks, uint32_t scale_stride,
                                                          uint8_t *__restrict__ nibbles,
                                                          uint16_t *__restrict__ scales) {
    for (size_t block = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; block < total_blocks;
         block += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const uint16_t *source = reinterpret_cast<const uint16_t *>(native + block * 18);  // blocks start on even bytes
        uint32_t words[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            words[i] = static_cast<uint32_t>(source[1 + 2 * i]) | (static_cast<uint32_t>(source[2 + 2 * i]) << 16);
        }
        reinterpret_cast<uint4 *>(nibbles)[block] = make_uint4(words[0], words[1], words[2], words[3]);
        scales[(block / blocks) * scale_stride + block % blocks] = source[0];
    }
}

uint32_t grid_for(size_t work_items, uint32_t per_block) {
    size_t grid = (work_items + per_block - 1) / per_block;
    if (grid > 148u * 64u) grid = 148u * 64u;
    return grid == 0 ? 1u : static_cast<uint32_t>(grid);
}

}  // namespace

namespace {

// Usable dynamic shared memory per CTA on sm_100 (227 KB) less the static scratch and mbarriers.
constexpr size_t kStagedSmemBudget = 227u * 1024u - 512u;

// The staged kernel's shared-memory attribute is raised to the whole budget once per device, so
// every row length fits; 1024 threads and at least half the shared memory per CTA leave one CTA
// per SM.
template <int THREADS, int STAGES>
cudaError_t configure_staged() {
    static PerDeviceOnce configured;
    return configured.run([] {
        return cudaFuncSetAttribute(quantize_rows_int8_bulk<THREADS, STAGES>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    static_cast<int>(kStagedSmemBudget));
    });
}

template <int THREADS, int STAGES>
cudaError_t launch_staged_config(const float *x, size_t x_stride, uint32_t rows, uint32_t cols, uint32_t padded_cols,
                                 int8_t *q, size_t q_stride, float *scales, unsigned int *error_word, int sm_count,
                                 cudaStream_t stream) {
    const size_t smem = static_cast<size_t>(STAGES) * cols * sizeof(float);
    auto kernel = quantize_rows_int8_bulk<THREADS, STAGES>;
    const cudaError_t error = configure_staged<THREADS, STAGES>();
    if (error != cudaSuccess) return error;
    const int per_sm = 1;
    const uint64_t slots = static_cast<uint64_t>(sm_count) * static_cast<uint64_t>(per_sm);
    const uint32_t grid = rows < slots ? rows : static_cast<uint32_t>(slots);
    kernel<<<grid, THREADS, smem, stream>>>(x, x_stride, rows, cols, padded_cols, q, q_stride, scales, error_word);
    return cudaGetLastError();
}

// Picks the bulk-staged kernel (1024 threads, two row stages) for aligned rows too long for the
// register-cached kernel to keep more than one row per SM (row > 1/4 of the shared memory budget,
// K > ~14.5K), with at least two rows per SM; returns cudaErrorNotSupported otherwise. Measured
// on B200 at M = 4096: K = 28672 takes 113 us (0.79 of HBM) against 136 us register-cached;
// at K <= 8192 the two kernels are within 3% and more stages (fewer CTAs per SM) were slower.
cudaError_t launch_staged(const float *x, size_t x_stride, uint32_t rows, uint32_t cols, uint32_t padded_cols,
                          int8_t *q, size_t q_stride, float *scales, unsigned int *error_word, cudaStream_t stream) {
    int device = 0, sm_count = 0;
    if (error_word == nullptr || cudaGetDevice(&device) != cudaSuccess ||
        cudaDeviceGetAttribute(&sm_count, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || sm_count <= 0) {
        (void)cudaGetLastError();
        return cudaErrorNotSupported;
    }
    const size_t row_bytes = static_cast<size_t>(cols) * sizeof(float);
    if (rows < 2u * static_cast<uint32_t>(sm_count) || 4 * row_bytes <= kStagedSmemBudget ||
        2 * row_bytes > kStagedSmemBudget) {
        return cudaErrorNotSupported;
    }
    return launch_staged_config<1024, 2>(x, x_stride, rows, cols, padded_cols, q, q_stride, scales, error_word,
                                        sm_count, stream);
}

}  // namespace

cudaError_t preload_quantize_rows_int8() {
    cudaFuncAttributes attributes;
    cudaError_t error = configure_staged<1024, 2>();
    if (error == cudaSuccess) error = cudaFuncGetAttributes(&attributes, quantize_rows_int8_vec<32, 8>);
    if (error == cudaSuccess) error = cudaFuncGetAttributes(&attributes, quantize_rows_int8_vec<64, 8>);
    if (error == cudaSuccess) error = cudaFuncGetAttributes(&attributes, quantize_rows_int8_vec<128, 8>);
    if (error == cudaSuccess) error = cudaFuncGetAttributes(&attributes, quantize_rows_int8_vec<256, 8>);
    if (error == cudaSuccess) error = cudaFuncGetAttributes(&attributes, quantize_rows_int8_vec<512, 8>);
    if (error == cudaSuccess) error = cudaFuncGetAttributes(&attributes, quantize_rows_int8_vec<1024, 8>);
    if (error == cudaSuccess) error = cudaFuncGetAttributes(&attributes, quantize_rows_int8_generic);
    return error;
}

cudaError_t launch_quantize_rows_int8(const float *x, size_t x_stride, uint32_t rows, uint32_t cols,
                                      uint32_t padded_cols, int8_t *q, size_t q_stride, float *scales,
                                      unsigned int *error_word, cudaStream_t stream) {
    if (rows == 0) return cudaSuccess;
    const bool vector_ok = cols % 4 == 0 && x_stride % 4 == 0 && (reinterpret_cast<uintptr_t>(x) & 15u) == 0 &&
                           q_stride % 4 == 0 && (reinterpret_cast<uintptr_t>(q) & 3u) == 0;
    const uint32_t vectors = cols / 4;
    if (vector_ok) {
        const cudaError_t staged =
            launch_staged(x, x_stride, rows, cols, padded_cols, q, q_stride, scales, error_word, stream);
        if (staged != cudaErrorNotSupported) return staged;
        // VEC = 8 float4 per thread; pick the smallest warp multiple of threads that covers the row.
        if (vectors <= 32 * 8) return launch_vec<32, 8>(x, x_stride, rows, cols, padded_cols, q, q_stride, scales, stream);
        if (vectors <= 64 * 8) return launch_vec<64, 8>(x, x_stride, rows, cols, padded_cols, q, q_stride, scales, stream);
        if (vectors <= 128 * 8) return launch_vec<128, 8>(x, x_stride, rows, cols, padded_cols, q, q_stride, scales, stream);
        if (vectors <= 256 * 8) return launch_vec<256, 8>(x, x_stride, rows, cols, padded_cols, q, q_stride, scales, stream);
        if (vectors <= 512 * 8) return launch_vec<512, 8>(x, x_stride, rows, cols, padded_cols, q, q_stride, scales, stream);
        if (vectors <= 1024 * 8) return launch_vec<1024, 8>(x, x_stride, rows, cols, padded_cols, q, q_stride, scales, stream);
    }
    const uint32_t grid = rows < 65535u * 4u ? rows : 65535u * 4u;
    quantize_rows_int8_generic<<<grid, 256, 0, stream>>>(x, x_stride, rows, cols, padded_cols, q, q_stride, scales);
    return cudaGetLastError();
}

cudaError_t launch_quantize_q8_0(const float *x, size_t x_stride, uint32_t rows, uint32_t cols, uint8_t *blocks,
                                 cudaStream_t stream) {
    const size_t total = static_cast<size_t>(rows) * (cols / 32);
    if (total == 0) return cudaSuccess;
    quantize_q8_0_kernel<<<grid_for(total, 8), 256, 0, stream>>>(x, x_stride, rows, cols / 32, blocks);
    return cudaGetLastError();
}

cudaError_t launch_quantize_rows_int8_layout(const float *x, uint32_t rows, uint32_t cols, uint32_t padded_cols,
                                             uint32_t rows_per_batch, size_t batch_stride, size_t row_stride,
                                             size_t col_stride, int8_t *q, size_t q_stride, float *scales,
                                             cudaStream_t stream) {
    if (rows == 0) return cudaSuccess;
    if (rows_per_batch == 0 || rows_per_batch >= rows) {
        rows_per_batch = rows;
        batch_stride = 0;
    }
    if (col_stride == 1 && rows_per_batch == rows) {
        return launch_quantize_rows_int8(x, row_stride, rows, cols, padded_cols, q, q_stride, scales, nullptr, stream);
    }
    if (padded_cols % 4 != 0 || q_stride % 4 != 0 || (reinterpret_cast<uintptr_t>(q) & 3u) != 0) return cudaErrorInvalidValue;
    quantize_rows_int8_layout_kernel<<<(rows + 255) / 256, 256, 0, stream>>>(
        x, rows, cols, padded_cols, rows_per_batch, batch_stride, row_stride, col_stride, q, q_stride, scales);
    return cudaGetLastError();
}

cudaError_t launch_quantize_q4_0(const float *x, size_t x_stride, uint32_t rows, uint32_t cols, uint8_t *blocks,
                                 cudaStream_t stream) {
    const size_t total = static_cast<size_t>(rows) * (cols / 32);
    if (total == 0) return cudaSuccess;
    quantize_q4_0_kernel<<<grid_for(total, 8), 256, 0, stream>>>(x, x_stride, rows, cols / 32, blocks);
    return cudaGetLastError();
}

cudaError_t launch_q4_0_repack(const uint8_t *native, uint32_t columns, uint32_t blocks, uint32_t scale_stride,
                               uint8_t *nibbles, uint16_t *scales, cudaStream_t stream) {
    const size_t total = static_cast<size_t>(columns) * blocks;
    if (total == 0) return cudaSuccess;
    q4_0_repack_kernel<<<grid_for(total, 256), 256, 0, stream>>>(native, total, blocks, scale_stride, nibbles, scales);
    return cudaGetLastError();
}

}  // namespace qpucuda
