// Internal declarations shared by the qpucuda translation units.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdarg>
#include <cstdint>
#include <mutex>

#include "qpucuda_runtime.h"

#ifndef QPUCUDA_VERSION
#define QPUCUDA_VERSION "0.1.0"
#endif

struct qpucuda_context {
    int device = 0;
    uint64_t timeout_ns = 0;
    uint32_t failure_mask = 0;
    cudaStream_t stream = nullptr;      // stream work is issued on
    cudaStream_t own_stream = nullptr;  // library-owned stream (always created)
    cudaEvent_t done_event = nullptr;   // reused for bounded waits
    bool poisoned = false;
    int sm_count = 0;
    int cc_major = 0;
    int cc_minor = 0;
    size_t l2_bytes = 0;
    size_t global_bytes = 0;
    char device_name[128] = {0};
    // Device error word written by kernels whose bounded waits expire, and a
    // pinned host mirror read back after synchronous waits.
    unsigned int *d_error = nullptr;
    unsigned int *h_error = nullptr;
    std::mutex mutex;
    char last_error[256] = {0};
};

namespace qpucuda {

// Kernel-side error codes stored in qpucuda_context::d_error.
enum KernelError : unsigned int {
    kKernelOk = 0,
    kKernelWaitTimeout = 1,  // an mbarrier wait exceeded its bound
};

// Upper bound for any single in-kernel barrier wait, in nanoseconds.
constexpr unsigned long long kKernelWaitLimitNs = 1000000000ull;

qpucuda_status fail(qpucuda_context *context, qpucuda_status status, const char *format, ...);
qpucuda_status cuda_fail(qpucuda_context *context, cudaError_t error, const char *operation,
                         qpucuda_status status = QPUCUDA_SUBMISSION_FAILED);
// Rejects work on a poisoned context and applies QPUCUDA_FAIL_SUBMISSION.
qpucuda_status begin_submit(qpucuda_context *context);
// Bounded wait on the context stream (event poll against timeout_ns), then
// applies QPUCUDA_FAIL_WAIT and checks the kernels' error word. A failure
// poisons the context.
qpucuda_status wait_stream(qpucuda_context *context);
// Current-device guard.
class DeviceGuard {
  public:
    explicit DeviceGuard(int device);
    ~DeviceGuard();

  private:
    int previous_ = -1;
    bool changed_ = false;
};

// Runs a kernel's one-time set-up (cudaFuncSetAttribute and the like) once per device: such
// attributes apply to the current device only, and several contexts of one process may sit on
// different devices. Thread-safe; a failed set-up is retried by the next call.
class PerDeviceOnce {
  public:
    template <typename Configure>
    cudaError_t run(Configure &&configure) {
        int device = 0;
        const cudaError_t error = cudaGetDevice(&device);
        if (error != cudaSuccess) return error;
        if (device < 0 || device >= kMaxDevices) return configure();
        const uint64_t bit = uint64_t{1} << device;
        if (done_.load(std::memory_order_acquire) & bit) return cudaSuccess;
        std::lock_guard<std::mutex> lock(mutex_);
        if (done_.load(std::memory_order_relaxed) & bit) return cudaSuccess;
        const cudaError_t result = configure();
        if (result == cudaSuccess) done_.fetch_or(bit, std::memory_order_release);
        return result;
    }

  private:
    static constexpr int kMaxDevices = 64;
    std::atomic<uint64_t> done_{0};
    std::mutex mutex_;
};

uint64_t monotonic_ns();
// Host memcpy split over several threads for large copies (pinned staging -> caller memory).
void parallel_memcpy(void *destination, const void *source, size_t bytes);
bool multiply_size(size_t left, size_t right, size_t *result);
bool valid_range(size_t total, size_t offset, size_t size);

// cuTensorMapEncodeTiled through the runtime's driver entry point (the library
// links only the static CUDA runtime, so it loads on machines without a driver).
bool encode_tensor_map_2d_u8(CUtensorMap *map, const void *base, uint64_t inner_bytes, uint64_t rows,
                             uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_rows);
// The same for 4-byte elements (fp32 / int32 outputs written by TMA stores), 128-byte swizzle.
bool encode_tensor_map_2d_b32(CUtensorMap *map, const void *base, uint64_t columns, uint64_t rows,
                              uint64_t row_stride_bytes, uint32_t box_columns, uint32_t box_rows);
// fp32 tiles without swizzle (scale boxes loaded next to swizzled operand tiles).
bool encode_tensor_map_2d_f32(CUtensorMap *map, const void *base, uint64_t columns, uint64_t rows,
                              uint64_t row_stride_bytes, uint32_t box_columns, uint32_t box_rows);

// ---- kernel launchers (one per .cu file) -------------------------------------------------

// Load (under CUDA's lazy module loading) and configure every kernel variant the row quantizer,
// the W8A8 GEMV and the tcgen05 GEMM launchers can pick, on the current device, and fill their
// cached occupancy figures, so later launches of them do no first-use set-up.
cudaError_t preload_quantize_rows_int8();
cudaError_t preload_w8a8_gemv();
cudaError_t preload_w8a8_gemm_sm100(int sm_count);

// Many long aligned rows take a bulk-copy staged kernel whose bounded waits report through
// error_word (the context's error word); with error_word null the register-cached kernel runs.
cudaError_t launch_quantize_rows_int8(const float *x, size_t x_stride, uint32_t rows, uint32_t cols,
                                      uint32_t padded_cols, int8_t *q, size_t q_stride, float *scales,
                                      unsigned int *error_word, cudaStream_t stream);
// Same quantizer over rows whose elements need not be contiguous: element (r, c) at
// (r / rows_per_batch) * batch_stride + (r % rows_per_batch) * row_stride + c * col_stride.
cudaError_t launch_quantize_rows_int8_layout(const float *x, uint32_t rows, uint32_t cols, uint32_t padded_cols,
                                             uint32_t rows_per_batch, size_t batch_stride, size_t row_stride,
                                             size_t col_stride, int8_t *q, size_t q_stride, float *scales,
                                             cudaStream_t stream);
cudaError_t launch_quantize_q8_0(const float *x, size_t x_stride, uint32_t rows, uint32_t cols, uint8_t *blocks,
                                 cudaStream_t stream);
// im2col of an NCHW fp32 tensor (row = output pixel, column = (channel, kernel row, kernel col)).
cudaError_t launch_im2col_nchw_f32(const float *source, uint32_t batch, uint32_t channels, uint32_t height,
                                   uint32_t width, uint32_t channel_offset, uint32_t group_channels,
                                   uint32_t kernel_height, uint32_t kernel_width, uint32_t stride_h,
                                   uint32_t stride_w, uint32_t pad_h, uint32_t pad_w, uint32_t dilation_h,
                                   uint32_t dilation_w, uint32_t output_height, uint32_t output_width,
                                   float *destination, size_t destination_stride, cudaStream_t stream);
cudaError_t launch_quantize_q4_0(const float *x, size_t x_stride, uint32_t rows, uint32_t cols, uint8_t *blocks,
                                 cudaStream_t stream);

enum class EpilogueMode : int { kStoreS32 = 0, kDequantize = 1, kDequantizeBias = 2 };

// Peer destinations one GEMM epilogue may write besides its own output (ranks of one node - 1).
constexpr uint32_t kGemmMaxPeers = 7;

struct GemmEpilogue {
    EpilogueMode mode = EpilogueMode::kDequantize;
    const float *row_scales = nullptr;
    const float *col_scales = nullptr;
    const float *bias = nullptr;
    void *out = nullptr;  // float* or int32_t*
    size_t out_stride = 0;  // elements
    // Other ranks' output buffers (mapped peer memory), each written at the same offsets as `out`.
    void *peer_out[kGemmMaxPeers] = {};
    uint32_t peer_count = 0;
    // Output (m, n) lies at (m / rows_per_batch) * batch_stride + (m % rows_per_batch) * out_stride
    // + n * col_stride elements from `out` (row-major by default; NCHW pixels-as-rows for convs).
    uint32_t rows_per_batch = 0xFFFFFFFFu;
    size_t batch_stride = 0;
    size_t col_stride = 1;
};

// tcgen05 int8 GEMM: a [m][k] and w [n][k] int8, K-major, 16-byte aligned rows. Tensor maps: A
// boxes of kGemmBlockK x kGemmBlockM, W boxes of kGemmBlockK x kGemmWeightBoxRows, 128-byte swizzle.
// Picks CTA pairs (tcgen05 cta_group::2, 256 x 256 tiles) when m spans two row blocks.
cudaError_t launch_w8a8_gemm_sm100(const CUtensorMap *map_a, const CUtensorMap *map_w, uint32_t m, uint32_t n,
                                   uint32_t k, const GemmEpilogue &epilogue, unsigned int *error_word,
                                   int sm_count, cudaStream_t stream);
// The same with the tile mode chosen by the caller (pair = CTA pairs).
cudaError_t launch_w8a8_gemm_sm100_mode(const CUtensorMap *map_a, const CUtensorMap *map_w, uint32_t m, uint32_t n,
                                        uint32_t k, const GemmEpilogue &epilogue, unsigned int *error_word,
                                        int sm_count, bool pair, cudaStream_t stream);
// Split-K for few output tiles (single-CTA tiles): the K stages are divided into `splits` slices
// (fewer if K is short; *used_splits says how many), and slice s writes its exact int32 partial
// rows to workspace rows [s * R, s * R + m), R = m rounded up to kGemmBlockM
// ([used_splits * R][n] int32, n a multiple of 4). launch_w8a8_splitk_reduce then adds the slices
// and applies the epilogue.
cudaError_t launch_w8a8_gemm_sm100_splitk(const CUtensorMap *map_a, const CUtensorMap *map_w, uint32_t m, uint32_t n,
                                          uint32_t k, int32_t *workspace, uint32_t splits, unsigned int *error_word,
                                          int sm_count, cudaStream_t stream, uint32_t *used_splits);
cudaError_t launch_w8a8_splitk_reduce(const int32_t *workspace, uint32_t splits, uint32_t m, uint32_t n,
                                      const GemmEpilogue &epilogue, int sm_count, cudaStream_t stream);
// Builds both tensor maps and launches; returns cudaErrorInvalidValue when a map cannot be encoded.
cudaError_t run_w8a8_gemm(const int8_t *a, size_t a_stride, const int8_t *w, size_t w_stride, uint32_t m,
                          uint32_t n, uint32_t k, const GemmEpilogue &epilogue, unsigned int *error_word,
                          int sm_count, cudaStream_t stream);
constexpr uint32_t kGemmBlockN = 256;  // box rows of the weight tensor map
constexpr uint32_t kGemmBlockM = 128;
constexpr uint32_t kGemmBlockK = 128;  // bytes of K per pipeline stage
constexpr uint32_t kGemmWeightBoxRows = 128;  // W rows per TMA box (a 256-row tile is two boxes)

cudaError_t launch_w8a8_gemv(const int8_t *a, size_t a_stride, const int8_t *w, size_t w_stride, uint32_t m,
                             uint32_t n, uint32_t k, const GemmEpilogue &epilogue, int sm_count,
                             cudaStream_t stream);
// One row, quantized by the GEMV itself: x[0 .. cols) fp32 -> int8 (every CTA into shared memory;
// CTA 0 also into q_out[0 .. k), zero padded, and *scale_out), then the dequantizing GEMV. Returns
// cudaErrorNotSupported (nothing launched) unless cols % 4 == 0, x is 16-byte and q_out 4-byte
// aligned and k <= 8192; the caller then runs the row quantizer and launch_w8a8_gemv.
cudaError_t launch_w8a8_gemv_quantize(const float *x, uint32_t cols, int8_t *q_out, float *scale_out, const int8_t *w,
                                      size_t w_stride, uint32_t n, uint32_t k, const GemmEpilogue &epilogue,
                                      int sm_count, cudaStream_t stream);
cudaError_t launch_w8a8_dequantize(const int32_t *acc, size_t acc_stride, uint32_t m, uint32_t n,
                                   const GemmEpilogue &epilogue, cudaStream_t stream);

// Q4_0 x Q8_0 over the prepared (repacked) weight layout.
struct Q40Weights {
    const uint8_t *nibbles = nullptr;  // [columns][blocks][16]
    const uint16_t *scales = nullptr;  // [columns][scale_stride] fp16 bits, zero padded
    uint32_t columns = 0;
    uint32_t blocks = 0;
    uint32_t scale_stride = 0;  // blocks rounded up to a multiple of 8 (16-byte rows)
    // Rows > 4 on sm_100 (the tcgen05 MX kernel), expanded once at prepare, or null: the codes as
    // int8 (code - 8) [columns][q4_0_mx_blocks_pad(blocks) * 32] and the fp32 scales block-major
    // [q4_0_mx_blocks_pad(blocks)][columns], both zero-padded.
    const int8_t *mx_values = nullptr;
    const float *mx_scales_t = nullptr;
};
uint32_t q4_0_mx_blocks_pad(uint32_t blocks);
// Fills the expanded MX operands above from the prepared nibbles and fp16 scales.
cudaError_t launch_q4_0_mx_expand(const uint8_t *nibbles, const uint16_t *scales, uint32_t columns, uint32_t blocks,
                                  uint32_t blocks_pad, uint32_t scale_stride, int8_t *values, float *scales_t,
                                  cudaStream_t stream);
// The tcgen05 MX kernel: split activation q (int8 [rows_pad][blocks_pad * 32]) and its scales
// da_t (fp32 [blocks_pad][rows_pad]) against the expanded weights; columns = resident columns.
cudaError_t launch_q4_0_mx_sm100(const int8_t *q, const float *da_t, uint32_t rows, uint32_t rows_pad,
                                 const int8_t *values, const float *scales_t, uint32_t columns, uint32_t blocks,
                                 uint32_t blocks_pad, float *destination, size_t destination_stride, uint32_t col0,
                                 uint32_t out_col0, uint32_t count, unsigned int *error_word, int sm_count,
                                 cudaStream_t stream);
// Whether a call of `rows` rows over `count` columns gives the tcgen05 MX kernel at least one tile
// per SM. Below that (few rows over a narrow window) each tile's block-serial K loop is the whole
// runtime, and the mma.sync kernel's smaller tiles spread the work over more SMs.
bool q4_0_mx_sm100_fills_wave(uint32_t rows, uint32_t count, int sm_count);
inline uint32_t q4_0_scale_stride(uint32_t blocks) { return (blocks + 7u) & ~7u; }
// activation: native Q8_0 rows [rows][blocks][34] (interleave 0) or CPU_REPACK
// block_q8_0x4 groups (interleave 4/8). Writes destination[r * stride + out_col0 + j]
// for weight columns col0 + j, j < count.
cudaError_t launch_q4_0_q8_0_gemv(const Q40Weights &weights, const uint8_t *activation, uint32_t rows,
                                  uint32_t interleave, float *destination, size_t destination_stride,
                                  uint32_t col0, uint32_t out_col0, uint32_t count, unsigned int *error_word,
                                  int sm_count, cudaStream_t stream);
// Same, with fp32 activation rows quantized to Q8_0 block by block while each CTA stages them
// (bit-identical to quantizing first and running the Q8_0 kernel, in one launch).
cudaError_t launch_q4_0_f32_gemv(const Q40Weights &weights, const float *source, size_t source_stride, uint32_t rows,
                                 float *destination, size_t destination_stride, uint32_t col0, uint32_t out_col0,
                                 uint32_t count, int sm_count, cudaStream_t stream);
// Rows > 4 (the reference's MX path) on the tensor cores: splits the activation (Q8_0 blocks, or
// fp32 rows quantized on the fly; exactly one of the two) into `scratch` of
// q4_0_mx_scratch_bytes(rows, blocks) bytes (16-byte aligned), then the tcgen05 kernel when the
// weights carry the expanded MX operands, else the tiled mma.sync kernel.
size_t q4_0_mx_scratch_bytes(uint32_t rows, uint32_t blocks);
cudaError_t launch_q4_0_mx(const Q40Weights &weights, const uint8_t *activation, const float *f32_source,
                           size_t f32_stride, uint32_t rows, uint32_t interleave, uint8_t *scratch, float *destination,
                           size_t destination_stride, uint32_t col0, uint32_t out_col0, uint32_t count,
                           unsigned int *error_word, int sm_count, cudaStream_t stream);
// Native 18-byte blocks [columns][blocks][18] -> prepared layout (scales rows of scale_stride,
// the padding must be zeroed beforehand).
cudaError_t launch_q4_0_repack(const uint8_t *native, uint32_t columns, uint32_t blocks, uint32_t scale_stride,
                               uint8_t *nibbles, uint16_t *scales, cudaStream_t stream);
// Reads native blocks directly (no prepared layout), for the single-kernel entry point.
cudaError_t launch_q4_0_q8_0_gemv_native(const uint8_t *activation, uint32_t rows, uint32_t blocks,
                                         const uint8_t *weight, float *destination, size_t destination_stride,
                                         uint32_t col0, uint32_t out_col0, uint32_t count, int sm_count,
                                         cudaStream_t stream);

}  // namespace qpucuda
