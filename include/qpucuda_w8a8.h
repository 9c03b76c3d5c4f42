/*
 * Prepared dynamic W8A8 linear on one CUDA device.
 *
 * The reference exposes this operator only in Python:
 * PreparedW8A8Linear (src/qpu_xla/models/tinyllama/quantization.py:57-878),
 * whose QPU dispatch goes through the raw program ABI
 * (integrations/llama_cpp/include/qpu_llama_runtime.h:114-131 with the
 * tiled-w8a8-gemm[-dequantize] and w8a8-gemv programs). This header is the
 * C-ABI form of that plan, with the same contract:
 *   y[m, n] = ((float)acc[m, n] * s_a[m]) * s_w[n]   (+ bias[n] when given)
 *   acc[m, n] = sum_k q_a[m, k] * q_w[n, k]          exact int32
 *   s_a[m] = max(max_k |x[m, k]| / 127, 1/127),  q_a = clip(rint(x / s_a), -127, 127)
 * (quantization.py:156-171 and :1065-1075; bias after dequantization as in
 * src/qpu_xla/models/smolvla/accelerated.py:260-261).
 *
 * The plan owns the resident int8 weights, scales, bias and the activation
 * scratch (int8 rows padded to a multiple of 16 bytes plus fp32 row scales),
 * sized for max_batch rows. One invocation may be in flight per plan
 * (quantization.py:290-291); a second concurrent execute returns
 * QPUCUDA_INTERNAL_ERROR.
 *
 * Output-channel (N) sharding: resident_output_start/count select a disjoint
 * column range of the weight; the destination then receives only those
 * columns (the multi-GPU N-split, and the reference's execute_hybrid output
 * split, quantization.py:350-514).
 */
#ifndef QPUCUDA_W8A8_H
#define QPUCUDA_W8A8_H

#include "qpucuda_runtime.h"

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

typedef struct qpucuda_w8a8_linear qpucuda_w8a8_linear;

typedef enum qpucuda_memory {
    QPUCUDA_MEMORY_HOST = 0,
    QPUCUDA_MEMORY_DEVICE = 1,
} qpucuda_memory;

/* Weight descriptor; the fields are QuantizedMatrixInt8 (quantization.py:31-54)
 * plus an optional bias. Pointers are host or device memory per `memory`;
 * they are only read during prepare (copied into the plan). */
typedef struct qpucuda_w8a8_linear_desc {
    const int8_t *weight_values;   /* [output_features][input_features] row-major */
    const float *weight_scales;    /* [output_features], finite and > 0 */
    const float *bias;             /* [output_features] or NULL */
    uint32_t input_features;       /* K */
    uint32_t output_features;      /* N of the full matrix */
    uint32_t max_batch;            /* maximum M per call, > 0 */
    uint32_t resident_output_start;  /* first resident output column */
    uint32_t resident_output_count;  /* 0 = all columns from resident_output_start */
    qpucuda_memory memory;
} qpucuda_w8a8_linear_desc;

/* Host-buffer execution, synchronous (bounded wait). source: host fp32
 * [rows][input_features]; destination: host fp32 [rows][resident count]. */
typedef struct qpucuda_w8a8_execution {
    const float *source;
    size_t source_size;           /* bytes available at source */
    float *destination;
    size_t destination_size;      /* bytes available at destination */
    uint32_t rows;                /* 1..max_batch */
} qpucuda_w8a8_execution;

qpucuda_status qpucuda_w8a8_linear_prepare(
    qpucuda_context *context,
    const qpucuda_w8a8_linear_desc *desc,
    qpucuda_w8a8_linear **result);
void qpucuda_w8a8_linear_destroy(qpucuda_w8a8_linear *linear);
size_t qpucuda_w8a8_linear_resident_bytes(const qpucuda_w8a8_linear *linear);
/* Host buffers in and out; copies through pinned staging; on a failed wait
 * the destination is left untouched and the context is poisoned. Batches of
 * more than 1024 rows are pipelined in 1024-row slices (host-to-device copy,
 * GEMM and device-to-host copy overlap); the destination is written only after
 * the wait for the whole call has succeeded. */
qpucuda_status qpucuda_w8a8_linear_execute(qpucuda_w8a8_linear *linear, const qpucuda_w8a8_execution *execution);

/* qpucuda_w8a8_linear_execute for a destination in page-locked host memory
 * (cudaMallocHost, cudaHostAlloc or cudaHostRegister over the whole range;
 * otherwise QPUCUDA_INVALID_ARGUMENT): the device-to-host copies write the
 * results straight into it, overlapping the kernels, with no staging copy on
 * the host. The price is the failure rule: after a failed or timed-out wait the
 * destination may hold part of the results (the staged entry point above leaves
 * it untouched, as the reference's Q4_0 operator does). No counterpart in the
 * reference, whose W8A8 operator has no C form. */
qpucuda_status qpucuda_w8a8_linear_execute_direct(qpucuda_w8a8_linear *linear,
                                                  const qpucuda_w8a8_execution *execution);

/* Asynchronous form of qpucuda_w8a8_linear_execute_direct: the copies and
 * kernels are queued and the call returns at once with a submission handle.
 * Batches above 1024 rows leave their device-to-host copies on the plan's own
 * copy stream, so the host-to-device copies and kernels of a submission on
 * another plan of the same context overlap them (e.g. the projections of one
 * layer). The source and the page-locked destination must stay valid and
 * untouched until qpucuda_w8a8_submission_wait returns; the plan accepts no
 * other call until then (QPUCUDA_INTERNAL_ERROR). The wait is bounded by the
 * context timeout and has the same failure rule as the direct entry point
 * (TIMEOUT poisons the context; the destination may hold part of the results).
 * No counterpart in the reference, whose W8A8 operator has no C form. */
typedef struct qpucuda_w8a8_submission qpucuda_w8a8_submission;
qpucuda_status qpucuda_w8a8_linear_submit_direct(qpucuda_w8a8_linear *linear, const qpucuda_w8a8_execution *execution,
                                                 qpucuda_w8a8_submission **submission);
/* Waits (bounded) for a submission; calling it again returns the same status. */
qpucuda_status qpucuda_w8a8_submission_wait(qpucuda_w8a8_submission *submission);
/* Frees a submission, waiting for it first if it was not waited for. */
void qpucuda_w8a8_submission_destroy(qpucuda_w8a8_submission *submission);

/* Device pointers, asynchronous on the context stream:
 * quantize source rows into the plan scratch, GEMM (tcgen05 kind::i8 for
 * rows > 8, int8 dot-product GEMV otherwise), fused dequant (+ bias) into
 * destination[row * destination_stride + column], columns 0..resident count-1. */
qpucuda_status qpucuda_w8a8_linear_execute_device(
    qpucuda_w8a8_linear *linear,
    const float *source,
    size_t source_stride,
    uint32_t rows,
    float *destination,
    size_t destination_stride);

/* Same, for activations already quantized by the caller (the reference's
 * execute_prepared, quantization.py:325-348): quantized int8 rows with row
 * stride quantized_stride bytes (multiple of 16) and fp32 row scales. */
qpucuda_status qpucuda_w8a8_linear_execute_prepared_device(
    qpucuda_w8a8_linear *linear,
    const int8_t *quantized,
    size_t quantized_stride,
    const float *row_scales,
    uint32_t rows,
    float *destination,
    size_t destination_stride);

/* A matrix view over device memory: element (r, c) lies at
 *   (r / rows_per_batch) * batch_stride + (r % rows_per_batch) * row_stride + c * column_stride
 * elements from the base pointer (rows_per_batch 0 = all rows in one batch).
 * Row-major [rows][ld] is {0, 0, ld, 1}; an NCHW tensor seen as pixels x channels
 * (the reference's pointwise lowering, src/qpu_xla/ops/conv2d.py:93-96) is
 * {H*W, C*H*W, 1, H*W} with the base at channel 0 of the range used. */
typedef struct qpucuda_matrix_layout {
    uint64_t rows_per_batch;
    uint64_t batch_stride;
    uint64_t row_stride;
    uint64_t column_stride;
} qpucuda_matrix_layout;

/* qpucuda_w8a8_linear_execute_device over arbitrary source and destination layouts
 * (source: rows x input features, destination: rows x resident columns). Used by the
 * W8A8 convolution plan to read NCHW pixels and write NCHW outputs in place, with no
 * transpose copies. Non row-major destinations always take the tcgen05 GEMM path. */
qpucuda_status qpucuda_w8a8_linear_execute_device_layout(
    qpucuda_w8a8_linear *linear,
    const float *source, const qpucuda_matrix_layout *source_layout, uint32_t rows,
    float *destination, const qpucuda_matrix_layout *destination_layout);

/* Read back the plan scratch after an execute (device pointers, valid until
 * the next call): int8 activations [max_batch][padded K] and fp32 row scales. */
qpucuda_status qpucuda_w8a8_linear_scratch(
    const qpucuda_w8a8_linear *linear,
    const int8_t **quantized,
    size_t *quantized_stride,
    const float **row_scales);

/* Size of the fixed device scratch used by qpucuda_w8a8_linear_execute_static
 * (16 MiB per GPU, reserved when the library's module is loaded on that GPU --
 * at the latest by the entry point's first call there -- and held until the
 * process exits). */
#define QPUCUDA_STATIC_SCRATCH_BYTES (16u * 1024u * 1024u)

/* W8A8 linear that allocates nothing. This entry point has no counterpart in
 * the reference; it exists for callers that cannot call cudaMalloc (or any
 * allocating routine) when they run the operator -- code running inside an
 * allocator callback it must not re-enter, or under a device-memory budget
 * fixed at start-up -- and so cannot use a prepared linear, which allocates
 * its activation scratch.
 *
 * Computes, on the context stream, the same result as a prepared linear:
 *   destination[m, n] = ((float)acc[m, n] * s_a[m]) * weight_scales[n] (+ bias[n])
 * with the activations quantized per row. The caller passes every input and
 * output in device memory: source fp32 [rows][k] (row stride source_stride
 * elements), weight int8 [n][weight_stride bytes] (16-byte aligned rows, the K
 * values zero-padded up to a multiple of 16), weight_scales fp32 [n], bias fp32
 * [n] or NULL, destination fp32 (row stride destination_stride elements).
 *
 * The quantized activations live in one fixed device array compiled into the
 * library: rows * (k rounded up to 16) bytes, rounded up to 256, plus 4 * rows
 * bytes must fit in QPUCUDA_STATIC_SCRATCH_BYTES (e.g. 1024 rows at k = 8192);
 * larger requests return QPUCUDA_INVALID_ARGUMENT with the reason in
 * qpucuda_context_last_error. No cudaMalloc, cudaFree or allocating library
 * routine is called.
 *
 * The first call on each device (in each CUDA context of it) is the set-up: it
 * looks up the array's device address (cudaGetSymbolAddress, with that device
 * current) and loads and configures every kernel this entry point can launch.
 * Under CUDA's lazy module loading that set-up can allocate device memory, so
 * make the first call at start-up: outside any region where allocation is
 * forbidden, and before any stream capture. Later calls allocate nothing. After
 * a device reset the next call repeats the set-up. All calls share the one
 * array and it keeps the last call's contents; each call rewrites every byte it
 * later reads, so nothing needs clearing, but calls whose work overlaps on the
 * GPU (different streams, or different contexts on one device) race on the
 * array. */
qpucuda_status qpucuda_w8a8_linear_execute_static(
    qpucuda_context *context,
    const float *source,
    size_t source_stride,
    uint32_t rows,
    const int8_t *weight,
    size_t weight_stride,
    const float *weight_scales,
    const float *bias,
    uint32_t k,
    uint32_t n,
    float *destination,
    size_t destination_stride);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif
#ifdef __cplusplus
}
#endif

#endif
