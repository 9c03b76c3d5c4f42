/*
 * Prepared GGML Q4_0 x Q8_0 linear on one CUDA device.
 *
 * Drop-in for integrations/llama_cpp/include/qpu_llama_q4_0.h:13-82: the same
 * functions, descriptors, argument rules and status codes, with the QPU
 * program replaced by an sm_100a CUDA kernel. Differences that a caller sees:
 *   - expected_source_hash is checked against qpucuda_q4_0_kernel_source_hash()
 *     (the SHA-256 of this library's kernel source), not a QPU program hash;
 *   - rows 1..4 run the decode matvec; rows 5..4*65535 run the tiled tensor-core
 *     path (the reference's MX path, qpu_llama_q4_0.c:238-290) with the exact
 *     per-block scaling of its program, ((float)dot * d_a) * d_w added block by
 *     block; prepare then also reserves the split-activation scratch;
 *   - weight_mode must be EXACT: the re-quantized COLUMN_W8 / ROWCOL_W8A8 modes
 *     (rows > 4 only in the reference, qpu_llama_q4_0.c:217-219) return
 *     QPUCUDA_CAPABILITY_MISSING;
 *   - workgroups_per_supergroup is a QPU dispatch knob and is ignored;
 *   - submission_cpu_fallback returns QPUCUDA_INVALID_ARGUMENT for rows <= 4,
 *     exactly as the reference does (qpu_llama_q4_0.c:834-839), and
 *     QPUCUDA_CAPABILITY_MISSING for rows > 4, where the reference would compute
 *     on the host: this library has no CPU path.
 *
 * Host pointers: desc->weights, execution->activation and
 * execution->destination are host memory, as in the reference. The
 * *_device entry points take device pointers and run asynchronously on the
 * context stream with no host copies.
 */
#ifndef QPUCUDA_Q4_0_H
#define QPUCUDA_Q4_0_H

#include "qpucuda_runtime.h"

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

typedef struct qpucuda_q4_0_linear qpucuda_q4_0_linear;
typedef struct qpucuda_q4_0_submission qpucuda_q4_0_submission;

/* qpu_llama_q4_0_weight_mode (qpu_llama_q4_0.h:16-20). */
typedef enum qpucuda_q4_0_weight_mode {
    QPUCUDA_Q4_0_WEIGHT_EXACT = 0,
    QPUCUDA_Q4_0_WEIGHT_COLUMN_W8 = 1,
    QPUCUDA_Q4_0_WEIGHT_ROWCOL_W8A8 = 2,
} qpucuda_q4_0_weight_mode;

/* qpu_llama_q4_0_linear_desc (qpu_llama_q4_0.h:22-33). weights: host,
 * native block_q4_0 rows [output_columns][input_columns/32][18 bytes];
 * only the resident column window is copied to the device. */
typedef struct qpucuda_q4_0_linear_desc {
    const void *weights;
    size_t weight_size;
    uint32_t input_columns;          /* K, multiple of 32 */
    uint32_t output_columns;         /* N of the full matrix */
    uint32_t rows;                   /* maximum M per call, 1..4*65535 */
    uint32_t resident_column_start;  /* multiple of 16 */
    uint32_t resident_column_count;  /* multiple of 16, > 0 */
    qpucuda_q4_0_weight_mode weight_mode;
    uint32_t workgroups_per_supergroup; /* ignored */
    const char *expected_source_hash;   /* must equal qpucuda_q4_0_kernel_source_hash() */
} qpucuda_q4_0_linear_desc;

/* qpu_llama_q4_0_execution (qpu_llama_q4_0.h:35-48). activation: host native
 * block_q8_0 rows [rows][K/32][34 bytes] (or CPU_REPACK block_q8_0x4 groups
 * when activation_interleave is 4 or 8); destination: host fp32
 * [rows][output_columns]; only columns [column_start, column_start +
 * column_count) are written. */
typedef struct qpucuda_q4_0_execution {
    const void *activation;
    size_t activation_size;
    size_t activation_offset;
    void *destination;
    size_t destination_size;
    size_t destination_offset;
    uint32_t column_start;
    uint32_t column_count;
    uint32_t rows;                  /* 0 = the prepared row capacity */
    uint32_t activation_interleave; /* 0, 4 or 8 */
} qpucuda_q4_0_execution;

/* qpu_llama_q4_0_timing (qpu_llama_q4_0.h:50-61); host monotonic ns. */
typedef struct qpucuda_q4_0_timing {
    uint64_t input_access_ns;
    uint64_t input_pack_ns;
    uint64_t input_sync_ns;
    uint64_t input_copy_ns;
    uint64_t submit_ns;
    uint64_t wait_ns;
    uint64_t submit_wait_ns;
    uint64_t output_sync_ns;
    uint64_t output_copy_ns;
    uint64_t complete_ns;
} qpucuda_q4_0_timing;

/* qpu_llama_q4_0_linear_prepare (qpu_llama_q4_0.h:63-66). */
qpucuda_status qpucuda_q4_0_linear_prepare(
    qpucuda_context *context,
    const qpucuda_q4_0_linear_desc *desc,
    qpucuda_q4_0_linear **result);
/* qpu_llama_q4_0_linear_destroy (qpu_llama_q4_0.h:67); NULL-safe. */
void qpucuda_q4_0_linear_destroy(qpucuda_q4_0_linear *linear);
/* qpu_llama_q4_0_linear_execute (qpu_llama_q4_0.h:68-71): submit + wait. */
qpucuda_status qpucuda_q4_0_linear_execute(
    qpucuda_q4_0_linear *linear,
    const qpucuda_q4_0_execution *execution,
    qpucuda_q4_0_timing *timing);
/* qpu_llama_q4_0_linear_submit (qpu_llama_q4_0.h:72-75). One submission in
 * flight per linear (a second returns QPUCUDA_INTERNAL_ERROR). */
qpucuda_status qpucuda_q4_0_linear_submit(
    qpucuda_q4_0_linear *linear,
    const qpucuda_q4_0_execution *execution,
    qpucuda_q4_0_submission **result);
/* qpu_llama_q4_0_submission_wait (qpu_llama_q4_0.h:76-78): bounded wait,
 * then the column window is copied to the host destination. On a failed
 * wait the destination is left untouched and the context is poisoned. */
qpucuda_status qpucuda_q4_0_submission_wait(
    qpucuda_q4_0_submission *submission,
    qpucuda_q4_0_timing *timing);
/* qpu_llama_q4_0_submission_cpu_fallback (qpu_llama_q4_0.h:79-80): never
 * computes (no CPU path; see the file comment). */
qpucuda_status qpucuda_q4_0_submission_cpu_fallback(qpucuda_q4_0_submission *submission);
/* qpu_llama_q4_0_submission_destroy (qpu_llama_q4_0.h:81); NULL-safe, waits if active. */
void qpucuda_q4_0_submission_destroy(qpucuda_q4_0_submission *submission);
/* qpu_llama_q4_0_linear_resident_bytes (qpu_llama_q4_0.h:82). */
size_t qpucuda_q4_0_linear_resident_bytes(const qpucuda_q4_0_linear *linear);

/* Device-pointer form of execute, asynchronous on the context stream, no
 * host copies (the path the Python operator and bench use).
 * activation: device native Q8_0 rows [rows][K/32][34]; destination: device
 * fp32, row stride destination_stride elements. Weight column column_start + j
 * (j < column_count, inside the resident window) is written to destination
 * column output_column_start + j, the weight/output column split of the
 * reference's kernel handle (ggml_q4_0.py:725-761). No counterpart in the
 * reference's C ABI (its buffers are host-mapped). */
qpucuda_status qpucuda_q4_0_linear_execute_device(
    qpucuda_q4_0_linear *linear,
    const void *activation,
    uint32_t rows,
    float *destination,
    size_t destination_stride,
    uint32_t column_start,
    uint32_t column_count,
    uint32_t output_column_start);

/* Fused device path: fp32 activations [rows][K] (row stride source_stride)
 * are quantized to Q8_0 on the device and multiplied in the same call
 * (the reference quantizes on the CPU per call, ggml-qpu.cpp:552-560). */
qpucuda_status qpucuda_q4_0_linear_execute_f32_device(
    qpucuda_q4_0_linear *linear,
    const float *source,
    size_t source_stride,
    uint32_t rows,
    float *destination,
    size_t destination_stride,
    uint32_t column_start,
    uint32_t column_count,
    uint32_t output_column_start);

/* SHA-256 (hex) of the kernel source this library was built from; the value
 * qpucuda_q4_0_linear_desc.expected_source_hash must carry. Replaces the
 * generated qpu_ggml_q4_0_q8_0_m{1,4}_source_hash constants. */
const char *qpucuda_q4_0_kernel_source_hash(void);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif
#ifdef __cplusplus
}
#endif

#endif
