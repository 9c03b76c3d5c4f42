/*
 * GGML MUL_MAT (Q4_0 weight x F32 activation) offload core for a llama.cpp backend.
 *
 * The reference's backend (integrations/llama_cpp/backend/ggml-qpu.cpp) wraps its QPU
 * operator in ggml's backend interface. Everything it does for a MUL_MAT node outside that
 * interface is here, over a plain tensor view instead of ggml's headers (llama.cpp is not
 * part of this build):
 *   - the support predicate: supports_q4_0_mul_mat (ggml-qpu.cpp:362-377) plus the device's
 *     minimum/maximum row window (ggml-qpu.cpp:631-633);
 *   - the weight cache: get_or_prepare_linear (ggml-qpu.cpp:319-360), keyed by the weight
 *     tensor, re-prepared when a call needs more rows than the cached plan holds;
 *   - canonical Q4_0 input, including weights ggml-cpu repacked into block_q4_0x4 groups
 *     (unpack_q4_0_4x4, ggml-qpu.cpp:250-283);
 *   - the call itself: compute_q4_0_mul_mat (ggml-qpu.cpp:539-620). Where the reference
 *     quantizes the F32 rows to Q8_0 on the CPU first, this build copies the F32 rows to the
 *     device and quantizes them inside the matvec (rows <= 4) or the tensor-core tiled path
 *     (rows > 4); the destination is written only after a successful bounded wait.
 * The ggml glue a maintainer adds on top (backend/device/buffer-type registration and
 * graph_compute's node loop, which calls qpucuda_ggml_supports_mul_mat and
 * qpucuda_ggml_mul_mat per node) needs llama.cpp's own headers and is not part of this library.
 */
#ifndef QPUCUDA_GGML_H
#define QPUCUDA_GGML_H

#include "qpucuda_runtime.h"

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

/* ggml_type values the offload reads (ggml.h numbering). */
#define QPUCUDA_GGML_TYPE_F32 0
#define QPUCUDA_GGML_TYPE_Q4_0 2

/* The ggml_tensor fields the offload reads. `identity` is the key of the weight cache (the
 * ggml_tensor pointer in a backend; `data` when NULL). `cpu_repack` is 1 when the tensor lives
 * in ggml-cpu's CPU_REPACK buffer (Q4_0 weights stored as block_q4_0x4 groups). */
typedef struct qpucuda_ggml_tensor {
    int32_t type;
    int32_t cpu_repack;
    int64_t ne[4];
    size_t nb[4];
    void *data;
    const void *identity;
} qpucuda_ggml_tensor;

typedef struct qpucuda_ggml_backend qpucuda_ggml_backend;

/* Counters and the last call's host timings (monotonic ns), as the reference's candidate JSON
 * line reports them (ggml-qpu.cpp:581-616). */
typedef struct qpucuda_ggml_stats {
    uint64_t dispatch_count;
    uint64_t weight_cache_hits;
    uint64_t weight_cache_misses;
    uint64_t input_copy_ns;   /* host time to prepare/stage and issue the F32 rows' copy */
    uint64_t submit_wait_ns;  /* issue of the kernel and result copy + the bounded wait */
    uint64_t output_copy_ns;  /* pinned staging to the ggml destination */
    uint64_t complete_ns;     /* the whole call */
    uint32_t rows;            /* M of the last call */
} qpucuda_ggml_stats;

/* 1 when the node is a MUL_MAT this offload computes: weight Q4_0 [K, N, 1, 1] contiguous with
 * K % 32 == 0 and N % 16 == 0 (N % 4 as well when cpu_repack), activation F32 [K, M, 1, 1] contiguous with
 * minimum_rows <= M <= maximum_rows and M <= 4 * 65535, destination F32 [N, M] contiguous. */
int qpucuda_ggml_supports_mul_mat(const qpucuda_ggml_tensor *weight, const qpucuda_ggml_tensor *activation,
                                  const qpucuda_ggml_tensor *destination, uint32_t minimum_rows,
                                  uint32_t maximum_rows);

/* block_q4_0x4 groups (4 weight rows per group, per K block: the 4 fp16 scales, then 64 quant
 * bytes as chunk x row x 4 bytes, each byte XOR 0x88) back to native block_q4_0 rows
 * [N][K/32][18]. Host only; returns QPUCUDA_INVALID_ARGUMENT on a size or shape mismatch. */
qpucuda_status qpucuda_ggml_unpack_q4_0x4(const void *packed, size_t packed_size, uint32_t input_columns,
                                          uint32_t output_columns, void *native, size_t native_size);

qpucuda_status qpucuda_ggml_backend_create(qpucuda_context *context, uint32_t minimum_rows, uint32_t maximum_rows,
                                           qpucuda_ggml_backend **result);
/* Frees every cached plan and the staging; NULL-safe. */
void qpucuda_ggml_backend_destroy(qpucuda_ggml_backend *backend);
/* compute_q4_0_mul_mat for one node: destination = activation x weight^T, fp32. Unsupported
 * nodes return QPUCUDA_INVALID_ARGUMENT (the reference fails graph_compute for them). */
qpucuda_status qpucuda_ggml_mul_mat(qpucuda_ggml_backend *backend, const qpucuda_ggml_tensor *weight,
                                    const qpucuda_ggml_tensor *activation, qpucuda_ggml_tensor *destination);
/* Drops the cached plan of a weight (when its buffer is freed or rewritten); no-op if absent.
 * No counterpart in the reference, whose cache lives as long as the backend. */
void qpucuda_ggml_backend_forget(qpucuda_ggml_backend *backend, const void *identity);
qpucuda_status qpucuda_ggml_backend_stats(const qpucuda_ggml_backend *backend, qpucuda_ggml_stats *result);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif
#ifdef __cplusplus
}
#endif

#endif /* QPUCUDA_GGML_H */
