/*
 * qpucuda runtime: the CUDA (sm_100a) context behind the quantized-linear
 * operators. It replaces the reference's DRM/V3D runtime ABI
 * (integrations/llama_cpp/include/qpu_llama_runtime.h:16-133) for the
 * operators this library exports. Status codes, the failure-injection mask,
 * the wait timeout and the "poisoned after a failed wait" rule keep the
 * reference's numbering and meaning so that callers written against the
 * reference can keep their error handling.
 *
 * Memory: every pointer argument documented as "host" is ordinary host memory
 * (the library copies it through its own pinned staging); every pointer
 * documented as "device" is CUDA device memory on the context's device.
 * Work is issued on the context's stream (cudaStream_t passed as void*).
 */
#ifndef QPUCUDA_RUNTIME_H
#define QPUCUDA_RUNTIME_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

typedef struct qpucuda_context qpucuda_context;

/* Same values and meanings as qpu_llama_status (qpu_llama_runtime.h:16-27). */
typedef enum qpucuda_status {
    QPUCUDA_OK = 0,
    QPUCUDA_INVALID_ARGUMENT = 1,
    QPUCUDA_DEVICE_UNAVAILABLE = 2,
    QPUCUDA_CAPABILITY_MISSING = 3,
    QPUCUDA_ALLOCATION_FAILED = 4,
    QPUCUDA_IO_FAILED = 5,
    QPUCUDA_SUBMISSION_FAILED = 6,
    QPUCUDA_TIMEOUT = 7,
    QPUCUDA_HASH_MISMATCH = 8,
    QPUCUDA_INTERNAL_ERROR = 9,
} qpucuda_status;

/* Host-side fault injection, same bits as qpu_llama_failure_point
 * (qpu_llama_runtime.h:29-36). Injection happens on the host before the
 * corresponding CUDA call; nothing is ever injected into a kernel. */
typedef enum qpucuda_failure_point {
    QPUCUDA_FAIL_NONE = 0,
    QPUCUDA_FAIL_DEVICE_OPEN = 1U << 0,
    QPUCUDA_FAIL_ALLOCATION = 1U << 1,
    QPUCUDA_FAIL_SUBMISSION = 1U << 2,
    QPUCUDA_FAIL_WAIT = 1U << 3,
    QPUCUDA_FAIL_SOURCE_HASH = 1U << 4,
} qpucuda_failure_point;

/* Replaces qpu_llama_context_config (qpu_llama_runtime.h:44-48): the render
 * node becomes a CUDA device ordinal, and an optional caller stream. */
typedef struct qpucuda_context_config {
    int32_t device_ordinal;  /* CUDA device; -1 = the calling thread's current device */
    uint64_t timeout_ns;     /* bounded host wait; 0 = 10 s default, as the reference */
    uint32_t failure_mask;   /* qpucuda_failure_point bits */
    void *stream;            /* cudaStream_t to issue on; NULL = a library-owned non-blocking stream */
} qpucuda_context_config;

/* Replaces qpu_llama_capabilities (qpu_llama_runtime.h:50-60). */
typedef struct qpucuda_capabilities {
    char device_name[128];
    int32_t device_ordinal;
    int32_t compute_capability_major;
    int32_t compute_capability_minor;
    int32_t multiprocessor_count;
    uint64_t global_memory_bytes;
    uint64_t l2_cache_bytes;
    uint8_t supports_tcgen05; /* 1 when the device is sm_100 (the int8 tensor-core GEMM can run) */
} qpucuda_capabilities;

/* qpu_llama_context_create (qpu_llama_runtime.h:85-87). config may be NULL. */
qpucuda_status qpucuda_context_create(const qpucuda_context_config *config, qpucuda_context **result);
/* qpu_llama_context_destroy; NULL-safe. Waits (bounded) for the context's work first. */
void qpucuda_context_destroy(qpucuda_context *context);
/* qpu_llama_context_last_error (qpu_llama_runtime.h:89). */
const char *qpucuda_context_last_error(const qpucuda_context *context);
/* qpu_llama_context_capabilities (qpu_llama_runtime.h:90-92). */
qpucuda_status qpucuda_context_capabilities(const qpucuda_context *context, qpucuda_capabilities *result);
/* qpu_llama_context_set_failure_mask (qpu_llama_runtime.h:93). */
void qpucuda_context_set_failure_mask(qpucuda_context *context, uint32_t failure_mask);
/* Re-target the context at another stream of the same device. The value is a
 * cudaStream_t with CUDA's meaning: NULL is the legacy default stream (the
 * stream PyTorch reports as 0). */
qpucuda_status qpucuda_context_set_stream(qpucuda_context *context, void *stream);
void *qpucuda_context_stream(const qpucuda_context *context);
/* The library-owned non-blocking stream (what a NULL config->stream selects at creation). */
void *qpucuda_context_library_stream(const qpucuda_context *context);
/* Bounded wait for all work issued on the context stream, then the kernels'
 * device-side error word is checked. A timeout or a kernel-reported error
 * poisons the context (as qpu_llama_submission_wait does,
 * qpu_llama_runtime.c:688-727); a poisoned context rejects new work with
 * QPUCUDA_IO_FAILED. */
qpucuda_status qpucuda_context_synchronize(qpucuda_context *context);
/* 1 when a failed wait poisoned the context. */
int qpucuda_context_poisoned(const qpucuda_context *context);

/* Device-side check of the wait-expiry path. Launches one CTA on the context
 * stream that waits, bounded by wait_limit_ns (1 .. 1e9 ns), on an mbarrier
 * nothing arrives at -- the same bounded wait every tcgen05 / bulk-copy barrier
 * wait of this library uses -- so the wait runs out, the kernel records the
 * expiry in the context's error word and returns. The call then waits for the
 * stream as every operator does and returns what an operator whose kernel wait
 * expired returns: QPUCUDA_TIMEOUT, with the context poisoned. No fault, trap or
 * unbounded wait is involved, so the CUDA device stays usable and a new context
 * on it runs normally. The reference checks this path only by host injection
 * (QPU_LLAMA_FAIL_WAIT, integrations/llama_cpp/tests/
 * qpu_llama_native_safety_smoke.c:655-669; poisoning at qpu_llama_runtime.c:616-619);
 * this entry point has no counterpart in its C API. */
qpucuda_status qpucuda_context_probe_wait_expiry(qpucuda_context *context, uint64_t wait_limit_ns);

/* qpu_llama_status_string (qpu_llama_runtime.h:133). */
const char *qpucuda_status_string(qpucuda_status status);
/* Library build identity: "<version> sm_100a". */
const char *qpucuda_build_info(void);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif
#ifdef __cplusplus
}
#endif

#endif
