/*
 * Peer memory and the fused W8A8 linear + all-gather for the output-channel (N)
 * split across the GPUs of one node (one process per GPU).
 *
 * No counterpart in the reference: its CPU/QPU output split
 * (src/qpu_xla/models/tinyllama/quantization.py:350-514, execute_hybrid) runs the
 * two column ranges on one host and joins them in host memory. Here each rank
 * keeps a full [rows][N] fp32 output in device memory that every other rank maps
 * (CUDA IPC), and the GEMM epilogue stores each finished tile of the rank's
 * columns into all of them over NVLink, so the exchange overlaps the main loop
 * tile by tile instead of following it as a separate all-gather.
 *
 * Ordering: after a fan-out execute, a peer's buffer holds this rank's columns
 * once this rank's kernel has completed. Callers therefore follow the launches
 * of all ranks with one collective on the same streams (e.g. a one-element NCCL
 * all-reduce) before reading the full output, and do not start the next fan-out
 * into a buffer until every rank has finished reading it.
 */
#ifndef QPUCUDA_PEER_H
#define QPUCUDA_PEER_H

#include "qpucuda_runtime.h"
#include "qpucuda_w8a8.h"

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

#define QPUCUDA_PEER_HANDLE_BYTES 64u /* sizeof(cudaIpcMemHandle_t) */
#define QPUCUDA_MAX_PEERS 7u          /* other ranks of one 8-GPU node */

/* Allocates `bytes` of device memory on the context's device that other processes
 * can map, and writes the QPUCUDA_PEER_HANDLE_BYTES handle to send them.
 * QPUCUDA_ALLOCATION_FAILED when the memory or the handle cannot be had. */
qpucuda_status qpucuda_peer_buffer_create(qpucuda_context *context, size_t bytes, void **device_pointer,
                                          unsigned char *handle);

/* Maps another process's buffer (its handle) into this context; the pointer is
 * valid in kernels and copies on this context's device. QPUCUDA_CAPABILITY_MISSING
 * when the mapping is refused (no peer access between the two devices). */
qpucuda_status qpucuda_peer_buffer_open(qpucuda_context *context, const unsigned char *handle,
                                        void **device_pointer);

/* Unmaps a buffer opened with qpucuda_peer_buffer_open. */
qpucuda_status qpucuda_peer_buffer_close(qpucuda_context *context, void *device_pointer);

/* Frees a buffer made by qpucuda_peer_buffer_create. Every process that opened it
 * must have closed it, or at least stopped writing to it, first. */
qpucuda_status qpucuda_peer_buffer_destroy(qpucuda_context *context, void *device_pointer);

/* qpucuda_w8a8_linear_execute_device that also writes the same fp32 outputs
 * [rows][resident columns] to `peer_count` further destinations at the same
 * offsets: out[r * destination_stride + c] for `destination` and for every
 * peer_destinations[p] (normally this rank's column slice of each other rank's
 * mapped full output). Asynchronous on the context stream. peer_count 0 is the
 * plain device execute. QPUCUDA_INVALID_ARGUMENT for more than
 * QPUCUDA_MAX_PEERS peers or a NULL pointer. */
qpucuda_status qpucuda_w8a8_linear_execute_device_fanout(qpucuda_w8a8_linear *linear, const float *source,
                                                         size_t source_stride, uint32_t rows, float *destination,
                                                         float *const *peer_destinations, uint32_t peer_count,
                                                         size_t destination_stride);

/* Copies a block of `rows` rows of `width_bytes` bytes from `source` (rows
 * `source_pitch` bytes apart) to `destination` (rows `destination_pitch` bytes
 * apart) with the copy engines, asynchronously on `stream` (a cudaStream_t of the
 * context's device; NULL for the context stream). With `destination` a mapped
 * peer buffer (qpucuda_peer_buffer_open) this pushes a column block of this
 * rank's output to another rank over NVLink without occupying the SMs: the
 * exchange of the N-split done by DMA instead of by the GEMM epilogue's stores.
 * No counterpart in the reference (its output split joins in host memory).
 * QPUCUDA_INVALID_ARGUMENT for NULL pointers, a zero size or pitches below the
 * width. */
qpucuda_status qpucuda_peer_copy_rows(qpucuda_context *context, void *destination, size_t destination_pitch,
                                      const void *source, size_t source_pitch, size_t width_bytes, size_t rows,
                                      void *stream);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif
#ifdef __cplusplus
}
#endif

#endif /* QPUCUDA_PEER_H */
