"""CUDA kernel handles of the quantized-linear path and their ``supports_*`` contracts.

Each handle is the CUDA counterpart of one reference ``Kernel`` object
(src/qpu_xla/kernels/__init__.py:22-58) and is submitted the same way,
``queue.submit(KERNEL, args, wait_for=..., buffers=...)``. Arguments are
:class:`~qpu_xla.memory.Tensor` views on a CUDA device; the executor launches
one libqpucuda entry point (include/qpucuda_kernels.h) on the queue's stream.

Operand layout difference from the reference: the reference packs four int8 K
values per uint32 and transposes the weight to ``[K/4, N]``
(gemm_int8.py:23-40). Here the weight stays ``[N, K]`` int8 rows (the
``QuantizedMatrixInt8.values`` layout, K contiguous), which is the K-major
operand layout the tensor-memory-accelerator and tcgen05 consume directly; K
rows are padded with zeros to a multiple of 16 bytes.

``supports_*`` predicates return a bool and never raise (gemm_int8.py:224-268).
"""

from __future__ import annotations

from typing import Any

import numpy as np

from qpu_xla.errors import KernelError
from qpu_xla.kernel import Kernel
from qpu_xla.memory import Tensor

Q4_0_BLOCK_ELEMENTS = 32
Q4_0_BLOCK_BYTES = 18
Q8_0_BLOCK_BYTES = 34
OUTPUT_TILE = 16
INT32_LIMIT = np.iinfo(np.int32).max


def _is_cuda(tensor: Tensor) -> bool:
    return bool(getattr(tensor.buffer.device, "is_cuda", False))


def _rows_aligned(tensor: Tensor) -> bool:
    """Rank-2, unit inner stride, 16-byte aligned base and row stride."""
    return (
        len(tensor.shape) == 2
        and tensor.strides[1] == tensor.dtype.itemsize
        and tensor.address % 16 == 0
        and tensor.strides[0] % 16 == 0
    )


def _row_major(tensor: Tensor) -> bool:
    return len(tensor.shape) == 2 and tensor.strides[1] == tensor.dtype.itemsize


def _vector(tensor: Tensor, length: int, dtype: Any) -> bool:
    return tensor.dtype == np.dtype(dtype) and tensor.shape == (length,) and tensor.strides == (np.dtype(dtype).itemsize,)


def _launch(backend: Any, stream: Any, what: str, call: Any) -> None:
    if getattr(backend, "kind", "") != "cuda":
        raise KernelError(f"{what} requires the CUDA backend")

    def run(native: Any) -> None:
        native.check(call(native.library, native.handle), what)

    backend.launch(stream, run)


# ---- per-row int8 quantizer (quantization.py:156-171) ------------------------------


def supports_quantize_rows_int8(source: Tensor, destination: Tensor, scales: Tensor) -> bool:
    try:
        return (
            _is_cuda(source)
            and source.dtype == np.dtype(np.float32)
            and destination.dtype == np.dtype(np.int8)
            and _row_major(source)
            and _row_major(destination)
            and destination.shape[0] == source.shape[0]
            and destination.shape[1] >= source.shape[1]
            and _vector(scales, source.shape[0], np.float32)
        )
    except Exception:
        return False


def _execute_quantize_rows_int8(backend: Any, args: tuple[Any, ...], grid: tuple[int, int, int], stream: Any) -> None:
    if len(args) != 3 or not all(isinstance(a, Tensor) for a in args):
        raise KernelError("int8 row quantizer expects (source, destination, scales)")
    source, destination, scales = args
    if not supports_quantize_rows_int8(source, destination, scales):
        raise KernelError("int8 row quantizer requires fp32 source rows, int8 destination rows and fp32 scales on CUDA")
    rows, cols = source.shape
    _launch(
        backend,
        stream,
        "quantize_rows_int8",
        lambda lib, ctx: lib.qpucuda_quantize_rows_int8(
            ctx, source.address, source.row_stride_elements, rows, cols, destination.shape[1], destination.address,
            destination.strides[0], scales.address,
        ),
    )


CUDA_QUANTIZE_ROWS_INT8_KERNEL = Kernel("cuda.quantize_rows_int8", _execute_quantize_rows_int8)


# ---- W8A8 GEMM (gemm_int8.py:43-204) -------------------------------------------------


def supports_w8a8_gemm(left: Tensor, right: Tensor, destination: Tensor) -> bool:
    """left int8 [M, Kp], right int8 [N, Kp] (weight rows), destination int32 [M, N]."""
    try:
        m, k = left.shape
        n, k_right = right.shape
        return (
            _is_cuda(left)
            and left.dtype == np.dtype(np.int8)
            and right.dtype == np.dtype(np.int8)
            and destination.dtype == np.dtype(np.int32)
            and k == k_right
            and destination.shape == (m, n)
            and _rows_aligned(left)
            and _rows_aligned(right)
            and _row_major(destination)
            and k * 127 * 127 <= INT32_LIMIT
        )
    except Exception:
        return False


def supports_w8a8_gemm_dequantize(
    left: Tensor, right: Tensor, row_scales: Tensor, column_scales: Tensor, destination: Tensor, bias: Tensor | None = None
) -> bool:
    try:
        m, k = left.shape
        n, k_right = right.shape
        return (
            _is_cuda(left)
            and left.dtype == np.dtype(np.int8)
            and right.dtype == np.dtype(np.int8)
            and destination.dtype == np.dtype(np.float32)
            and k == k_right
            and destination.shape == (m, n)
            and _rows_aligned(left)
            and _rows_aligned(right)
            and _row_major(destination)
            and _vector(row_scales, m, np.float32)
            and _vector(column_scales, n, np.float32)
            and (bias is None or _vector(bias, n, np.float32))
            and k * 127 * 127 <= INT32_LIMIT
        )
    except Exception:
        return False


def _execute_w8a8_gemm(backend: Any, args: tuple[Any, ...], grid: tuple[int, int, int], stream: Any) -> None:
    if len(args) != 3 or not all(isinstance(a, Tensor) for a in args):
        raise KernelError("W8A8 GEMM expects (left, right, destination)")
    left, right, destination = args
    if not supports_w8a8_gemm(left, right, destination):
        raise KernelError("W8A8 GEMM requires int8 [M,K] x int8 [N,K] -> int32 [M,N] with 16-byte aligned rows")
    (m, k), n = left.shape, right.shape[0]
    _launch(
        backend,
        stream,
        "w8a8_gemm_s32",
        lambda lib, ctx: lib.qpucuda_w8a8_gemm_s32(
            ctx, left.address, left.strides[0], right.address, right.strides[0], m, n, k, destination.address,
            destination.row_stride_elements,
        ),
    )


def _execute_w8a8_gemm_dequantize(backend: Any, args: tuple[Any, ...], grid: tuple[int, int, int], stream: Any) -> None:
    if len(args) not in (5, 6) or not all(isinstance(a, Tensor) for a in args):
        raise KernelError("fused W8A8 GEMM expects (left, right, row_scales, column_scales, destination[, bias])")
    left, right, row_scales, column_scales, destination = args[:5]
    bias = args[5] if len(args) == 6 else None
    if not supports_w8a8_gemm_dequantize(left, right, row_scales, column_scales, destination, bias):
        raise KernelError("fused W8A8 GEMM requires aligned int8 operands, fp32 scales and an fp32 destination")
    (m, k), n = left.shape, right.shape[0]
    _launch(
        backend,
        stream,
        "w8a8_gemm_dequantize",
        lambda lib, ctx: lib.qpucuda_w8a8_gemm_dequantize(
            ctx, left.address, left.strides[0], right.address, right.strides[0], m, n, k, row_scales.address,
            column_scales.address, None if bias is None else bias.address, destination.address,
            destination.row_stride_elements,
        ),
    )


CUDA_W8A8_GEMM_KERNEL = Kernel("cuda.w8a8_gemm", _execute_w8a8_gemm)
CUDA_W8A8_GEMM_DEQUANTIZE_KERNEL = Kernel("cuda.w8a8_gemm_dequantize", _execute_w8a8_gemm_dequantize)


# ---- standalone dequantize (w8a8_epilogue.py:20-96) ----------------------------------


def supports_w8a8_dequantize(accumulator: Tensor, row_scales: Tensor, column_scales: Tensor, destination: Tensor) -> bool:
    try:
        m, n = accumulator.shape
        return (
            _is_cuda(accumulator)
            and accumulator.dtype == np.dtype(np.int32)
            and destination.dtype == np.dtype(np.float32)
            and destination.shape == (m, n)
            and _row_major(accumulator)
            and _row_major(destination)
            and _vector(row_scales, m, np.float32)
            and _vector(column_scales, n, np.float32)
        )
    except Exception:
        return False


def _execute_w8a8_dequantize(backend: Any, args: tuple[Any, ...], grid: tuple[int, int, int], stream: Any) -> None:
    if len(args) not in (4, 5) or not all(isinstance(a, Tensor) for a in args):
        raise KernelError("W8A8 dequantize expects (accumulator, row_scales, column_scales, destination[, bias])")
    accumulator, row_scales, column_scales, destination = args[:4]
    bias = args[4] if len(args) == 5 else None
    if not supports_w8a8_dequantize(accumulator, row_scales, column_scales, destination):
        raise KernelError("W8A8 dequantize requires int32 accumulators, fp32 scales and an fp32 destination")
    m, n = accumulator.shape
    _launch(
        backend,
        stream,
        "w8a8_dequantize",
        lambda lib, ctx: lib.qpucuda_w8a8_dequantize(
            ctx, accumulator.address, accumulator.row_stride_elements, m, n, row_scales.address, column_scales.address,
            None if bias is None else bias.address, destination.address, destination.row_stride_elements,
        ),
    )


CUDA_W8A8_DEQUANTIZE_KERNEL = Kernel("cuda.w8a8_dequantize", _execute_w8a8_dequantize)


# ---- W8A8 GEMV (gemv_int8.py:20-153) ---------------------------------------------------


def supports_w8a8_gemv(source: Tensor, weight: Tensor, destination: Tensor) -> bool:
    try:
        m, k = source.shape
        return (
            supports_w8a8_gemm(source, weight, destination)
            and 1 <= m <= 8
            and k % 16 == 0
        )
    except Exception:
        return False


def _execute_w8a8_gemv(backend: Any, args: tuple[Any, ...], grid: tuple[int, int, int], stream: Any) -> None:
    if len(args) != 3 or not all(isinstance(a, Tensor) for a in args):
        raise KernelError("W8A8 GEMV expects (source, weight, destination)")
    source, weight, destination = args
    if not supports_w8a8_gemv(source, weight, destination):
        raise KernelError("W8A8 GEMV requires 1..8 int8 rows with K a multiple of 16 and an int32 destination")
    (m, k), n = source.shape, weight.shape[0]
    _launch(
        backend,
        stream,
        "w8a8_gemv",
        lambda lib, ctx: lib.qpucuda_w8a8_gemv(
            ctx, source.address, source.strides[0], weight.address, weight.strides[0], m, n, k, destination.address,
            destination.row_stride_elements, None, None, None, None, 0,
        ),
    )


CUDA_W8A8_GEMV_KERNEL = Kernel("cuda.w8a8_gemv", _execute_w8a8_gemv)


# ---- GGML Q4_0 x Q8_0 (ggml_q4_0.py:551-841) -------------------------------------------


def supports_ggml_q4_0_q8_0_linear(
    activation: Tensor,
    weight: Tensor,
    destination: Tensor,
    weight_column_start: int,
    output_column_start: int,
    column_count: int,
) -> bool:
    """Contract of the reference's small-M kernel (ggml_q4_0.py:725-761), rows 1..4."""
    try:
        if not _is_cuda(activation):
            return False
        if activation.dtype != np.dtype(np.uint8) or weight.dtype != np.dtype(np.uint8):
            return False
        if destination.dtype != np.dtype(np.float32) or len(activation.shape) != 3 or len(weight.shape) != 3:
            return False
        rows, blocks, activation_bytes = activation.shape
        weight_outputs, weight_blocks, weight_bytes = weight.shape
        if not 1 <= rows <= 4 or activation_bytes != Q8_0_BLOCK_BYTES or weight_bytes != Q4_0_BLOCK_BYTES:
            return False
        if blocks != weight_blocks or destination.shape[0] != rows:
            return False
        starts = (weight_column_start, output_column_start)
        if any(start < 0 or start % OUTPUT_TILE for start in starts) or column_count <= 0 or column_count % OUTPUT_TILE:
            return False
        if weight_column_start + column_count > weight_outputs or output_column_start + column_count > destination.shape[1]:
            return False
        return activation.is_contiguous and weight.is_contiguous and destination.is_contiguous
    except Exception:
        return False


def _execute_ggml_q4_0_q8_0_linear(backend: Any, args: tuple[Any, ...], grid: tuple[int, int, int], stream: Any) -> None:
    if len(args) != 6 or not all(isinstance(a, Tensor) for a in args[:3]):
        raise KernelError(
            "GGML Q4_0 linear expects (activation, weight, destination, weight_column_start, output_column_start, column_count)"
        )
    activation, weight, destination, weight_column_start, output_column_start, column_count = args
    if not all(isinstance(value, int) for value in (weight_column_start, output_column_start, column_count)):
        raise KernelError("GGML Q4_0 column bounds must be integers")
    if not supports_ggml_q4_0_q8_0_linear(activation, weight, destination, weight_column_start, output_column_start, column_count):
        raise KernelError("GGML Q4_0 linear requires native contiguous Q8_0/Q4_0 blocks and aligned columns")
    rows, blocks, _ = activation.shape
    _launch(
        backend,
        stream,
        "ggml_q4_0_q8_0_linear",
        lambda lib, ctx: lib.qpucuda_ggml_q4_0_q8_0_linear(
            ctx, activation.address, rows, blocks, weight.address, weight.shape[0], destination.address,
            destination.shape[1], weight_column_start, output_column_start, column_count,
        ),
    )


CUDA_GGML_Q4_0_Q8_0_LINEAR_KERNEL = Kernel("cuda.ggml_q4_0_q8_0_linear", _execute_ggml_q4_0_q8_0_linear)


def _execute_quantize_blocks(kind: str) -> Any:
    def executor(backend: Any, args: tuple[Any, ...], grid: tuple[int, int, int], stream: Any) -> None:
        if len(args) != 2 or not all(isinstance(a, Tensor) for a in args):
            raise KernelError(f"{kind} quantizer expects (source, blocks)")
        source, blocks = args
        block_bytes = Q8_0_BLOCK_BYTES if kind == "q8_0" else Q4_0_BLOCK_BYTES
        if (
            not _is_cuda(source)
            or source.dtype != np.dtype(np.float32)
            or not _row_major(source)
            or source.shape[1] % Q4_0_BLOCK_ELEMENTS
            or blocks.dtype != np.dtype(np.uint8)
            or blocks.shape != (source.shape[0], source.shape[1] // Q4_0_BLOCK_ELEMENTS, block_bytes)
            or not blocks.is_contiguous
        ):
            raise KernelError(f"{kind} quantizer requires fp32 [rows, K % 32 == 0] and contiguous uint8 blocks")
        rows, cols = source.shape
        entry = "qpucuda_quantize_q8_0" if kind == "q8_0" else "qpucuda_quantize_q4_0"
        _launch(
            backend,
            stream,
            entry,
            lambda lib, ctx: getattr(lib, entry)(ctx, source.address, source.row_stride_elements, rows, cols, blocks.address),
        )

    return executor


CUDA_GGML_QUANTIZE_Q8_0_KERNEL = Kernel("cuda.ggml_quantize_q8_0", _execute_quantize_blocks("q8_0"))
CUDA_GGML_QUANTIZE_Q4_0_KERNEL = Kernel("cuda.ggml_quantize_q4_0", _execute_quantize_blocks("q4_0"))


__all__ = [
    "CUDA_GGML_QUANTIZE_Q4_0_KERNEL",
    "CUDA_GGML_QUANTIZE_Q8_0_KERNEL",
    "CUDA_GGML_Q4_0_Q8_0_LINEAR_KERNEL",
    "CUDA_QUANTIZE_ROWS_INT8_KERNEL",
    "CUDA_W8A8_DEQUANTIZE_KERNEL",
    "CUDA_W8A8_GEMM_DEQUANTIZE_KERNEL",
    "CUDA_W8A8_GEMM_KERNEL",
    "CUDA_W8A8_GEMV_KERNEL",
    "supports_ggml_q4_0_q8_0_linear",
    "supports_quantize_rows_int8",
    "supports_w8a8_dequantize",
    "supports_w8a8_gemm",
    "supports_w8a8_gemm_dequantize",
    "supports_w8a8_gemv",
]
