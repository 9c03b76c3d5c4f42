"""GGML Q4_0 / Q8_0 blocks and the prepared Q4_0 x Q8_0 linear on CUDA.

Block format helpers follow src/qpu_xla/kernels/ggml_q4_0.py:21-78: a native
``block_q4_0`` is an fp16 scale (little-endian) and 16 bytes whose byte j holds
code j (low nibble) and code j + 16 (high nibble), value = code - 8; a native
``block_q8_0`` is an fp16 scale and 32 signed bytes. These are host-side format
conversions (building inputs, reading results); the arithmetic runs in CUDA.

:class:`PreparedQ4_0Linear` is the Python face of the C operator
``qpucuda_q4_0_linear_*`` (include/qpucuda_q4_0.h), itself the drop-in for the
reference's ``qpu_llama_q4_0_linear_*`` (integrations/llama_cpp/include/qpu_llama_q4_0.h:63-82).
"""

from __future__ import annotations

import ctypes
from collections.abc import Iterable
from typing import Any, Self

import numpy as np
import numpy.typing as npt

from qpu_xla import _native
from qpu_xla.device import Device
from qpu_xla.errors import DependencyError
from qpu_xla.kernel import Kernel
from qpu_xla.kernels import OUTPUT_TILE, Q4_0_BLOCK_BYTES, Q4_0_BLOCK_ELEMENTS, Q8_0_BLOCK_BYTES
from qpu_xla.memory import AccessMode, Tensor
from qpu_xla.queue import Event, Queue


def pack_ggml_q4_0_blocks(scales: npt.ArrayLike, codes: npt.ArrayLike) -> npt.NDArray[np.uint8]:
    """Pack explicit 0..15 codes into native ``block_q4_0`` bytes (ggml_q4_0.py:28-40)."""
    scales = np.asarray(scales, dtype=np.float16)
    codes = np.asarray(codes)
    if codes.shape != (*scales.shape, Q4_0_BLOCK_ELEMENTS) or np.any((codes < 0) | (codes > 15)):
        raise ValueError("Q4_0 codes must have scales.shape + (32,) and values in 0..15")
    packed = np.empty((*scales.shape, Q4_0_BLOCK_BYTES), dtype=np.uint8)
    packed[..., :2] = scales.astype("<f2").view(np.uint8).reshape(*scales.shape, 2)
    packed[..., 2:] = codes[..., :16].astype(np.uint8) | (codes[..., 16:].astype(np.uint8) << 4)
    return np.ascontiguousarray(packed)


def pack_ggml_q8_0_blocks(scales: npt.ArrayLike, values: npt.ArrayLike) -> npt.NDArray[np.uint8]:
    """Pack explicit signed bytes into native ``block_q8_0`` bytes (ggml_q4_0.py:43-54)."""
    scales = np.asarray(scales, dtype=np.float16)
    values = np.asarray(values)
    if values.shape != (*scales.shape, Q4_0_BLOCK_ELEMENTS) or np.any((values < -128) | (values > 127)):
        raise ValueError("Q8_0 values must have scales.shape + (32,) and values in -128..127")
    packed = np.empty((*scales.shape, Q8_0_BLOCK_BYTES), dtype=np.uint8)
    packed[..., :2] = scales.astype("<f2").view(np.uint8).reshape(*scales.shape, 2)
    packed[..., 2:] = values.astype(np.int8).view(np.uint8)
    return np.ascontiguousarray(packed)


def unpack_ggml_q4_0_blocks(blocks: npt.NDArray[np.uint8]) -> tuple[npt.NDArray[np.float32], npt.NDArray[np.int8]]:
    """Decode native Q4_0 blocks into fp32 scales and int8 values in -8..7 (ggml_q4_0.py:57-67)."""
    blocks = np.asarray(blocks)
    if blocks.dtype != np.dtype(np.uint8) or blocks.ndim < 1 or blocks.shape[-1] != Q4_0_BLOCK_BYTES:
        raise ValueError("Q4_0 blocks must be uint8 with a final extent of 18 bytes")
    scales = blocks[..., :2].copy().reshape(-1, 2).view("<f2").reshape(blocks.shape[:-1]).astype(np.float32)
    packed = blocks[..., 2:]
    values = np.empty((*blocks.shape[:-1], Q4_0_BLOCK_ELEMENTS), dtype=np.int8)
    values[..., :16] = (packed & 0x0F).astype(np.int8) - 8
    values[..., 16:] = (packed >> 4).astype(np.int8) - 8
    return scales, values


def unpack_ggml_q8_0_blocks(blocks: npt.NDArray[np.uint8]) -> tuple[npt.NDArray[np.float32], npt.NDArray[np.int8]]:
    """Decode native Q8_0 blocks into fp32 scales and int8 values (ggml_q4_0.py:70-78)."""
    blocks = np.asarray(blocks)
    if blocks.dtype != np.dtype(np.uint8) or blocks.ndim < 1 or blocks.shape[-1] != Q8_0_BLOCK_BYTES:
        raise ValueError("Q8_0 blocks must be uint8 with a final extent of 34 bytes")
    scales = blocks[..., :2].copy().reshape(-1, 2).view("<f2").reshape(blocks.shape[:-1])
    return scales.astype(np.float32), blocks[..., 2:].view(np.int8)


def q4_0_kernel_source_hash() -> str:
    """The identity a Q4_0 linear is prepared against (``qpucuda_q4_0_kernel_source_hash``)."""
    return _native.load().qpucuda_q4_0_kernel_source_hash().decode()


def quantize_q8_0(device: Device, source: Any) -> Any:
    """fp32 rows (torch CUDA tensor [rows, K]) -> native Q8_0 blocks (torch uint8 [rows, K/32, 34]) on the device."""
    import torch

    if source.dtype != torch.float32 or source.dim() != 2 or source.shape[1] % Q4_0_BLOCK_ELEMENTS or source.stride(1) != 1:
        raise ValueError("quantize_q8_0 requires a row-major float32 [rows, K] tensor with K % 32 == 0")
    rows, cols = source.shape
    blocks = torch.empty((rows, cols // Q4_0_BLOCK_ELEMENTS, Q8_0_BLOCK_BYTES), dtype=torch.uint8, device=source.device)
    backend = device.backend
    backend.launch(  # type: ignore[attr-defined]
        torch.cuda.current_stream(source.device),
        lambda native: native.check(
            native.library.qpucuda_quantize_q8_0(native.handle, source.data_ptr(), source.stride(0), rows, cols, blocks.data_ptr()),
            "quantize_q8_0",
        ),
    )
    return blocks


def quantize_q4_0(device: Device, source: Any) -> Any:
    """fp32 rows -> native Q4_0 blocks on the device (ggml's published quantize_row_q4_0_ref)."""
    import torch

    if source.dtype != torch.float32 or source.dim() != 2 or source.shape[1] % Q4_0_BLOCK_ELEMENTS or source.stride(1) != 1:
        raise ValueError("quantize_q4_0 requires a row-major float32 [rows, K] tensor with K % 32 == 0")
    rows, cols = source.shape
    blocks = torch.empty((rows, cols // Q4_0_BLOCK_ELEMENTS, Q4_0_BLOCK_BYTES), dtype=torch.uint8, device=source.device)
    backend = device.backend
    backend.launch(  # type: ignore[attr-defined]
        torch.cuda.current_stream(source.device),
        lambda native: native.check(
            native.library.qpucuda_quantize_q4_0(native.handle, source.data_ptr(), source.stride(0), rows, cols, blocks.data_ptr()),
            "quantize_q4_0",
        ),
    )
    return blocks


class PreparedQ4_0Linear:
    """Resident Q4_0 weight window on one GPU, executed for M = 1..4 rows.

    ``weight_blocks`` are native ``block_q4_0`` rows ``[outputs, K/32, 18]`` in host
    memory; the resident column window (16-aligned) is copied and repacked on the
    device once. Calls:

    * :meth:`execute` -- queue submission over device tensors (the reference's
      ``queue.submit(GGML_Q4_0_Q8_0_LINEAR_KERNEL, ...)``), weight/output column split;
    * :meth:`execute_f32` -- fp32 activations, Q8_0 quantization fused on the device;
    * :meth:`forward` -- torch tensors on the current stream (bench path);
    * :meth:`execute_host` -- host NumPy buffers through ``qpucuda_q4_0_linear_execute``
      (the C drop-in path, synchronous, with the reference's timing record).
    """

    def __init__(
        self: Self,
        device: Device,
        weight_blocks: npt.NDArray[np.uint8],
        *,
        rows: int,
        resident_column_start: int = 0,
        resident_column_count: int | None = None,
        expected_source_hash: str | None = None,
    ) -> None:
        if not device.is_cuda:
            raise ValueError("PreparedQ4_0Linear requires the CUDA backend")
        weight_blocks = np.ascontiguousarray(weight_blocks)
        if weight_blocks.dtype != np.uint8 or weight_blocks.ndim != 3 or weight_blocks.shape[2] != Q4_0_BLOCK_BYTES:
            raise ValueError("Q4_0 weights must be uint8 [outputs, blocks, 18]")
        outputs, blocks, _ = weight_blocks.shape
        count = outputs - resident_column_start if resident_column_count is None else resident_column_count
        self.device = device
        self.rows = rows
        self.input_columns = blocks * Q4_0_BLOCK_ELEMENTS
        self.output_columns = outputs
        self.resident_column_start = resident_column_start
        self.resident_column_count = count
        self._backend = device.backend
        native = self._backend.native  # type: ignore[attr-defined]
        self._native = native
        self._weights_host = weight_blocks  # kept alive for the duration of prepare only
        desc = _native.Q40LinearDesc(
            weight_blocks.ctypes.data,
            weight_blocks.nbytes,
            self.input_columns,
            outputs,
            rows,
            resident_column_start,
            count,
            0,
            0,
            (expected_source_hash if expected_source_hash is not None else q4_0_kernel_source_hash()).encode(),
        )
        handle = ctypes.c_void_p()
        with self._backend.launch_lock:  # type: ignore[attr-defined]
            status = native.library.qpucuda_q4_0_linear_prepare(native.handle, ctypes.byref(desc), ctypes.byref(handle))
        native.check(status, "qpucuda_q4_0_linear_prepare")
        self._handle = int(handle.value)  # type: ignore[arg-type]
        self._weights_host = None
        self._queue: Queue | None = None
        self._closed = False

    @property
    def resident_bytes(self: Self) -> int:
        return int(self._native.library.qpucuda_q4_0_linear_resident_bytes(self._handle))

    def _require_open(self: Self) -> None:
        if self._closed:
            raise RuntimeError("prepared Q4_0 linear is closed")

    def execute(
        self: Self,
        destination: Tensor,
        activation: Tensor,
        *,
        queue: Queue,
        column_start: int | None = None,
        column_count: int | None = None,
        output_column_start: int | None = None,
        wait_for: Iterable[Event] = (),
    ) -> Event:
        """Submit ``destination[:, out0:out0+count] = activation (Q8_0) x W[col0:col0+count]``."""
        self._require_open()
        if queue.device is not self.device or activation.buffer.device is not self.device or destination.buffer.device is not self.device:
            raise DependencyError("prepared Q4_0 linear queue and tensors must belong to the plan device")
        col0 = self.resident_column_start if column_start is None else column_start
        count = self.resident_column_count if column_count is None else column_count
        out0 = col0 if output_column_start is None else output_column_start
        rows = activation.shape[0]
        if (
            activation.dtype != np.dtype(np.uint8)
            or activation.shape[1:] != (self.input_columns // Q4_0_BLOCK_ELEMENTS, Q8_0_BLOCK_BYTES)
            or not activation.is_contiguous
            or destination.dtype != np.dtype(np.float32)
            or len(destination.shape) != 2
            or destination.shape[0] != rows
            or not destination.is_contiguous
            or out0 % OUTPUT_TILE
            or out0 + count > destination.shape[1]
        ):
            raise ValueError("prepared Q4_0 linear requires Q8_0 [rows, K/32, 34] and fp32 [rows, >= out0 + count]")
        handle = self._handle

        def executor(backend: Any, args: tuple[Any, ...], grid: tuple[int, int, int], stream: Any) -> None:
            backend.launch(
                stream,
                lambda native: native.check(
                    native.library.qpucuda_q4_0_linear_execute_device(
                        handle, activation.address, rows, destination.address, destination.shape[1], col0, count, out0
                    ),
                    "qpucuda_q4_0_linear_execute_device",
                ),
            )

        return queue.submit(
            Kernel("cuda.ggml_q4_0_q8_0_linear", executor),
            (),
            wait_for=wait_for,
            buffers=(activation.access(AccessMode.READ), destination.access(AccessMode.WRITE)),
        )

    def execute_f32(
        self: Self,
        destination: Tensor,
        source: Tensor,
        *,
        queue: Queue,
        column_start: int | None = None,
        column_count: int | None = None,
        output_column_start: int | None = None,
        wait_for: Iterable[Event] = (),
    ) -> Event:
        """Submit the fused device path: fp32 rows -> Q8_0 -> Q4_0 x Q8_0 linear."""
        self._require_open()
        col0 = self.resident_column_start if column_start is None else column_start
        count = self.resident_column_count if column_count is None else column_count
        out0 = col0 if output_column_start is None else output_column_start
        rows = source.shape[0]
        if (
            source.dtype != np.dtype(np.float32)
            or len(source.shape) != 2
            or source.shape[1] != self.input_columns
            or source.strides[1] != 4
            or destination.dtype != np.dtype(np.float32)
            or destination.shape[0] != rows
            or not destination.is_contiguous
        ):
            raise ValueError("prepared Q4_0 linear requires fp32 [rows, K] source and fp32 [rows, N] destination")
        handle = self._handle

        def executor(backend: Any, args: tuple[Any, ...], grid: tuple[int, int, int], stream: Any) -> None:
            backend.launch(
                stream,
                lambda native: native.check(
                    native.library.qpucuda_q4_0_linear_execute_f32_device(
                        handle, source.address, source.row_stride_elements, rows, destination.address,
                        destination.shape[1], col0, count, out0,
                    ),
                    "qpucuda_q4_0_linear_execute_f32_device",
                ),
            )

        return queue.submit(
            Kernel("cuda.ggml_q8_0_quantize_q4_0_linear", executor),
            (),
            wait_for=wait_for,
            buffers=(source.access(AccessMode.READ), destination.access(AccessMode.WRITE)),
        )

    def forward(self: Self, activation: Any, out: Any = None, *, fp32_source: bool = False) -> Any:
        """Torch path on the current stream: activation Q8_0 uint8 [rows, K/32, 34] (or fp32 [rows, K])."""
        import torch

        self._require_open()
        rows = activation.shape[0]
        if out is None:
            out = torch.empty((rows, self.resident_column_count), dtype=torch.float32, device=activation.device)
        col0, count = self.resident_column_start, self.resident_column_count
        handle = self._handle
        stream = torch.cuda.current_stream(activation.device)
        if fp32_source:
            call = lambda native: native.check(  # noqa: E731
                native.library.qpucuda_q4_0_linear_execute_f32_device(
                    handle, activation.data_ptr(), activation.stride(0), rows, out.data_ptr(), out.stride(0), col0, count, 0
                ),
                "qpucuda_q4_0_linear_execute_f32_device",
            )
        else:
            call = lambda native: native.check(  # noqa: E731
                native.library.qpucuda_q4_0_linear_execute_device(
                    handle, activation.data_ptr(), rows, out.data_ptr(), out.stride(0), col0, count, 0
                ),
                "qpucuda_q4_0_linear_execute_device",
            )
        self._backend.launch(stream, call)  # type: ignore[attr-defined]
        return out

    def execute_host(
        self: Self,
        activation: npt.NDArray[np.uint8],
        destination: npt.NDArray[np.float32],
        *,
        column_start: int | None = None,
        column_count: int | None = None,
        rows: int = 0,
        activation_interleave: int = 0,
    ) -> dict[str, int]:
        """``qpucuda_q4_0_linear_execute`` over host buffers; returns the timing record (ns)."""
        self._require_open()
        if not activation.flags.c_contiguous or not destination.flags.c_contiguous or destination.dtype != np.float32:
            raise ValueError("host activation and destination must be C-contiguous (destination fp32)")
        execution = _native.Q40Execution(
            activation.ctypes.data,
            activation.nbytes,
            0,
            destination.ctypes.data,
            destination.nbytes,
            0,
            self.resident_column_start if column_start is None else column_start,
            self.resident_column_count if column_count is None else column_count,
            rows,
            activation_interleave,
        )
        timing = _native.Q40Timing()
        with self._backend.launch_lock:  # type: ignore[attr-defined]
            self._native.use_library_stream()
            status = self._native.library.qpucuda_q4_0_linear_execute(self._handle, ctypes.byref(execution), ctypes.byref(timing))
        self._native.check(status, "qpucuda_q4_0_linear_execute")
        return {name: int(getattr(timing, name)) for name, _ in _native.Q40Timing._fields_}

    def close(self: Self) -> None:
        if not self._closed:
            import torch

            torch.cuda.synchronize(self._backend.torch_device)  # type: ignore[attr-defined]
            self._native.library.qpucuda_q4_0_linear_destroy(self._handle)
            self._closed = True

    def __enter__(self: Self) -> Self:
        self._require_open()
        return self

    def __exit__(self: Self, exc_type: object, exc_value: object, traceback: object) -> None:
        self.close()


__all__ = [
    "PreparedQ4_0Linear",
    "pack_ggml_q4_0_blocks",
    "pack_ggml_q8_0_blocks",
    "q4_0_kernel_source_hash",
    "quantize_q4_0",
    "quantize_q8_0",
    "unpack_ggml_q4_0_blocks",
    "unpack_ggml_q8_0_blocks",
]
