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


# ---------------------------------------------------------------------------------------------
# GGML MUL_MAT offload core (include/qpucuda_ggml.h): what the reference's llama.cpp backend does
# per MUL_MAT node (integrations/llama_cpp/backend/ggml-qpu.cpp:245-377, 539-620), over tensor
# views with ggml's conventions: ne[0] is the innermost (K) extent, nb[i] the byte strides.


def ggml_tensor_view(
    array: npt.NDArray[Any], ggml_type: int, *, cpu_repack: bool = False, identity: int | None = None
) -> Any:
    """A ``qpucuda_ggml_tensor`` over a host array: F32 ``[M, K]`` rows, or Q4_0 weight blocks
    ``[N, K/32, 18]`` (native) / the same bytes in block_q4_0x4 groups (``cpu_repack``)."""
    if not array.flags.c_contiguous:
        raise ValueError("ggml tensor view needs a C-contiguous array")
    if ggml_type == _native.GGML_TYPE_F32 and (array.dtype != np.float32 or array.ndim != 2):
        raise ValueError(f"F32 view needs a float32 [M, K] array, got {array.dtype} {array.shape}")
    if ggml_type == _native.GGML_TYPE_Q4_0 and (
        array.dtype != np.uint8 or array.ndim != 3 or array.shape[2] != Q4_0_BLOCK_BYTES
    ):
        raise ValueError(f"Q4_0 view needs uint8 [N, K/32, {Q4_0_BLOCK_BYTES}] blocks, got {array.dtype} {array.shape}")
    view = _native.GgmlTensor()
    view.type = ggml_type
    view.cpu_repack = 1 if cpu_repack else 0
    if ggml_type == _native.GGML_TYPE_F32:
        rows, columns = array.shape
        ne = (columns, rows, 1, 1)
        nb0 = 4
        nb1 = nb0 * columns
    elif ggml_type == _native.GGML_TYPE_Q4_0:
        outputs, blocks = array.shape[0], array.shape[1]
        ne = (blocks * Q4_0_BLOCK_ELEMENTS, outputs, 1, 1)
        nb0 = Q4_0_BLOCK_BYTES
        nb1 = Q4_0_BLOCK_BYTES * blocks
    else:
        raise ValueError(f"unsupported ggml type {ggml_type}")
    for i, extent in enumerate(ne):
        view.ne[i] = extent
    view.nb[0] = nb0
    view.nb[1] = nb1
    view.nb[2] = nb1 * ne[1]
    view.nb[3] = view.nb[2] * ne[2]
    view.data = array.ctypes.data
    view.identity = identity if identity is not None else array.ctypes.data
    return view


def ggml_supports_mul_mat(weight: Any, activation: Any, destination: Any, *, minimum_rows: int = 1, maximum_rows: int = 4 * 65535) -> bool:
    """``supports_q4_0_mul_mat`` with the device's row window (ggml-qpu.cpp:362-377, 631-633)."""
    library = _native.load()
    return bool(library.qpucuda_ggml_supports_mul_mat(ctypes.byref(weight), ctypes.byref(activation), ctypes.byref(destination), minimum_rows, maximum_rows))


def ggml_unpack_q4_0x4(packed: npt.NDArray[np.uint8], input_columns: int, output_columns: int) -> npt.NDArray[np.uint8]:
    """block_q4_0x4 groups back to native ``[N, K/32, 18]`` blocks (ggml-qpu.cpp:250-283)."""
    packed = np.ascontiguousarray(packed, dtype=np.uint8)
    native = np.empty((output_columns, input_columns // Q4_0_BLOCK_ELEMENTS, Q4_0_BLOCK_BYTES), dtype=np.uint8)
    status = _native.load().qpucuda_ggml_unpack_q4_0x4(packed.ctypes.data, packed.nbytes, input_columns, output_columns, native.ctypes.data, native.nbytes)
    _native.raise_for_status(status, what="qpucuda_ggml_unpack_q4_0x4")
    return native


class GgmlMulMatBackend:
    """The MUL_MAT offload of one llama.cpp backend instance on one GPU: a weight cache of
    prepared Q4_0 linears keyed by tensor identity, staging, and per-call statistics."""

    def __init__(self: Self, device: Device, *, minimum_rows: int = 1, maximum_rows: int = 4 * 65535) -> None:
        if not device.is_cuda:
            raise ValueError("GgmlMulMatBackend requires the CUDA backend")
        self.device = device
        self.minimum_rows = minimum_rows
        self.maximum_rows = maximum_rows
        self._backend = device.backend
        self._native = self._backend.native  # type: ignore[attr-defined]
        handle = ctypes.c_void_p()
        status = self._native.library.qpucuda_ggml_backend_create(self._native.handle, minimum_rows, maximum_rows, ctypes.byref(handle))
        self._native.check(status, "qpucuda_ggml_backend_create")
        self._handle = int(handle.value)  # type: ignore[arg-type]
        self._closed = False

    def supports(self: Self, weight: Any, activation: Any, destination: Any) -> bool:
        return ggml_supports_mul_mat(weight, activation, destination, minimum_rows=self.minimum_rows, maximum_rows=self.maximum_rows)

    def mul_mat_views(self: Self, weight: Any, activation: Any, destination: Any) -> int:
        """``compute_q4_0_mul_mat`` over tensor views; returns the status (no raise)."""
        with self._backend.launch_lock:  # type: ignore[attr-defined]
            self._native.use_library_stream()
            return int(self._native.library.qpucuda_ggml_mul_mat(self._handle, ctypes.byref(weight), ctypes.byref(activation), ctypes.byref(destination)))

    def mul_mat(
        self: Self,
        weight_blocks: npt.NDArray[np.uint8],
        activation: npt.NDArray[np.float32],
        *,
        cpu_repack: bool = False,
        output_columns: int | None = None,
        identity: int | None = None,
    ) -> npt.NDArray[np.float32]:
        """``activation [M, K] x weight^T`` for native Q4_0 blocks ``[N, K/32, 18]``, or, with
        ``cpu_repack``, the same weight as block_q4_0x4 bytes (give ``output_columns``)."""
        activation = np.ascontiguousarray(activation, dtype=np.float32)
        if cpu_repack:
            if output_columns is None:
                raise ValueError("output_columns is required for a CPU_REPACK weight")
            blocks = activation.shape[1] // Q4_0_BLOCK_ELEMENTS
            weight_blocks = np.ascontiguousarray(weight_blocks, dtype=np.uint8).reshape(output_columns, blocks, Q4_0_BLOCK_BYTES)
        weight_view = ggml_tensor_view(weight_blocks, _native.GGML_TYPE_Q4_0, cpu_repack=cpu_repack, identity=identity)
        destination = np.empty((activation.shape[0], weight_blocks.shape[0]), dtype=np.float32)
        status = self.mul_mat_views(weight_view, ggml_tensor_view(activation, _native.GGML_TYPE_F32), ggml_tensor_view(destination, _native.GGML_TYPE_F32))
        self._native.check(status, "qpucuda_ggml_mul_mat")
        return destination

    def forget(self: Self, identity: int) -> None:
        self._native.library.qpucuda_ggml_backend_forget(self._handle, identity)

    @property
    def stats(self: Self) -> dict[str, int]:
        stats = _native.GgmlStats()
        self._native.check(self._native.library.qpucuda_ggml_backend_stats(self._handle, ctypes.byref(stats)), "qpucuda_ggml_backend_stats")
        return {name: int(getattr(stats, name)) for name, _ in _native.GgmlStats._fields_}

    def close(self: Self) -> None:
        if not self._closed:
            self._native.library.qpucuda_ggml_backend_destroy(self._handle)
            self._closed = True

    def __enter__(self: Self) -> Self:
        return self

    def __exit__(self: Self, exc_type: object, exc_value: object, traceback: object) -> None:
        self.close()


__all__ = [
    "GgmlMulMatBackend",
    "PreparedQ4_0Linear",
    "ggml_supports_mul_mat",
    "ggml_tensor_view",
    "ggml_unpack_q4_0x4",
    "pack_ggml_q4_0_blocks",
    "pack_ggml_q8_0_blocks",
    "q4_0_kernel_source_hash",
    "quantize_q4_0",
    "quantize_q8_0",
    "unpack_ggml_q4_0_blocks",
    "unpack_ggml_q8_0_blocks",
]
