"""Dynamic W8A8 quantized-linear plans on CUDA.

The drop-in for src/qpu_xla/models/tinyllama/quantization.py: same class and
function names, argument checks and error types. The arithmetic is the
reference's (``s = max(max|x|/127, 1/127)``, ``q = clip(rint(x/s), -127, 127)``,
exact int32 accumulation, ``((float)acc * s_a) * s_w``, bias after), executed by
libqpucuda: int8 row quantizer, tcgen05 int8 GEMM (or the dp4a GEMV for <= 8
rows) with the dequant (+bias) epilogue fused. There is no CPU execution path:
``qpu_dequantize`` / ``fuse_dequantize`` are accepted for signature
compatibility, and the dequantization always runs fused on the GPU.

The reference's CPU/QPU hybrid splits (``execute_hybrid*``) keep their calls and
argument rules, with both parts on the GPU; an output-channel split across GPUs
is :class:`qpu_xla.sharded.ShardedW8A8Linear`.
"""

from __future__ import annotations

import ctypes
from collections.abc import Iterable, Sequence
from dataclasses import dataclass
from typing import Any, Self

import numpy as np
import numpy.typing as npt

from qpu_xla import _native
from qpu_xla.candidates import CandidateRecord, CandidateRegistry
from qpu_xla.device import Device
from qpu_xla.errors import DependencyError
from qpu_xla.kernel import Kernel
from qpu_xla.memory import AccessMode, Tensor
from qpu_xla.placement import Placement
from qpu_xla.queue import Event, Queue

GEMV_MAX_ROWS = 8


@dataclass(frozen=True, slots=True)
class QuantizedMatrixInt8:
    """Row-wise symmetric int8 matrix plus one fp32 scale per row (quantization.py:31-54)."""

    values: npt.NDArray[np.int8]
    scales: npt.NDArray[np.float32]

    def __post_init__(self: Self) -> None:
        if self.values.ndim != 2 or self.scales.ndim != 1 or self.scales.shape != (self.values.shape[0],):
            raise ValueError("quantized matrix values must be rank-2 with one scale per output row")
        if not self.values.flags.c_contiguous or not self.scales.flags.c_contiguous:
            raise ValueError("quantized matrix values and scales must be contiguous")
        if self.values.dtype != np.dtype(np.int8) or self.scales.dtype != np.dtype(np.float32):
            raise ValueError("quantized matrix values must be int8 and scales float32")
        if not np.all(np.isfinite(self.scales)) or np.any(self.scales <= 0):
            raise ValueError("quantized matrix scales must be finite and positive")

    @property
    def shape(self: Self) -> tuple[int, int]:
        """``(output_features, input_features)``."""
        return (int(self.values.shape[0]), int(self.values.shape[1]))

    def dequantize(self: Self) -> npt.NDArray[np.float32]:
        """fp32 reconstruction ``values * scales[:, None]``."""
        return np.ascontiguousarray(self.values.astype(np.float32) * self.scales[:, None])


def quantize_per_output_channel_int8(weight: npt.NDArray[np.float32], *, device: Device | None = None) -> QuantizedMatrixInt8:
    """Quantize fp32 ``(output, input)`` weights to int8 rows on the GPU (quantization.py:1085-1092).

    Runs the CUDA per-row quantizer (the same kernel as the activation
    quantizer) and returns host arrays, as the reference does. ``device``
    defaults to a CUDA device opened on the current GPU.
    """
    import torch

    if weight.ndim != 2 or weight.dtype != np.dtype(np.float32):
        raise ValueError("quantize_per_output_channel_int8 requires a rank-2 float32 matrix")
    owned = device is None
    device = Device.open() if device is None else device
    try:
        if not device.is_cuda:
            raise ValueError("quantize_per_output_channel_int8 runs on the CUDA backend")
        torch_device = device.backend.torch_device  # type: ignore[attr-defined]
        rows, cols = weight.shape
        source = torch.from_numpy(np.ascontiguousarray(weight)).to(torch_device)
        values = torch.empty((rows, cols), dtype=torch.int8, device=torch_device)
        scales = torch.empty((rows,), dtype=torch.float32, device=torch_device)
        stream = torch.cuda.current_stream(torch_device)
        device.backend.launch(  # type: ignore[attr-defined]
            stream,
            lambda native: native.check(
                native.library.qpucuda_quantize_rows_int8(
                    native.handle, source.data_ptr(), cols, rows, cols, cols, values.data_ptr(), cols, scales.data_ptr()
                ),
                "qpucuda_quantize_rows_int8",
            ),
        )
        stream.synchronize()
        return QuantizedMatrixInt8(np.ascontiguousarray(values.cpu().numpy()), np.ascontiguousarray(scales.cpu().numpy()))
    finally:
        if owned:
            device.close()


class PreparedW8A8Linear:
    """Persistent int8 weight (+scales, bias) resident on one GPU, with activation scratch.

    Mirrors quantization.py:57-878: the plan owns the padded weight and the
    reusable activation scratch, is bound to its first queue and admits one
    in-flight invocation (:290-295). ``resident_outputs=(start, count)`` keeps
    only an output-channel window of the weight (the N-split shard); the
    destination then has ``count`` columns.
    """

    def __init__(
        self: Self,
        device: Device,
        weight: QuantizedMatrixInt8,
        *,
        max_batch: int,
        qpu_dequantize: bool = True,
        fuse_dequantize: bool = True,
        bias: npt.NDArray[np.float32] | None = None,
        resident_outputs: tuple[int, int] | None = None,
    ) -> None:
        if max_batch <= 0:
            raise ValueError("PreparedW8A8Linear max_batch must be positive")
        if not device.is_cuda:
            raise ValueError("PreparedW8A8Linear requires the CUDA backend (this build has no CPU path)")
        outputs, features = weight.shape
        if features * 127 * 127 > np.iinfo(np.int32).max:
            raise ValueError("prepared W8A8 linear accumulation can overflow int32")
        start, count = (0, outputs) if resident_outputs is None else resident_outputs
        if start < 0 or count <= 0 or start + count > outputs:
            raise ValueError("resident output window lies outside the weight")
        if bias is not None:
            bias = np.ascontiguousarray(bias, dtype=np.float32)
            if bias.shape != (outputs,):
                raise ValueError("bias must have one fp32 value per output feature")
        self.device = device
        self.weight = weight
        self.max_batch = max_batch
        self.bias = bias
        self.qpu_dequantize = qpu_dequantize
        self.fuse_dequantize = fuse_dequantize
        self.output_start = start
        self.output_count = count
        self.padded_features = (features + 15) // 16 * 16
        self._backend = device.backend
        self._native = self._backend.native  # type: ignore[attr-defined]
        desc = _native.W8A8LinearDesc(
            weight.values.ctypes.data,
            weight.scales.ctypes.data,
            None if bias is None else bias.ctypes.data,
            features,
            outputs,
            max_batch,
            start,
            count,
            _native.MEMORY_HOST,
        )
        handle = ctypes.c_void_p()
        with self._backend.launch_lock:  # type: ignore[attr-defined]
            self._native.use_library_stream()
            status = self._native.library.qpucuda_w8a8_linear_prepare(self._native.handle, ctypes.byref(desc), ctypes.byref(handle))
        self._native.check(status, "qpucuda_w8a8_linear_prepare")
        self._handle = int(handle.value)  # type: ignore[arg-type]
        self._queue: Queue | None = None
        self._cpu_queue: Queue | None = None
        self._last_event: Event | None = None
        self._closed = False

    # -- lifetime -------------------------------------------------------------------

    def __enter__(self: Self) -> Self:
        if self._closed:
            raise RuntimeError("prepared W8A8 linear plan is closed")
        return self

    def __exit__(self: Self, exc_type: object, exc_value: object, traceback: object) -> None:
        self.close()

    def close(self: Self) -> None:
        """Wait for outstanding work and release the plan's device memory."""
        if self._closed:
            return
        if self._last_event is not None:
            try:
                self._last_event.wait()
            except Exception:
                pass
        import torch

        torch.cuda.synchronize(self._backend.torch_device)  # type: ignore[attr-defined]
        self._native.library.qpucuda_w8a8_linear_destroy(self._handle)
        self._closed = True

    @property
    def resident_bytes(self: Self) -> int:
        return int(self._native.library.qpucuda_w8a8_linear_resident_bytes(self._handle))

    def scratch(self: Self) -> tuple[Any, Any]:
        """Torch views of the activation scratch: int8 ``[max_batch, padded K]`` and fp32 ``[max_batch]``."""
        import torch

        quantized = ctypes.c_void_p()
        stride = ctypes.c_size_t()
        scales = ctypes.c_void_p()
        self._native.check(
            self._native.library.qpucuda_w8a8_linear_scratch(self._handle, ctypes.byref(quantized), ctypes.byref(stride), ctypes.byref(scales)),
            "qpucuda_w8a8_linear_scratch",
        )
        device = self._backend.torch_device  # type: ignore[attr-defined]
        return (
            _torch_view(int(quantized.value), (self.max_batch, int(stride.value)), torch.int8, device),  # type: ignore[arg-type]
            _torch_view(int(scales.value), (self.max_batch,), torch.float32, device),  # type: ignore[arg-type]
        )

    # -- submission -----------------------------------------------------------------

    def _check_submission(self: Self, queue: Queue) -> None:
        if self._closed:
            raise RuntimeError("prepared W8A8 linear plan is closed")
        if self._last_event is not None and not self._last_event.done:
            raise RuntimeError("prepared W8A8 linear plan already has an in-flight invocation")
        if self._queue is None:
            self._queue = queue
        elif self._queue is not queue:
            raise DependencyError("prepared W8A8 linear plan is bound to its first submission queue")
        if queue.device is not self.device:
            raise DependencyError("prepared W8A8 linear queue and tensors must belong to the plan device")

    def kernel_name(self: Self, batch: int) -> str:
        return "cuda.w8a8_gemv" if batch <= GEMV_MAX_ROWS else "cuda.w8a8_gemm_dequantize"

    def execute(self: Self, destination: Tensor, source: Tensor, *, queue: Queue, wait_for: Iterable[Event] = ()) -> Event:
        """Quantize ``source`` rows, GEMM and fused dequant into ``destination`` (quantization.py:279-323)."""
        self._check_submission(queue)
        if source.buffer.device is not self.device or destination.buffer.device is not self.device:
            raise DependencyError("prepared W8A8 linear source and destination must belong to the plan device")
        if source.dtype != np.dtype(np.float32) or destination.dtype != np.dtype(np.float32):
            raise ValueError("prepared W8A8 linear requires float32 source and destination")
        if len(source.shape) != 2 or len(destination.shape) != 2:
            raise ValueError("prepared W8A8 linear requires rank-2 source and destination")
        batch, features = source.shape
        if batch > self.max_batch or features != self.weight.shape[1]:
            raise ValueError("prepared W8A8 linear source exceeds the plan shape")
        if destination.shape != (batch, self.output_count):
            raise ValueError("prepared W8A8 linear destination shape does not align")
        if source.strides[1] != 4 or destination.strides[1] != 4:
            raise ValueError("prepared W8A8 linear requires unit inner strides")
        handle = self._handle

        def executor(backend: Any, args: tuple[Any, ...], grid: tuple[int, int, int], stream: Any) -> None:
            backend.launch(
                stream,
                lambda native: native.check(
                    native.library.qpucuda_w8a8_linear_execute_device(
                        handle, source.address, source.row_stride_elements, batch, destination.address,
                        destination.row_stride_elements,
                    ),
                    "qpucuda_w8a8_linear_execute_device",
                ),
            )

        event = queue.submit(
            Kernel(self.kernel_name(batch), executor),
            (),
            wait_for=wait_for,
            buffers=(source.access(AccessMode.READ), destination.access(AccessMode.WRITE)),
        )
        self._last_event = event
        return event

    def _bind_hybrid_queues(self: Self, qpu_queue: Queue, cpu_queue: Queue) -> None:
        """The reference's queue rules for every hybrid split (quantization.py:361-375, 717-732):
        an open plan with nothing in flight, two distinct queues of the plan device, each bound to
        the plan on first use."""
        if self._closed:
            raise RuntimeError("prepared W8A8 linear plan is closed")
        if self._last_event is not None and not self._last_event.done:
            raise RuntimeError("prepared W8A8 linear plan already has an in-flight invocation")
        if qpu_queue is cpu_queue:
            raise DependencyError("hybrid W8A8 linear requires distinct CPU and QPU queues")
        if qpu_queue.device is not self.device or cpu_queue.device is not self.device:
            raise DependencyError("hybrid W8A8 queues must belong to the plan device")
        if self._queue is None:
            self._queue = qpu_queue
        elif self._queue is not qpu_queue:
            raise DependencyError("prepared W8A8 linear plan is bound to its first QPU queue")
        if self._cpu_queue is None:
            self._cpu_queue = cpu_queue
        elif self._cpu_queue is not cpu_queue:
            raise DependencyError("prepared W8A8 linear plan is bound to its first CPU queue")

    def _check_hybrid_units(self: Self, name: str, units: int, total: int) -> None:
        if units <= 0 or units >= total or units % 16:
            raise ValueError(f"hybrid W8A8 {name} must be aligned and leave a non-empty CPU tail")

    # The reference's CPU/QPU splits (quantization.py:350-514, 516-662, 664-878) keep their calls
    # and argument rules here, and both parts of every split run on the GPU: this build has no CPU
    # compute path. The reference computes its two parts with the same exact arithmetic (rows are
    # quantized independently, output channels are independent), so the output is the whole
    # linear either way; ``cpu_queue`` is validated and bound but receives no work.

    def execute_hybrid(
        self: Self,
        destination: Tensor,
        source: Tensor,
        *,
        qpu_queue: Queue,
        cpu_queue: Queue,
        qpu_outputs: int,
        wait_for: Iterable[Event] = (),
    ) -> Event:
        """An aligned output-channel prefix and the disjoint tail (quantization.py:350-514)."""
        self._bind_hybrid_queues(qpu_queue, cpu_queue)
        self._check_hybrid_units("qpu_outputs", qpu_outputs, self.output_count)
        return self.execute(destination, source, queue=qpu_queue, wait_for=wait_for)

    def execute_hybrid_rows(
        self: Self,
        destination: Tensor,
        source: Tensor,
        *,
        qpu_queue: Queue,
        cpu_queue: Queue,
        qpu_rows: int,
        wait_for: Iterable[Event] = (),
    ) -> Event:
        """An aligned row prefix and the disjoint tail (quantization.py:516-662)."""
        self._bind_hybrid_queues(qpu_queue, cpu_queue)
        if len(source.shape) != 2:
            raise ValueError("prepared W8A8 linear requires rank-2 source and destination")
        self._check_hybrid_units("qpu_rows", qpu_rows, source.shape[0])
        return self.execute(destination, source, queue=qpu_queue, wait_for=wait_for)

    def execute_prepared_hybrid_rows(
        self: Self, destination: Tensor, *, batch: int, qpu_queue: Queue, cpu_queue: Queue, qpu_rows: int, wait_for: Iterable[Event] = ()
    ) -> Event:
        """The row split over activations already in the plan scratch (quantization.py:664-683)."""
        self._bind_hybrid_queues(qpu_queue, cpu_queue)
        if batch <= 0 or batch > self.max_batch:
            raise ValueError("prepared W8A8 linear batch exceeds the plan shape")
        self._check_hybrid_units("qpu_rows", qpu_rows, batch)
        return self.execute_prepared(destination, batch=batch, queue=qpu_queue, wait_for=wait_for)

    def execute_prepared_hybrid_outputs(
        self: Self, destination: Tensor, *, batch: int, qpu_queue: Queue, cpu_queue: Queue, qpu_outputs: int, wait_for: Iterable[Event] = ()
    ) -> Event:
        """The output split over activations already in the plan scratch (quantization.py:685-704)."""
        self._bind_hybrid_queues(qpu_queue, cpu_queue)
        if batch <= 0 or batch > self.max_batch:
            raise ValueError("prepared W8A8 linear batch exceeds the plan shape")
        self._check_hybrid_units("qpu_outputs", qpu_outputs, self.output_count)
        return self.execute_prepared(destination, batch=batch, queue=qpu_queue, wait_for=wait_for)

    def execute_prepared(self: Self, destination: Tensor, *, batch: int, queue: Queue, wait_for: Iterable[Event] = ()) -> Event:
        """Run on activations already quantized into the plan scratch (quantization.py:325-348)."""
        self._check_submission(queue)
        if destination.buffer.device is not self.device:
            raise DependencyError("prepared W8A8 linear queue and destination must belong to the plan device")
        if destination.dtype != np.dtype(np.float32) or len(destination.shape) != 2:
            raise ValueError("prepared W8A8 linear destination must be rank-2 float32")
        if batch <= 0 or batch > self.max_batch or destination.shape != (batch, self.output_count):
            raise ValueError("prepared W8A8 linear destination shape does not align")
        quantized, scales = self.scratch()
        handle = self._handle

        def executor(backend: Any, args: tuple[Any, ...], grid: tuple[int, int, int], stream: Any) -> None:
            backend.launch(
                stream,
                lambda native: native.check(
                    native.library.qpucuda_w8a8_linear_execute_prepared_device(
                        handle, quantized.data_ptr(), quantized.stride(0), scales.data_ptr(), batch,
                        destination.address, destination.row_stride_elements,
                    ),
                    "qpucuda_w8a8_linear_execute_prepared_device",
                ),
            )

        event = queue.submit(Kernel(self.kernel_name(batch), executor), (), wait_for=wait_for, buffers=(destination.access(AccessMode.WRITE),))
        self._last_event = event
        return event

    def forward(self: Self, source: Any, out: Any = None) -> Any:
        """Torch path on the current stream: fp32 ``[batch, K]`` CUDA tensor -> fp32 ``[batch, count]``."""
        import torch

        if self._closed:
            raise RuntimeError("prepared W8A8 linear plan is closed")
        batch = source.shape[0]
        if source.dtype != torch.float32 or source.dim() != 2 or source.shape[1] != self.weight.shape[1] or source.stride(1) != 1:
            raise ValueError("prepared W8A8 linear requires a row-major float32 [batch, K] source")
        if batch > self.max_batch:
            raise ValueError("prepared W8A8 linear source exceeds the plan shape")
        if out is None:
            out = torch.empty((batch, self.output_count), dtype=torch.float32, device=source.device)
        handle = self._handle
        self._backend.launch(  # type: ignore[attr-defined]
            torch.cuda.current_stream(source.device),
            lambda native: native.check(
                native.library.qpucuda_w8a8_linear_execute_device(handle, source.data_ptr(), source.stride(0), batch, out.data_ptr(), out.stride(0)),
                "qpucuda_w8a8_linear_execute_device",
            ),
        )
        return out

    def forward_fanout(self: Self, source: Any, destination: int, peer_destinations: Sequence[int], destination_stride: int) -> None:
        """``qpucuda_w8a8_linear_execute_device_fanout`` on the current stream: the fp32 outputs
        ``[batch, count]`` go to ``destination`` (a device address) and to every address in
        ``peer_destinations`` (other ranks' mapped buffers), rows ``destination_stride`` floats
        apart. No counterpart in the reference (the fused GEMM + all-gather of the N-split)."""
        import torch

        if self._closed:
            raise RuntimeError("prepared W8A8 linear plan is closed")
        batch = source.shape[0]
        if source.dtype != torch.float32 or source.dim() != 2 or source.shape[1] != self.weight.shape[1] or source.stride(1) != 1:
            raise ValueError("prepared W8A8 linear requires a row-major float32 [batch, K] source")
        peers = (ctypes.c_void_p * max(1, len(peer_destinations)))(*[ctypes.c_void_p(int(p)) for p in peer_destinations])
        handle = self._handle
        self._backend.launch(  # type: ignore[attr-defined]
            torch.cuda.current_stream(source.device),
            lambda native: native.check(
                native.library.qpucuda_w8a8_linear_execute_device_fanout(
                    handle, source.data_ptr(), source.stride(0), batch, int(destination), peers, len(peer_destinations), destination_stride
                ),
                "qpucuda_w8a8_linear_execute_device_fanout",
            ),
        )

    def execute_host(
        self: Self, source: npt.NDArray[np.float32], destination: npt.NDArray[np.float32] | None = None, *, direct: bool = False
    ) -> npt.NDArray[np.float32]:
        """Host buffers through ``qpucuda_w8a8_linear_execute`` (synchronous, bounded wait).

        ``direct=True`` calls ``qpucuda_w8a8_linear_execute_direct`` instead: ``destination`` must
        then be page-locked host memory (e.g. a ``pin_memory=True`` torch tensor's ``.numpy()``),
        the results are copied into it by DMA with no staging copy, and a failed wait may leave
        part of the results in it."""
        source = np.ascontiguousarray(source, dtype=np.float32)
        batch = source.shape[0]
        if destination is None:
            if direct:
                raise ValueError("direct host execution needs a page-locked destination")
            destination = np.empty((batch, self.output_count), dtype=np.float32)
        execution = _native.W8A8Execution(source.ctypes.data, source.nbytes, destination.ctypes.data, destination.nbytes, batch)
        name = "qpucuda_w8a8_linear_execute_direct" if direct else "qpucuda_w8a8_linear_execute"
        with self._backend.launch_lock:  # type: ignore[attr-defined]
            self._native.use_library_stream()
            status = getattr(self._native.library, name)(self._handle, ctypes.byref(execution))
        self._native.check(status, name)
        return destination

    def submit_direct(self: Self, source: npt.NDArray[np.float32], destination: npt.NDArray[np.float32]) -> W8A8Submission:
        """``qpucuda_w8a8_linear_submit_direct``: queue the host-buffer execution of ``execute_host(direct=True)``
        and return at once; ``W8A8Submission.wait`` returns the page-locked ``destination`` once it holds the
        results. Submissions on different plans overlap their host copies (for batches above 1024 rows)."""
        source = np.ascontiguousarray(source, dtype=np.float32)
        batch = source.shape[0]
        execution = _native.W8A8Execution(source.ctypes.data, source.nbytes, destination.ctypes.data, destination.nbytes, batch)
        handle = ctypes.c_void_p()
        with self._backend.launch_lock:  # type: ignore[attr-defined]
            self._native.use_library_stream()
            status = self._native.library.qpucuda_w8a8_linear_submit_direct(self._handle, ctypes.byref(execution), ctypes.byref(handle))
        self._native.check(status, "qpucuda_w8a8_linear_submit_direct")
        return W8A8Submission(self._native, int(handle.value), (source, destination))  # type: ignore[arg-type]


class W8A8Submission:
    """A queued host-buffer execution (``qpucuda_w8a8_linear_submit_direct``); ``wait`` blocks
    (bounded by the context timeout) until the results are in the destination."""

    def __init__(self: Self, native: Any, handle: int, keep: tuple[Any, ...]) -> None:
        self._native = native
        self._handle = handle
        self._keep = keep  # the source and destination stay alive until the wait
        self._status: int | None = None

    def wait(self: Self) -> Any:
        if self._status is None:
            self._status = int(self._native.library.qpucuda_w8a8_submission_wait(self._handle))
            self._native.library.qpucuda_w8a8_submission_destroy(self._handle)
        self._native.check(self._status, "qpucuda_w8a8_submission_wait")
        return self._keep[1]


def concatenate_output_channels(weights: Sequence[QuantizedMatrixInt8]) -> QuantizedMatrixInt8:
    """Stack int8 weight matrices of the same input width along the output-channel axis (each row
    keeps its own scale)."""
    if not weights:
        raise ValueError("concatenate_output_channels needs at least one weight")
    features = weights[0].shape[1]
    if any(w.shape[1] != features for w in weights):
        raise ValueError("merged W8A8 linears must share the input width")
    return QuantizedMatrixInt8(
        np.ascontiguousarray(np.concatenate([w.values for w in weights], axis=0)),
        np.ascontiguousarray(np.concatenate([w.scales for w in weights])),
    )


class MergedW8A8Linear:
    """Linears that read the same input (a layer's q/k/v, an FFN's gate/up) run as one plan.

    No counterpart in the reference, which quantizes the input once per linear
    (models/tinyllama/accelerated.py:228-266 calls each projection's plan). Here the int8 weights
    are stacked along the output channels, so one row quantization and one GEMM (or GEMV) launch
    produce every section. Each section equals its own :class:`PreparedW8A8Linear` bit for bit:
    activation rows are quantized without reference to the weights, the int32 dot of a column is
    exact in any order, and every output channel has its own scale (and bias). Either every section
    has a bias or none has one (a zero bias would turn a -0.0 output into +0.0).
    """

    def __init__(
        self: Self,
        device: Device,
        weights: Sequence[QuantizedMatrixInt8],
        *,
        max_batch: int,
        biases: Sequence[npt.NDArray[np.float32]] | None = None,
    ) -> None:
        merged = concatenate_output_channels(weights)
        self.sections = tuple(int(w.shape[0]) for w in weights)
        bias = None
        if biases is not None:
            if len(biases) != len(weights) or any(b is None for b in biases):
                raise ValueError("merged W8A8 linears need a bias for every section or for none")
            parts = [np.ascontiguousarray(b, dtype=np.float32) for b in biases]
            if any(p.shape != (n,) for p, n in zip(parts, self.sections)):
                raise ValueError("bias must have one fp32 value per output feature")
            bias = np.ascontiguousarray(np.concatenate(parts))
        self.bounds = tuple((int(a), int(b)) for a, b in zip(np.cumsum((0, *self.sections[:-1])), np.cumsum(self.sections)))
        self.plan = PreparedW8A8Linear(device, merged, max_batch=max_batch, bias=bias)

    @property
    def output_count(self: Self) -> int:
        return self.plan.output_count

    def split(self: Self, out: Any) -> list[Any]:
        """Column views of a merged ``[batch, output_count]`` output, one per section."""
        return [out[:, a:b] for a, b in self.bounds]

    def forward(self: Self, source: Any, out: Any = None) -> list[Any]:
        """Torch path on the current stream: fp32 ``[batch, K]`` -> one ``[batch, n_i]`` view per
        section of the merged output (``out``, ``[batch, output_count]``, when given)."""
        return self.split(self.plan.forward(source, out=out))

    def close(self: Self) -> None:
        self.plan.close()

    def __enter__(self: Self) -> Self:
        return self

    def __exit__(self: Self, exc_type: object, exc_value: object, traceback: object) -> None:
        self.close()


def _torch_view(address: int, shape: tuple[int, ...], dtype: Any, device: Any) -> Any:
    """Zero-copy torch tensor over device memory owned by libqpucuda."""
    import torch

    class _Holder:
        def __init__(self, address: int, shape: tuple[int, ...], typestr: str) -> None:
            self.__cuda_array_interface__ = {"shape": shape, "typestr": typestr, "data": (address, False), "version": 3}

    typestr = {torch.int8: "|i1", torch.float32: "<f4", torch.int32: "<i4", torch.uint8: "|u1"}[dtype]
    with torch.cuda.device(device):
        return torch.as_tensor(_Holder(address, shape, typestr), device=device)


class CalibratedW8A8Linear:
    """Placement-aware W8A8 linear (quantization.py:881-1082), with the single ``cuda`` placement.

    ``Placement.AUTO`` and ``Placement.CUDA`` run the prepared CUDA plan. The
    reference's AUTO gate on exact-shape "supported-win" records existed because
    its QPU could lose to the CPU; records with ``placement="cuda"`` are still
    consulted (the fastest one is reported by :attr:`last_selection`), but the
    CUDA path needs none to run. ``CPU``, ``QPU`` and ``HYBRID`` have no
    implementation in this build and raise ``ValueError``.
    """

    def __init__(
        self: Self,
        device: Device,
        weight: QuantizedMatrixInt8,
        *,
        max_batch: int,
        candidates: CandidateRegistry,
        bias: npt.NDArray[np.float32] | None = None,
    ) -> None:
        if max_batch <= 0:
            raise ValueError("calibrated W8A8 linear max_batch must be positive")
        self.device = device
        self.weight = weight
        self.max_batch = max_batch
        self.candidates = candidates
        self._cuda = PreparedW8A8Linear(device, weight, max_batch=max_batch, bias=bias) if device.is_cuda else None
        self.last_selection: CandidateRecord | None = None
        self._closed = False

    def __enter__(self: Self) -> Self:
        if self._closed:
            raise RuntimeError("calibrated W8A8 linear is closed")
        return self

    def __exit__(self: Self, exc_type: object, exc_value: object, traceback: object) -> None:
        self.close()

    def close(self: Self) -> None:
        if self._closed:
            return
        if self._cuda is not None:
            self._cuda.close()
        self._closed = True

    def supported_records(self: Self, batch: int) -> tuple[CandidateRecord, ...]:
        shape_class = f"{batch}x{self.weight.shape[1]}x{self.weight.shape[0]}"
        records = self.candidates.supported_for(operation="linear", dtype="w8a8-i32-fp32", layout="row-major-k", shape_class=shape_class)
        return tuple(record for record in records if record.placement == Placement.CUDA.value)

    def execute(
        self: Self,
        destination: Tensor,
        source: Tensor,
        *,
        queue: Queue,
        cpu_queue: Queue | None = None,
        placement: Placement = Placement.AUTO,
        qpu_rows: int | None = None,
        qpu_outputs: int | None = None,
        wait_for: Iterable[Event] = (),
    ) -> Event:
        if self._closed:
            raise RuntimeError("calibrated W8A8 linear is closed")
        if queue.device is not self.device:
            raise DependencyError("calibrated W8A8 queue belongs to a different device")
        if source.buffer.device is not self.device or destination.buffer.device is not self.device:
            raise DependencyError("calibrated W8A8 tensors belong to a different device")
        if source.dtype != np.dtype(np.float32) or destination.dtype != np.dtype(np.float32):
            raise ValueError("calibrated W8A8 linear requires FP32 source and destination")
        if len(source.shape) != 2 or len(destination.shape) != 2:
            raise ValueError("calibrated W8A8 linear requires rank-2 tensors")
        batch, features = source.shape
        if batch > self.max_batch or features != self.weight.shape[1]:
            raise ValueError("calibrated W8A8 source exceeds its planned shape")
        if destination.shape != (batch, self.weight.shape[0]):
            raise ValueError("calibrated W8A8 destination shape does not align")
        if qpu_rows is not None and qpu_outputs is not None:
            raise ValueError("qpu_rows and qpu_outputs are mutually exclusive")
        if qpu_rows is not None or qpu_outputs is not None:
            raise ValueError("CPU/QPU hybrid partitions do not exist on the CUDA build; use ShardedW8A8Linear")
        if placement not in (Placement.AUTO, Placement.CUDA):
            raise ValueError(f"placement {placement.value!r} is not available on the CUDA build; use 'cuda'")
        if self._cuda is None:
            raise ValueError("the cuda placement needs a device opened on the CUDA backend")
        records = self.supported_records(batch)
        self.last_selection = (
            min(records, key=lambda r: r.performance.candidate_median_seconds if r.performance else float("inf"))
            if records
            else None
        )
        return self._cuda.execute(destination, source, queue=queue, wait_for=wait_for)


__all__ = [
    "CalibratedW8A8Linear",
    "MergedW8A8Linear",
    "W8A8Submission",
    "PreparedW8A8Linear",
    "QuantizedMatrixInt8",
    "concatenate_output_channels",
    "quantize_per_output_channel_int8",
]
