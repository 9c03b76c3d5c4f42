"""Persistent W8A8 convolution plan on the GPU (src/qpu_xla/ops/conv2d_w8a8.py:22-137).

Same constructor and ``execute`` contract as the reference: a fixed NCHW source shape and fp32
OIHW weight quantized per output channel once at construction, one W8A8 linear plan per group,
fp32 in and out. The lowering runs on the device:

* pointwise 1x1 convolutions (stride 1, no padding, no dilation) hand the NCHW pixels to the row
  quantizer in place, through a ``qpucuda_matrix_layout`` of pixels x channels (the reference's
  ``_pointwise_nchw_matrix`` view, src/qpu_xla/ops/conv2d.py:93-96), with no transpose copy;
* other kernels are lowered by ``qpucuda_im2col_nchw_f32`` (``_im2col_nchw``, conv2d.py:47-79)
  into a plan-owned fp32 workspace, one group at a time;

and every group's GEMM writes its output channels straight into the NCHW destination through
the epilogue's layout (the reference restores NCHW on the host, conv2d_w8a8.py:296-305). Each
group is the dynamic W8A8 linear of the reference, so the result equals the reference's per-group
dynamic W8A8 convolution (tests/test_qpu_xla_conv2d_w8a8.py:14-54) bit for bit.

Not built here: the reference's direct depthwise 3x3 QPU kernel (a depthwise convolution runs as
per-group GEMMs) and the CPU/QPU ``execute_hybrid`` split (this build has no CPU path).
"""

from __future__ import annotations

import ctypes
from collections.abc import Iterable
from typing import Any, Self, cast

import numpy as np
import numpy.typing as npt

from qpu_xla import _native
from qpu_xla.device import Device
from qpu_xla.errors import DependencyError, DeviceClosedError
from qpu_xla.kernel import Kernel
from qpu_xla.memory import AccessMode, Tensor
from qpu_xla.queue import Event, Queue


def _pair(value: int | tuple[int, int], *, name: str) -> tuple[int, int]:
    """One non-negative scalar or pair convolution parameter (conv2d.py:17-22)."""
    pair = (value, value) if isinstance(value, int) else tuple(value)
    if len(pair) != 2 or any(component < 0 for component in pair):
        raise ValueError(f"{name} must contain two non-negative integers")
    return cast(tuple[int, int], pair)


def output_hw(height: int, width: int, kernel_height: int, kernel_width: int, stride: tuple[int, int], padding: tuple[int, int], dilation: tuple[int, int]) -> tuple[int, int]:
    """Valid NCHW convolution output size (conv2d.py:25-39)."""
    output_height = (height + 2 * padding[0] - dilation[0] * (kernel_height - 1) - 1) // stride[0] + 1
    output_width = (width + 2 * padding[1] - dilation[1] * (kernel_width - 1) - 1) // stride[1] + 1
    if output_height <= 0 or output_width <= 0:
        raise ValueError("convolution parameters produce an empty output")
    return output_height, output_width


def is_pointwise_1x1(kernel_height: int, kernel_width: int, stride: tuple[int, int], padding: tuple[int, int], dilation: tuple[int, int]) -> bool:
    """The reference's in-place lowering condition (conv2d.py:82-90)."""
    return (kernel_height, kernel_width) == (1, 1) and stride == (1, 1) and padding == (0, 0) and dilation == (1, 1)


class Conv2dW8A8Plan:
    """Reuse quantized weights and workspaces for fp32-in/fp32-out W8A8 convolution."""

    def __init__(
        self: Self,
        device: Device,
        *,
        source_shape: tuple[int, int, int, int],
        weight: npt.NDArray[np.float32],
        stride: int | tuple[int, int] = 1,
        padding: int | tuple[int, int] = 0,
        dilation: int | tuple[int, int] = 1,
        groups: int = 1,
    ) -> None:
        import torch

        from qpu_xla.quantization import PreparedW8A8Linear, quantize_per_output_channel_int8

        if len(source_shape) != 4 or any(dimension <= 0 for dimension in source_shape):
            raise ValueError("W8A8 convolution source shape must be positive NCHW")
        if weight.ndim != 4 or weight.dtype != np.dtype(np.float32) or not weight.flags.c_contiguous:
            raise ValueError("W8A8 convolution weight must be contiguous FP32 OIHW")
        if groups <= 0:
            raise ValueError("W8A8 convolution groups must be positive")
        if not device.is_cuda:
            raise ValueError("Conv2dW8A8Plan requires the CUDA backend (this build has no CPU path)")
        batch, in_channels, height, width = source_shape
        out_channels, weight_channels, kernel_height, kernel_width = weight.shape
        if in_channels % groups or out_channels % groups or weight_channels != in_channels // groups:
            raise ValueError("W8A8 grouped convolution channels do not align")
        self.device = device
        self.source_shape = tuple(int(d) for d in source_shape)
        self.weight_shape = cast(tuple[int, int, int, int], weight.shape)
        self.stride = _pair(stride, name="stride")
        self.padding = _pair(padding, name="padding")
        self.dilation = _pair(dilation, name="dilation")
        if any(component == 0 for component in self.stride + self.dilation):
            raise ValueError("W8A8 convolution stride and dilation must be positive")
        self.groups = groups
        output_height, output_width = output_hw(height, width, kernel_height, kernel_width, self.stride, self.padding, self.dilation)
        self.destination_shape = (batch, out_channels, output_height, output_width)
        self.rows = batch * output_height * output_width
        self.input_channels_per_group = in_channels // groups
        self.output_channels_per_group = out_channels // groups
        self.reduction_per_group = self.input_channels_per_group * kernel_height * kernel_width
        self.pointwise = is_pointwise_1x1(kernel_height, kernel_width, self.stride, self.padding, self.dilation)
        self._plans: list[PreparedW8A8Linear] = []
        try:
            for group in range(groups):
                start = group * self.output_channels_per_group
                matrix = np.ascontiguousarray(weight[start : start + self.output_channels_per_group].reshape(self.output_channels_per_group, self.reduction_per_group))
                quantized = quantize_per_output_channel_int8(matrix, device=device)
                self._plans.append(PreparedW8A8Linear(device, quantized, max_batch=self.rows))
        except BaseException:
            for plan in self._plans:
                plan.close()
            raise
        self._workspace = (
            None
            if self.pointwise
            else torch.empty((self.rows, self.reduction_per_group), dtype=torch.float32, device=device.backend.torch_device)  # type: ignore[attr-defined]
        )
        self._queue: Queue | None = None
        self._tail: Event | None = None
        self._closed = False

    def __enter__(self: Self) -> Self:
        if self._closed:
            raise DeviceClosedError("W8A8 convolution plan is closed")
        return self

    def __exit__(self: Self, exc_type: object, exc_value: object, traceback: object) -> None:
        self.close()

    def close(self: Self) -> None:
        """Wait for outstanding work and release the per-group plans."""
        if self._closed:
            return
        if self._tail is not None:
            self._tail.wait()
        for plan in self._plans:
            plan.close()
        self._workspace = None
        self._closed = True

    def _layouts(self: Self, source: Tensor, destination: Tensor, group: int) -> tuple[int, Any, int, Any]:
        """(source address, source layout, destination address, destination layout) of one group."""
        batch, channels, height, width = self.source_shape
        _, out_channels, output_height, output_width = self.destination_shape
        pixels = output_height * output_width
        destination_address = destination.address + 4 * group * self.output_channels_per_group * pixels
        destination_layout = _native.MatrixLayout(pixels, out_channels * pixels, 1, pixels)
        if self.pointwise:
            source_address = source.address + 4 * group * self.input_channels_per_group * height * width
            source_layout = _native.MatrixLayout(height * width, channels * height * width, 1, height * width)
        else:
            assert self._workspace is not None
            source_address = self._workspace.data_ptr()
            source_layout = _native.MatrixLayout(0, 0, self.reduction_per_group, 1)
        return source_address, source_layout, destination_address, destination_layout

    def execute(self: Self, destination: Tensor, source: Tensor, *, queue: Queue, wait_for: Iterable[Event] = ()) -> Event:
        """Lower ``source``, run one W8A8 GEMM per group and write NCHW ``destination`` (conv2d_w8a8.py:171-305)."""
        if self._closed:
            raise DeviceClosedError("W8A8 convolution plan is closed")
        if self._tail is not None and not self._tail.done:
            raise RuntimeError("W8A8 convolution plan already has an in-flight invocation")
        if self._queue is None:
            self._queue = queue
        elif self._queue is not queue:
            raise DependencyError("W8A8 convolution plan is bound to its first submission queue")
        if queue.device is not self.device:
            raise DependencyError("W8A8 convolution queue belongs to a different device")
        if source.buffer.device is not self.device or destination.buffer.device is not self.device:
            raise DependencyError("W8A8 convolution tensors must belong to the plan device")
        if source.dtype != np.dtype(np.float32) or destination.dtype != np.dtype(np.float32):
            raise ValueError("W8A8 convolution requires FP32 source and destination")
        if source.shape != self.source_shape or destination.shape != self.destination_shape:
            raise ValueError("W8A8 convolution tensors do not match the planned topology")
        if not source.is_contiguous or not destination.is_contiguous:
            raise ValueError("W8A8 convolution requires contiguous NCHW tensors")
        batch, channels, height, width = self.source_shape
        kernel_height, kernel_width = self.weight_shape[2:]
        groups = [(plan._handle, *self._layouts(source, destination, group)) for group, plan in enumerate(self._plans)]
        workspace = self._workspace
        rows = self.rows

        def run(native: Any) -> None:
            for group, (handle, source_address, source_layout, destination_address, destination_layout) in enumerate(groups):
                if workspace is not None:
                    native.check(
                        native.library.qpucuda_im2col_nchw_f32(
                            native.handle, source.address, batch, channels, height, width,
                            group * self.input_channels_per_group, self.input_channels_per_group, kernel_height, kernel_width,
                            self.stride[0], self.stride[1], self.padding[0], self.padding[1], self.dilation[0], self.dilation[1],
                            workspace.data_ptr(), self.reduction_per_group,
                        ),
                        "qpucuda_im2col_nchw_f32",
                    )
                native.check(
                    native.library.qpucuda_w8a8_linear_execute_device_layout(
                        handle, source_address, ctypes.byref(source_layout), rows, destination_address, ctypes.byref(destination_layout)
                    ),
                    "qpucuda_w8a8_linear_execute_device_layout",
                )

        def executor(backend: Any, args: tuple[Any, ...], grid: tuple[int, int, int], stream: Any) -> None:
            backend.launch(stream, run)

        event = queue.submit(
            Kernel("cuda.conv2d_w8a8", executor),
            (),
            wait_for=wait_for,
            buffers=(source.access(AccessMode.READ), destination.access(AccessMode.WRITE)),
        )
        self._tail = event
        return event


__all__ = ["Conv2dW8A8Plan", "is_pointwise_1x1", "output_hw"]
