"""Buffers and typed tensor views over backend allocations.

Same surface and checks as src/qpu_xla/memory.py:18-265 (``AccessMode``,
``BufferAccess`` hazard ranges, ``Buffer.slice/access/tensor``, strided
``Tensor`` views with unit-step ``slice``). Differences forced by CUDA memory:

* ``Tensor.numpy()`` is zero-copy on the fake backend, as in the reference, but
  a device-to-host *copy* on the CUDA backend (device memory is not host-mapped);
* ``Tensor.torch()`` is the zero-copy view of CUDA memory, and
  ``Tensor.write(values)`` copies host data in.
"""

from __future__ import annotations

from dataclasses import dataclass
from enum import Enum
from typing import TYPE_CHECKING, Any, Self

import numpy as np
import numpy.typing as npt

from qpu_xla.backend import BackendAllocation
from qpu_xla.errors import AllocationError, BufferClosedError

if TYPE_CHECKING:
    from qpu_xla.device import Device


class AccessMode(Enum):
    """Declared access mode for a buffer range used by a queue submission."""

    READ = "read"
    WRITE = "write"
    READ_WRITE = "read_write"

    @property
    def writes(self: Self) -> bool:
        return self is not AccessMode.READ


@dataclass(slots=True)
class _AllocationState:
    """Close state shared by a buffer and every view derived from it."""

    allocation: BackendAllocation
    closed: bool = False

    def require_open(self: Self) -> None:
        if self.closed:
            raise BufferClosedError("buffer is closed")


@dataclass(frozen=True, slots=True)
class BufferAccess:
    """A declared byte range and access mode, used for hazard tracking."""

    buffer: Buffer
    mode: AccessMode
    offset: int = 0
    nbytes: int | None = None

    def __post_init__(self: Self) -> None:
        self.buffer._state.require_open()
        nbytes = self.buffer.nbytes - self.offset if self.nbytes is None else self.nbytes
        if self.offset < 0 or nbytes <= 0 or self.offset + nbytes > self.buffer.nbytes:
            raise AllocationError("buffer access range is outside the buffer")
        object.__setattr__(self, "nbytes", nbytes)

    @property
    def absolute_offset(self: Self) -> int:
        return self.buffer.offset + self.offset

    def conflicts_with(self: Self, other: BufferAccess) -> bool:
        """Two accesses conflict when they overlap in one allocation and one of them writes."""
        if self.buffer._state is not other.buffer._state or not (self.mode.writes or other.mode.writes):
            return False
        assert self.nbytes is not None and other.nbytes is not None
        return (
            self.absolute_offset < other.absolute_offset + other.nbytes
            and other.absolute_offset < self.absolute_offset + self.nbytes
        )


class Buffer:
    """A runtime-owned byte range of one allocation."""

    def __init__(self: Self, device: Device, state: _AllocationState, *, offset: int = 0, nbytes: int | None = None) -> None:
        state.require_open()
        total = state.allocation.nbytes
        nbytes = total - offset if nbytes is None else nbytes
        if offset < 0 or nbytes <= 0 or offset + nbytes > total:
            raise AllocationError("buffer range is outside its allocation")
        self._device = device
        self._state = state
        self._offset = offset
        self._nbytes = nbytes

    @property
    def device(self: Self) -> Device:
        return self._device

    @property
    def offset(self: Self) -> int:
        return self._offset

    @property
    def nbytes(self: Self) -> int:
        self._state.require_open()
        return self._nbytes

    @property
    def address(self: Self) -> int:
        """Device address of this range (a 64-bit CUDA pointer on the cuda backend)."""
        self._state.require_open()
        return self._state.allocation.address + self._offset

    @property
    def closed(self: Self) -> bool:
        return self._state.closed

    def close(self: Self) -> None:
        if self._state.closed:
            return
        self._state.closed = True
        self._device._release_allocation(self._state)

    def slice(self: Self, offset: int, nbytes: int | None = None) -> Buffer:
        self._state.require_open()
        nbytes = self._nbytes - offset if nbytes is None else nbytes
        return Buffer(self._device, self._state, offset=self._offset + offset, nbytes=nbytes)

    def access(self: Self, mode: AccessMode, *, offset: int = 0, nbytes: int | None = None) -> BufferAccess:
        return BufferAccess(self, mode, offset, nbytes)

    def tensor(
        self: Self, shape: tuple[int, ...], dtype: npt.DTypeLike, *, offset: int = 0, strides: tuple[int, ...] | None = None
    ) -> Tensor:
        return Tensor(self, shape, dtype, offset=offset, strides=strides)


_TORCH_DTYPES: dict[str, str] = {
    "float32": "float32",
    "float16": "float16",
    "int8": "int8",
    "uint8": "uint8",
    "int16": "int16",
    "int32": "int32",
    "int64": "int64",
    "uint16": "uint16",
    "uint32": "uint32",
}


def torch_dtype(dtype: np.dtype[Any]) -> Any:
    import torch

    name = _TORCH_DTYPES.get(np.dtype(dtype).name)
    if name is None:
        raise AllocationError(f"dtype {dtype} has no torch equivalent")
    return getattr(torch, name)


class Tensor:
    """A typed, strided view of one buffer (byte offsets and byte strides)."""

    def __init__(
        self: Self,
        buffer: Buffer,
        shape: tuple[int, ...],
        dtype: npt.DTypeLike,
        *,
        offset: int = 0,
        strides: tuple[int, ...] | None = None,
    ) -> None:
        buffer._state.require_open()
        shape = tuple(int(d) for d in shape)
        if not shape or any(dimension <= 0 for dimension in shape):
            raise AllocationError("tensor shape must contain only positive dimensions")
        dtype = np.dtype(dtype)
        if offset < 0 or offset % dtype.itemsize:
            raise AllocationError("tensor offset must be non-negative and aligned to the dtype")
        strides = self._contiguous_strides(shape, dtype.itemsize) if strides is None else tuple(int(s) for s in strides)
        if len(strides) != len(shape) or any(stride <= 0 or stride % dtype.itemsize for stride in strides):
            raise AllocationError("tensor strides must be positive, dtype-aligned byte strides for every dimension")
        if offset + self._required_nbytes(shape, dtype.itemsize, strides) > buffer.nbytes:
            raise AllocationError("tensor view exceeds its buffer")
        self._buffer = buffer
        self._shape = shape
        self._dtype = dtype
        self._offset = offset
        self._strides = strides

    @staticmethod
    def _contiguous_strides(shape: tuple[int, ...], itemsize: int) -> tuple[int, ...]:
        strides: list[int] = []
        stride = itemsize
        for dimension in reversed(shape):
            strides.append(stride)
            stride *= dimension
        return tuple(reversed(strides))

    @staticmethod
    def _required_nbytes(shape: tuple[int, ...], itemsize: int, strides: tuple[int, ...]) -> int:
        return itemsize + sum((dimension - 1) * stride for dimension, stride in zip(shape, strides, strict=True))

    @property
    def buffer(self: Self) -> Buffer:
        return self._buffer

    @property
    def shape(self: Self) -> tuple[int, ...]:
        return self._shape

    @property
    def dtype(self: Self) -> np.dtype[Any]:
        return self._dtype

    @property
    def strides(self: Self) -> tuple[int, ...]:
        return self._strides

    @property
    def nbytes(self: Self) -> int:
        self._buffer._state.require_open()
        return self._required_nbytes(self._shape, self._dtype.itemsize, self._strides)

    @property
    def address(self: Self) -> int:
        self._buffer._state.require_open()
        return self._buffer.address + self._offset

    @property
    def is_contiguous(self: Self) -> bool:
        return self._strides == self._contiguous_strides(self._shape, self._dtype.itemsize)

    @property
    def row_stride_elements(self: Self) -> int:
        """Leading-dimension stride in elements (rank-2 views)."""
        return self._strides[0] // self._dtype.itemsize

    def _host_mapped(self: Self) -> bool:
        return bool(self._buffer._state.allocation.host_mapped)

    def numpy(self: Self) -> npt.NDArray[Any]:
        """Zero-copy view on the fake backend; a device-to-host copy on the CUDA backend.

        On CUDA the copy is taken after synchronizing the device, so call it
        once the producing event has been waited on.
        """
        self._buffer._state.require_open()
        if self._host_mapped():
            return np.ndarray(
                self._shape,
                dtype=self._dtype,
                buffer=self._buffer._state.allocation.storage,
                offset=self._buffer.offset + self._offset,
                strides=self._strides,
            )
        import torch

        view = self.torch()
        torch.cuda.synchronize(view.device)
        return view.cpu().numpy()

    def torch(self: Self) -> Any:
        """Zero-copy torch view (CUDA backend) or a torch view of the NumPy memory (fake backend)."""
        import torch

        self._buffer._state.require_open()
        if self._host_mapped():
            return torch.from_numpy(self.numpy())
        storage = self._buffer._state.allocation.storage
        start = self._buffer.offset + self._offset
        span = self.nbytes
        flat = storage[start : start + span].view(torch_dtype(self._dtype))
        itemsize = self._dtype.itemsize
        return flat.as_strided(self._shape, tuple(stride // itemsize for stride in self._strides))

    def write(self: Self, values: npt.ArrayLike) -> None:
        """Copy host ``values`` (broadcast to this shape) into the tensor."""
        array = np.broadcast_to(np.asarray(values, dtype=self._dtype), self._shape)
        if self._host_mapped():
            self.numpy()[...] = array
            return
        import torch

        host = np.ascontiguousarray(array)
        if not host.flags.writeable:
            host = host.copy()
        self.torch().copy_(torch.from_numpy(host))

    def slice(self: Self, slices: tuple[slice, ...]) -> Tensor:
        """Unit-step slice without copying (memory.py:247-261)."""
        if len(slices) != len(self._shape):
            raise AllocationError("one slice is required for each tensor dimension")
        shape: list[int] = []
        offset = self._offset
        for dimension, stride, item in zip(self._shape, self._strides, slices, strict=True):
            start, stop, step = item.indices(dimension)
            if step != 1:
                raise AllocationError("only unit-step tensor slices are currently supported")
            if stop <= start:
                raise AllocationError("tensor slices must not be empty")
            shape.append(stop - start)
            offset += start * stride
        return Tensor(self._buffer, tuple(shape), self._dtype, offset=offset, strides=self._strides)

    def access(self: Self, mode: AccessMode) -> BufferAccess:
        return self._buffer.access(mode, offset=self._offset, nbytes=self.nbytes)


__all__ = ["AccessMode", "Buffer", "BufferAccess", "Tensor"]
