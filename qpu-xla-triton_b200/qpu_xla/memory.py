"""Buffers and typed tensor views over device allocations.

The drop-in surface of src/qpu_xla/memory.py (``AccessMode``, ``BufferAccess``,
``Buffer.slice/access/tensor``, strided ``Tensor`` views with unit-step
``slice``), built around this build's allocation blocks:

* every allocation handed out by a device is a :class:`_Block`; buffers and
  tensors are byte windows ``[start, start + length)`` of one block, and a block
  retired by ``Buffer.close()`` or ``Device.close()`` invalidates every window
  over it at once;
* a declared access is the byte interval it covers in its block, so hazard
  checks are interval tests between accesses of the same block;
* CUDA memory is not host-mapped: ``Tensor.numpy()`` is a zero-copy view on the
  fake backend but a device-to-host copy on the CUDA backend,
  ``Tensor.torch()`` is the zero-copy view of CUDA memory, and
  ``Tensor.write(values)`` copies host data in.
"""

from __future__ import annotations

import math
from enum import Enum
from typing import TYPE_CHECKING, Any, Self

import numpy as np
import numpy.typing as npt

from qpu_xla.backend import BackendAllocation
from qpu_xla.errors import AllocationError, BufferClosedError

if TYPE_CHECKING:
    from qpu_xla.device import Device


class AccessMode(Enum):
    """How a queue submission uses a declared byte range."""

    READ = "read"
    WRITE = "write"
    READ_WRITE = "read_write"

    @property
    def writes(self: Self) -> bool:
        return self in _WRITING_MODES


_WRITING_MODES = frozenset({AccessMode.WRITE, AccessMode.READ_WRITE})


class _Block:
    """One allocation lent out by a device's pool. ``live`` turns false exactly once, when the
    block is retired; every buffer, tensor and access over it checks that flag."""

    __slots__ = ("allocation", "live", "_on_retire")

    def __init__(self: Self, allocation: BackendAllocation, on_retire: Any = None) -> None:
        self.allocation = allocation
        self.live = True
        self._on_retire = on_retire

    @property
    def size(self: Self) -> int:
        return self.allocation.nbytes

    def check(self: Self) -> None:
        if not self.live:
            raise BufferClosedError("buffer is closed")

    def retire(self: Self, *, recycle: bool) -> None:
        """Invalidate the block; with ``recycle`` its allocation goes back to the owner's pool."""
        if not self.live:
            return
        self.live = False
        if recycle and self._on_retire is not None:
            self._on_retire(self.allocation)


def _window(size: int, start: int, length: int | None, message: str) -> tuple[int, int]:
    """``[start, start + length)`` inside ``[0, size)`` with a non-empty length (default: to the end)."""
    length = size - start if length is None else length
    if start < 0 or length <= 0 or start + length > size:
        raise AllocationError(message)
    return start, length


class BufferAccess:
    """A declared byte range of a buffer and its access mode, for queue hazard tracking."""

    __slots__ = ("buffer", "mode", "offset", "nbytes", "_lo", "_hi")

    def __init__(self: Self, buffer: Buffer, mode: AccessMode, offset: int = 0, nbytes: int | None = None) -> None:
        buffer._block.check()
        offset, nbytes = _window(buffer._length, offset, nbytes, "buffer access range is outside the buffer")
        self.buffer = buffer
        self.mode = mode
        self.offset = offset
        self.nbytes = nbytes
        self._lo = buffer._start + offset
        self._hi = self._lo + nbytes

    @property
    def absolute_offset(self: Self) -> int:
        """Offset of the range from the start of its allocation."""
        return self._lo

    def conflicts_with(self: Self, other: BufferAccess) -> bool:
        """True when both ranges lie in one allocation, overlap, and at least one of them writes."""
        if self.buffer._block is not other.buffer._block:
            return False
        if not (self.mode.writes or other.mode.writes):
            return False
        return max(self._lo, other._lo) < min(self._hi, other._hi)

    def __repr__(self: Self) -> str:
        return f"BufferAccess({self.mode.value}, [{self._lo}, {self._hi}))"


class Buffer:
    """A byte window of one device allocation."""

    def __init__(self: Self, device: Device, block: _Block, *, offset: int = 0, nbytes: int | None = None) -> None:
        block.check()
        self._start, self._length = _window(block.size, offset, nbytes, "buffer range is outside its allocation")
        self._device = device
        self._block = block

    @property
    def device(self: Self) -> Device:
        return self._device

    @property
    def offset(self: Self) -> int:
        """Byte offset of this window in its allocation."""
        return self._start

    @property
    def nbytes(self: Self) -> int:
        self._block.check()
        return self._length

    @property
    def address(self: Self) -> int:
        """Device address of the window (a 64-bit CUDA pointer on the cuda backend)."""
        self._block.check()
        return self._block.allocation.address + self._start

    @property
    def closed(self: Self) -> bool:
        return not self._block.live

    def close(self: Self) -> None:
        """Invalidate this allocation and every view of it, and give it back to the device."""
        self._block.retire(recycle=True)

    def slice(self: Self, offset: int, nbytes: int | None = None) -> Buffer:
        self._block.check()
        offset, nbytes = _window(self._length, offset, nbytes, "buffer range is outside its allocation")
        return Buffer(self._device, self._block, offset=self._start + offset, nbytes=nbytes)

    def access(self: Self, mode: AccessMode, *, offset: int = 0, nbytes: int | None = None) -> BufferAccess:
        return BufferAccess(self, mode, offset, nbytes)

    def tensor(
        self: Self, shape: tuple[int, ...], dtype: npt.DTypeLike, *, offset: int = 0, strides: tuple[int, ...] | None = None
    ) -> Tensor:
        return Tensor(self, shape, dtype, offset=offset, strides=strides)


_TORCH_DTYPES = frozenset({"float32", "float16", "int8", "uint8", "int16", "int32", "int64", "uint16", "uint32"})


def torch_dtype(dtype: np.dtype[Any]) -> Any:
    import torch

    name = np.dtype(dtype).name
    if name not in _TORCH_DTYPES:
        raise AllocationError(f"dtype {dtype} has no torch equivalent")
    return getattr(torch, name)


def _row_major(shape: tuple[int, ...], itemsize: int) -> tuple[int, ...]:
    """Byte strides of a C-ordered array of ``shape``."""
    tail = np.cumprod((1,) + shape[:0:-1])[::-1] if len(shape) > 1 else np.ones(1, dtype=np.int64)
    return tuple(int(value) * itemsize for value in tail)


def _extent(shape: tuple[int, ...], itemsize: int, strides: tuple[int, ...]) -> int:
    """Bytes from the first element to the end of the last one, for positive strides."""
    return itemsize + math.sumprod((d - 1 for d in shape), strides)


class Tensor:
    """A typed, strided view of a buffer (byte offset, byte strides)."""

    def __init__(
        self: Self,
        buffer: Buffer,
        shape: tuple[int, ...],
        dtype: npt.DTypeLike,
        *,
        offset: int = 0,
        strides: tuple[int, ...] | None = None,
    ) -> None:
        buffer._block.check()
        dims = tuple(int(d) for d in shape)
        if not dims or min(dims) <= 0:
            raise AllocationError("tensor shape must contain only positive dimensions")
        element = np.dtype(dtype)
        size = element.itemsize
        if offset < 0 or offset % size:
            raise AllocationError("tensor offset must be non-negative and aligned to the dtype")
        steps = _row_major(dims, size) if strides is None else tuple(int(s) for s in strides)
        if len(steps) != len(dims) or any(s <= 0 or s % size for s in steps):
            raise AllocationError("tensor strides must be positive, dtype-aligned byte strides for every dimension")
        if offset + _extent(dims, size, steps) > buffer.nbytes:
            raise AllocationError("tensor view exceeds its buffer")
        self._buffer = buffer
        self._shape = dims
        self._dtype = element
        self._offset = offset
        self._strides = steps

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
        """Bytes the view spans in its buffer."""
        self._buffer._block.check()
        return _extent(self._shape, self._dtype.itemsize, self._strides)

    @property
    def address(self: Self) -> int:
        """Device address of element [0, ..., 0]."""
        return self._buffer.address + self._offset

    @property
    def is_contiguous(self: Self) -> bool:
        return self._strides == _row_major(self._shape, self._dtype.itemsize)

    @property
    def row_stride_elements(self: Self) -> int:
        """Leading-dimension stride in elements (rank-2 views)."""
        return self._strides[0] // self._dtype.itemsize

    def _allocation(self: Self) -> BackendAllocation:
        block = self._buffer._block
        block.check()
        return block.allocation

    def numpy(self: Self) -> npt.NDArray[Any]:
        """Zero-copy view on the fake backend; a device-to-host copy on the CUDA backend.

        On CUDA the copy is taken after synchronizing the device, so call it once the
        producing event has been waited on.
        """
        allocation = self._allocation()
        if allocation.host_mapped:
            return np.ndarray(
                self._shape, dtype=self._dtype, buffer=allocation.storage,
                offset=self._buffer.offset + self._offset, strides=self._strides,
            )
        import torch

        view = self.torch()
        torch.cuda.synchronize(view.device)
        return view.cpu().numpy()

    def torch(self: Self) -> Any:
        """Zero-copy torch view (CUDA backend), or a torch view of the NumPy memory (fake backend)."""
        import torch

        allocation = self._allocation()
        if allocation.host_mapped:
            return torch.from_numpy(self.numpy())
        first = self._buffer.offset + self._offset
        flat = allocation.storage[first : first + self.nbytes].view(torch_dtype(self._dtype))
        size = self._dtype.itemsize
        return flat.as_strided(self._shape, tuple(step // size for step in self._strides))

    def write(self: Self, values: npt.ArrayLike) -> None:
        """Copy host ``values`` (broadcast to this shape) into the tensor."""
        host = np.broadcast_to(np.asarray(values, dtype=self._dtype), self._shape)
        if self._allocation().host_mapped:
            self.numpy()[...] = host
            return
        import torch

        self.torch().copy_(torch.from_numpy(np.array(host, order="C", copy=True)))

    def slice(self: Self, slices: tuple[slice, ...]) -> Tensor:
        """A unit-step sub-view sharing this tensor's memory."""
        if len(slices) != len(self._shape):
            raise AllocationError("one slice is required for each tensor dimension")
        bounds = [item.indices(extent) for item, extent in zip(slices, self._shape, strict=True)]
        if any(step != 1 for _, _, step in bounds):
            raise AllocationError("only unit-step tensor slices are currently supported")
        if any(stop <= start for start, stop, _ in bounds):
            raise AllocationError("tensor slices must not be empty")
        first = self._offset + sum(start * step for (start, _, _), step in zip(bounds, self._strides, strict=True))
        shape = tuple(stop - start for start, stop, _ in bounds)
        return Tensor(self._buffer, shape, self._dtype, offset=first, strides=self._strides)

    def access(self: Self, mode: AccessMode) -> BufferAccess:
        return self._buffer.access(mode, offset=self._offset, nbytes=self.nbytes)


__all__ = ["AccessMode", "Buffer", "BufferAccess", "Tensor"]
