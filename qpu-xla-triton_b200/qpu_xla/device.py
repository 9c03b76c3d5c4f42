"""Device lifetime and allocation entry points (src/qpu_xla/device.py:17-121).

``Device.open()`` opens the CUDA backend on one GPU (the reference opened the
VideoCore DRM driver); ``Device.fake()`` keeps the CPU-only test backend.
"""

from __future__ import annotations

from typing import TYPE_CHECKING, Any, Self
from weakref import WeakSet

import numpy as np
import numpy.typing as npt

from qpu_xla.backend import Backend, BackendAllocation, CudaBackend, FakeBackend, _validate_allocation_request
from qpu_xla.errors import DeviceClosedError
from qpu_xla.memory import Buffer, Tensor, _AllocationState

if TYPE_CHECKING:
    from qpu_xla.queue import Queue


class Device:
    """An owned device context over one backend."""

    def __init__(self: Self, backend: Backend) -> None:
        self._backend = backend
        self._closed = False
        self._allocations: list[_AllocationState] = []
        self._free_allocations: list[BackendAllocation] = []
        self._queues: WeakSet[Queue] = WeakSet()

    @classmethod
    def fake(cls: type[Device]) -> Device:
        """CPU-only device for runtime tests; it cannot launch kernels."""
        return cls(FakeBackend())

    @classmethod
    def open(cls: type[Device], *, device_ordinal: int | None = None, backend: str = "cuda", **options: Any) -> Device:
        """Open the CUDA backend on ``device_ordinal`` (default: the current CUDA device).

        ``options`` go to :class:`CudaBackend` (``timeout_ns``, ``failure_mask``).
        ``backend="cuda"`` is the only hardware backend of this build.
        """
        if backend != "cuda":
            raise ValueError("this build provides the 'cuda' backend only")
        return cls(CudaBackend(device_ordinal, **options))

    @property
    def backend(self: Self) -> Backend:
        self._require_open()
        return self._backend

    @property
    def is_cuda(self: Self) -> bool:
        return getattr(self._backend, "kind", "") == "cuda"

    @property
    def closed(self: Self) -> bool:
        return self._closed

    def _require_open(self: Self) -> None:
        if self._closed:
            raise DeviceClosedError("device is closed")

    def allocate(self: Self, nbytes: int, *, alignment: int = 1) -> Buffer:
        """Allocate (or reuse a released) byte buffer owned by this device."""
        self._require_open()
        _validate_allocation_request(nbytes, alignment)
        allocation = self._take_free_allocation(nbytes, alignment)
        state = _AllocationState(allocation)
        self._allocations.append(state)
        return Buffer(self, state, nbytes=nbytes)

    def _take_free_allocation(self: Self, nbytes: int, alignment: int) -> BackendAllocation:
        compatible = [
            (index, allocation)
            for index, allocation in enumerate(self._free_allocations)
            if allocation.nbytes >= nbytes and allocation.address % alignment == 0
        ]
        if not compatible:
            return self._backend.allocate(nbytes, alignment=alignment)
        index, allocation = min(compatible, key=lambda candidate: candidate[1].nbytes)
        del self._free_allocations[index]
        return allocation

    def _release_allocation(self: Self, state: _AllocationState) -> None:
        if self._closed:
            return
        self._free_allocations.append(state.allocation)

    def tensor(self: Self, shape: tuple[int, ...], dtype: npt.DTypeLike, *, alignment: int = 1) -> Tensor:
        """Allocate a contiguous typed tensor."""
        if not shape or any(dimension <= 0 for dimension in shape):
            raise ValueError("tensor shape must contain only positive dimensions")
        nbytes = int(np.prod(shape, dtype=np.int64)) * np.dtype(dtype).itemsize
        return self.allocate(nbytes, alignment=alignment).tensor(shape, dtype)

    def queue(self: Self) -> Queue:
        """Create an in-order submission queue (a CUDA stream on the cuda backend)."""
        from qpu_xla.queue import Queue

        self._require_open()
        queue = Queue(self)
        self._queues.add(queue)
        return queue

    def close(self: Self) -> None:
        """Wait for submitted work, close queues and invalidate allocations."""
        if self._closed:
            return
        for queue in tuple(self._queues):
            queue.close()
        for state in self._allocations:
            state.closed = True
        self._free_allocations.clear()
        self._backend.close()
        self._closed = True

    def __enter__(self: Self) -> Self:
        self._require_open()
        return self

    def __exit__(self: Self, exc_type: object, exc_value: object, traceback: object) -> None:
        self.close()


__all__ = ["Device"]
