"""Device lifetime and allocation (the drop-in surface of src/qpu_xla/device.py).

``Device.open()`` opens the CUDA backend on one GPU (the reference opened the
VideoCore DRM driver); ``Device.fake()`` keeps the CPU-only test backend.

Allocations come from a per-device :class:`_Pool`. A buffer that is closed
returns its allocation to the pool, where the next request reuses the smallest
released allocation that is large enough and suitably aligned (so a closed
buffer's address comes back for a request it fits); requests nothing fits go to
the backend. Closing the device retires every block still lent out, which makes
all buffers and tensor views over them raise ``BufferClosedError``.
"""

from __future__ import annotations

import bisect
import itertools
from typing import TYPE_CHECKING, Any, Self
from weakref import WeakSet

import numpy as np
import numpy.typing as npt

from qpu_xla.backend import Backend, BackendAllocation, CudaBackend, FakeBackend, _validate_allocation_request
from qpu_xla.errors import DeviceClosedError
from qpu_xla.memory import Buffer, Tensor, _Block

if TYPE_CHECKING:
    from qpu_xla.queue import Queue


class _Pool:
    """Released allocations ordered by size, plus every block currently lent out."""

    def __init__(self: Self, backend: Backend) -> None:
        self._backend = backend
        self._free: list[tuple[int, int, BackendAllocation]] = []  # (nbytes, arrival, allocation), sorted
        self._arrivals = itertools.count()
        self._lent: list[_Block] = []

    def lend(self: Self, nbytes: int, alignment: int) -> _Block:
        allocation = self._reuse(nbytes, alignment) or self._backend.allocate(nbytes, alignment=alignment)
        block = _Block(allocation, self._give_back)
        self._lent.append(block)
        return block

    def _reuse(self: Self, nbytes: int, alignment: int) -> BackendAllocation | None:
        first = bisect.bisect_left(self._free, (nbytes, -1))
        for position in range(first, len(self._free)):
            allocation = self._free[position][2]
            if allocation.address % alignment == 0:
                del self._free[position]
                return allocation
        return None

    def _give_back(self: Self, allocation: BackendAllocation) -> None:
        if self._backend is None:  # the device is closed: nothing is reused any more
            return
        bisect.insort(self._free, (allocation.nbytes, next(self._arrivals), allocation))
        self._lent = [block for block in self._lent if block.live]

    def retire_all(self: Self) -> None:
        for block in self._lent:
            block.retire(recycle=False)
        self._lent.clear()
        self._free.clear()
        self._backend = None  # type: ignore[assignment]


class Device:
    """An owned device context over one backend."""

    def __init__(self: Self, backend: Backend) -> None:
        self._backend = backend
        self._pool = _Pool(backend)
        self._closed = False
        self._queues: WeakSet[Queue] = WeakSet()

    @classmethod
    def fake(cls: type[Device]) -> Device:
        """CPU-only device for runtime tests; it cannot launch CUDA kernels."""
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
        """A byte buffer owned by this device (a released allocation is reused when one fits)."""
        self._require_open()
        _validate_allocation_request(nbytes, alignment)
        return Buffer(self, self._pool.lend(nbytes, alignment), nbytes=nbytes)

    def tensor(self: Self, shape: tuple[int, ...], dtype: npt.DTypeLike, *, alignment: int = 1) -> Tensor:
        """A contiguous typed tensor in a buffer of its own."""
        if not shape or min(shape) <= 0:
            raise ValueError("tensor shape must contain only positive dimensions")
        nbytes = int(np.prod(shape, dtype=np.int64)) * np.dtype(dtype).itemsize
        return self.allocate(nbytes, alignment=alignment).tensor(shape, dtype)

    def queue(self: Self) -> Queue:
        """A new in-order submission queue (a CUDA stream on the cuda backend)."""
        from qpu_xla.queue import Queue

        self._require_open()
        queue = Queue(self)
        self._queues.add(queue)
        return queue

    def close(self: Self) -> None:
        """Finish and close every queue, invalidate every allocation, release the backend."""
        if self._closed:
            return
        for queue in list(self._queues):
            queue.close()
        self._pool.retire_all()
        self._backend.close()
        self._closed = True

    def __enter__(self: Self) -> Self:
        self._require_open()
        return self

    def __exit__(self: Self, exc_type: object, exc_value: object, traceback: object) -> None:
        self.close()


__all__ = ["Device"]
