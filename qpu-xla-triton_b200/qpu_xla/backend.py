"""Backends behind a :class:`~qpu_xla.device.Device`.

Mirrors the narrow protocol of src/qpu_xla/backend.py:32-39 (``allocate`` and
``close``). Two backends exist:

* :class:`CudaBackend` -- allocations are CUDA device memory on one GPU (through
  PyTorch's caching allocator) and kernels are launched through libqpucuda's
  context. This replaces ``PyVideoCore7Backend`` (backend.py:83-134).
* :class:`FakeBackend` -- NumPy memory with deterministic fake addresses, for
  CPU-only tests of the runtime's queue, event and memory semantics
  (backend.py:50-80). It runs no kernels.

Unlike the reference, a CUDA allocation is not host-mapped and its address is
a 64-bit device pointer; ``Tensor.numpy()`` is therefore an explicit copy on
the CUDA backend (see :mod:`qpu_xla.memory`).
"""

from __future__ import annotations

import threading
from dataclasses import dataclass
from typing import Any, Protocol, Self

import numpy as np

from qpu_xla.errors import AllocationError, DeviceClosedError


@dataclass(frozen=True, slots=True)
class BackendAllocation:
    """One contiguous allocation: a 1-D uint8 storage object and its base address."""

    storage: Any  # numpy.ndarray (fake) or torch.Tensor (cuda), 1-D uint8
    address: int
    host_mapped: bool

    @property
    def nbytes(self: Self) -> int:
        return int(self.storage.numel() if hasattr(self.storage, "numel") else self.storage.nbytes)


class Backend(Protocol):
    """Protocol isolating the runtime from the device implementation."""

    kind: str

    def allocate(self: Self, nbytes: int, *, alignment: int) -> BackendAllocation:
        """Allocate ``nbytes`` aligned to ``alignment`` bytes."""

    def close(self: Self) -> None:
        """Release all backend resources."""


def _validate_allocation_request(nbytes: int, alignment: int) -> None:
    if nbytes <= 0:
        raise AllocationError("allocation size must be positive")
    if alignment <= 0 or alignment & (alignment - 1):
        raise AllocationError("alignment must be a positive power of two")


class FakeBackend:
    """CPU-only backend with deterministic fake addresses; it cannot run kernels."""

    kind = "fake"

    def __init__(self: Self, *, address_base: int = 0x1000) -> None:
        if address_base < 0:
            raise AllocationError("address_base must be non-negative")
        self._address = address_base
        self._closed = False
        self._allocations: list[np.ndarray] = []

    def allocate(self: Self, nbytes: int, *, alignment: int) -> BackendAllocation:
        _validate_allocation_request(nbytes, alignment)
        if self._closed:
            raise DeviceClosedError("backend is closed")
        address = (self._address + alignment - 1) & -alignment
        storage = np.empty(nbytes + alignment - 1, dtype=np.uint8)
        offset = (-int(storage.ctypes.data)) % alignment
        array = storage[offset : offset + nbytes]
        self._allocations.append(storage)
        self._address = address + nbytes
        return BackendAllocation(array, address, True)

    def close(self: Self) -> None:
        self._closed = True
        self._allocations.clear()


class CudaBackend:
    """CUDA device memory plus a libqpucuda context on one GPU."""

    kind = "cuda"

    def __init__(
        self: Self,
        device_ordinal: int | None = None,
        *,
        timeout_ns: int = 0,
        failure_mask: int = 0,
    ) -> None:
        import torch

        from qpu_xla import _native

        if not torch.cuda.is_available():
            raise DeviceClosedError("CUDA is not available: the cuda backend needs a GPU")
        self._torch = torch
        self.device_ordinal = torch.cuda.current_device() if device_ordinal is None else int(device_ordinal)
        self.torch_device = torch.device("cuda", self.device_ordinal)
        with torch.cuda.device(self.device_ordinal):
            self.native = _native.NativeContext(
                self.device_ordinal, timeout_ns=timeout_ns, failure_mask=failure_mask, stream=None
            )
        self.launch_lock = threading.RLock()
        self._closed = False

    def allocate(self: Self, nbytes: int, *, alignment: int) -> BackendAllocation:
        _validate_allocation_request(nbytes, alignment)
        if self._closed:
            raise DeviceClosedError("backend is closed")
        torch = self._torch
        alignment = max(alignment, 256)
        raw = torch.empty(nbytes + alignment, dtype=torch.uint8, device=self.torch_device)
        offset = (-int(raw.data_ptr())) % alignment
        storage = raw[offset : offset + nbytes]
        return BackendAllocation(storage, int(storage.data_ptr()), False)

    def launch(self: Self, stream: Any, fn: Any) -> Any:
        """Run ``fn(native_context)`` with the context retargeted at ``stream`` (a torch CUDA stream)."""
        if self._closed:
            raise DeviceClosedError("backend is closed")
        with self.launch_lock:
            self.native.set_stream(int(stream.cuda_stream))
            return fn(self.native)

    def close(self: Self) -> None:
        if not self._closed:
            self._torch.cuda.synchronize(self.torch_device)
            self.native.close()
            self._closed = True


__all__ = ["Backend", "BackendAllocation", "CudaBackend", "FakeBackend"]
