"""Kernel handles and launch configuration (src/qpu_xla/kernel.py:12-38)."""

from __future__ import annotations

from collections.abc import Callable
from dataclasses import dataclass
from typing import Any, Self

from qpu_xla.errors import KernelError

# executor(backend, args, grid, stream) -> None. ``stream`` is the torch CUDA
# stream of the submitting queue (None on the fake backend).
KernelCallable = Callable[[Any, tuple[Any, ...], tuple[int, int, int], Any], None]


@dataclass(frozen=True, slots=True)
class LaunchConfig:
    """A three-dimensional launch grid (kept for interface parity; CUDA kernels size their own grids)."""

    grid: tuple[int, int, int] = (1, 1, 1)

    def __post_init__(self: Self) -> None:
        if len(self.grid) != 3 or any(int(dimension) <= 0 for dimension in self.grid):
            raise KernelError("kernel grid must contain three positive dimensions")


@dataclass(frozen=True, slots=True)
class Kernel:
    """A named kernel with its execution adapter."""

    name: str
    executor: KernelCallable

    def execute(self: Self, backend: Any, args: tuple[Any, ...], launch: LaunchConfig, stream: Any = None) -> None:
        """Run the executor; failures other than :class:`KernelError` are wrapped in one."""
        try:
            self.executor(backend, args, launch.grid, stream)
        except KernelError:
            raise
        except BaseException as exc:
            raise KernelError(f"kernel {self.name!r} failed") from exc


__all__ = ["Kernel", "KernelCallable", "LaunchConfig"]
