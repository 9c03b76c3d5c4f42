"""Kernel handles and launch grids (the drop-in surface of src/qpu_xla/kernel.py).

An executor comes in one of two forms:

* ``executor(backend, args, grid)`` -- the reference's form. On the CUDA backend it runs
  with the submitting queue's stream made torch's current stream, so anything it
  launches through torch, or through ``backend.launch(torch.cuda.current_stream(), ...)``,
  is ordered on that queue;
* ``executor(backend, args, grid, stream)`` -- this build's kernel handles, which take the
  queue's torch CUDA stream explicitly (None on the fake backend).

The form is read once from the executor's signature when the handle is made.
"""

from __future__ import annotations

import contextlib
import inspect
from collections.abc import Callable
from dataclasses import dataclass, field
from typing import Any, Self

from qpu_xla.errors import KernelError

KernelCallable = Callable[..., None]


@dataclass(frozen=True, slots=True)
class LaunchConfig:
    """A three-dimensional launch grid (kept for the interface; the CUDA kernels size their own grids)."""

    grid: tuple[int, int, int] = (1, 1, 1)

    def __post_init__(self: Self) -> None:
        dims = tuple(self.grid)
        if len(dims) != 3 or min(int(d) for d in dims) <= 0:
            raise KernelError("kernel grid must contain three positive dimensions")


def _takes_stream(executor: KernelCallable) -> bool:
    """Whether ``executor`` accepts a fourth positional argument (the stream)."""
    try:
        parameters = inspect.signature(executor).parameters.values()
    except (TypeError, ValueError):  # builtins without a signature: the reference's form
        return False
    positional = 0
    for parameter in parameters:
        if parameter.kind is inspect.Parameter.VAR_POSITIONAL:
            return True
        if parameter.kind in (inspect.Parameter.POSITIONAL_ONLY, inspect.Parameter.POSITIONAL_OR_KEYWORD):
            positional += 1
    return positional >= 4


@dataclass(frozen=True, slots=True)
class Kernel:
    """A named kernel with its execution adapter."""

    name: str
    executor: KernelCallable
    _with_stream: bool = field(init=False, repr=False, compare=False)

    def __post_init__(self: Self) -> None:
        object.__setattr__(self, "_with_stream", _takes_stream(self.executor))

    def execute(self: Self, backend: Any, args: tuple[Any, ...], launch: LaunchConfig, stream: Any = None) -> None:
        """Run the executor; a failure other than :class:`KernelError` is raised as one."""
        try:
            if self._with_stream:
                self.executor(backend, args, launch.grid, stream)
                return
            with _current_stream(stream):
                self.executor(backend, args, launch.grid)
        except KernelError:
            raise
        except BaseException as exc:
            raise KernelError(f"kernel {self.name!r} failed") from exc


def _current_stream(stream: Any) -> Any:
    if stream is None:
        return contextlib.nullcontext()
    import torch

    return torch.cuda.stream(stream)


__all__ = ["Kernel", "KernelCallable", "LaunchConfig"]
