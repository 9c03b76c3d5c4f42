"""Per-projection routing of a model's W8A8 linears to the ``cuda`` placement.

Mirrors the TinyLlama runtime's ``_linear`` (src/qpu_xla/models/tinyllama/accelerated.py:228-266):
the shape class ``"{M}x{K}x{N}"`` of a call is looked up in the candidate registry under
operation ``linear`` and dtype ``w8a8-i32-fp32``, and a supported candidate (or an explicit
``Placement.CUDA``) runs the projection's prepared plan on the model's queue after the call's
dependency. Where the reference falls back to a host fp32 matmul (placement CPU, or AUTO without
a supported candidate), this build has no CPU path: ``Placement.CPU`` is rejected when the
dispatcher is made, and AUTO without a candidate raises the reference's error for an explicit
accelerator placement without one.
"""

from __future__ import annotations

from collections.abc import Mapping
from typing import Any, Self

from qpu_xla.candidates import CandidateRegistry
from qpu_xla.memory import Tensor
from qpu_xla.placement import Placement
from qpu_xla.queue import Event, Queue

LINEAR_OPERATION = "linear"
LINEAR_DTYPE = "w8a8-i32-fp32"
# Operand layout of this build's plans: int8 rows padded to 16 bytes of K (the reference's QPU
# plans use "row-major-packed-k4").
LINEAR_LAYOUT = "row-major-k16"


def linear_shape_class(source: Tensor, destination: Tensor) -> str:
    """``"{M}x{K}x{N}"`` as the reference names a linear call (accelerated.py:235)."""
    return f"{source.shape[0]}x{source.shape[1]}x{destination.shape[1]}"


class LinearDispatch:
    """``_linear(name, destination, source, dependency)`` over a set of prepared W8A8 plans."""

    def __init__(
        self: Self,
        plans: Mapping[str, Any],
        queue: Queue,
        *,
        placement: Placement = Placement.AUTO,
        candidates: CandidateRegistry | None = None,
    ) -> None:
        if placement not in (Placement.AUTO, Placement.CUDA):
            raise ValueError(f"placement {placement.value!r} has no path in this build (AUTO or CUDA only)")
        self.plans = dict(plans)
        self.queue = queue
        self.placement = placement
        self.candidates = candidates if candidates is not None else CandidateRegistry()

    def supported(self: Self, shape_class: str) -> bool:
        return bool(self.candidates.supported_for(operation=LINEAR_OPERATION, dtype=LINEAR_DTYPE, layout=LINEAR_LAYOUT, shape_class=shape_class))

    def __call__(self: Self, name: str, destination: Tensor, source: Tensor, dependency: Event | None = None) -> Event:
        if name not in self.plans:
            raise KeyError(f"no prepared W8A8 plan for projection {name!r}")
        if self.placement is Placement.AUTO and not self.supported(linear_shape_class(source, destination)):
            raise ValueError("no measured supported-win W8A8 CUDA candidate exists for this exact shape")
        wait_for = () if dependency is None else (dependency,)
        return self.plans[name].execute(destination, source, queue=self.queue, wait_for=wait_for)


__all__ = ["LINEAR_DTYPE", "LINEAR_LAYOUT", "LINEAR_OPERATION", "LinearDispatch", "linear_shape_class"]
