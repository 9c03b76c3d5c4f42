"""Whole-operator placement (src/qpu_xla/scheduler/placement.py:14-240) with the ``cuda`` placement.

``Placement`` keeps the reference's values and adds ``CUDA``. ``CapabilityRegistry.choose``
picks the cheapest supported candidate by a calibrated median (``CostModel``)
or the candidate's own estimate; ``CostModel`` persists calibration samples as
JSON (the reference's checkpoint/resume of calibration state, :122-171).
"""

from __future__ import annotations

import json
from collections.abc import Callable, Iterable
from dataclasses import dataclass, field
from enum import Enum
from os import PathLike
from statistics import median
from typing import Self


class Placement(Enum):
    """A requested or selected whole-operator execution strategy."""

    AUTO = "auto"
    CPU = "cpu"
    QPU = "qpu"
    HYBRID = "hybrid"
    CUDA = "cuda"


@dataclass(frozen=True, slots=True)
class PartitionSpec:
    """A disjoint split of one operator's units (rows or output columns) between two executors."""

    axis: str
    qpu_units: int
    total_units: int
    alignment: int = 1

    def __post_init__(self: Self) -> None:
        if not self.axis or self.total_units <= 0 or self.alignment <= 0:
            raise ValueError("hybrid partitions require an axis and positive sizes")
        if self.qpu_units <= 0 or self.qpu_units >= self.total_units:
            raise ValueError("hybrid partitions must assign non-empty work to both sides")
        if self.qpu_units % self.alignment:
            raise ValueError("partition units must satisfy the kernel alignment")


@dataclass(frozen=True, slots=True)
class OperationSpec:
    """Normalized operator identity for capabilities and cost samples."""

    name: str
    dtype: str
    shape: tuple[int, ...]
    layout: str = ""

    def key(self: Self) -> str:
        return f"{self.name}|{self.dtype}|{'x'.join(map(str, self.shape))}|{self.layout}"


@dataclass(frozen=True, slots=True)
class ExecutionCandidate:
    """One implementation with a capability check and a fallback cost estimate."""

    name: str
    placement: Placement
    supported: Callable[[OperationSpec], bool]
    estimate_seconds: Callable[[OperationSpec], float]
    partition: PartitionSpec | None = None
    requires_calibration: bool = False

    def __post_init__(self: Self) -> None:
        if self.placement is Placement.AUTO:
            raise ValueError("execution candidates must name a concrete placement")
        if self.placement is Placement.HYBRID and self.partition is None:
            raise ValueError("hybrid execution candidates require a partition")
        if self.placement is not Placement.HYBRID and self.partition is not None:
            raise ValueError("only hybrid execution candidates may carry a partition")


@dataclass(frozen=True, slots=True)
class PlannedExecution:
    candidate: ExecutionCandidate
    estimated_seconds: float
    calibrated: bool


@dataclass(slots=True)
class CostModel:
    """Measured seconds per (operation, candidate); medians drive placement."""

    samples: dict[str, dict[str, list[float]]] = field(default_factory=dict)

    def record(self: Self, specification: OperationSpec, candidate: str, seconds: float) -> None:
        if seconds <= 0:
            raise ValueError("cost samples must be positive")
        self.samples.setdefault(specification.key(), {}).setdefault(candidate, []).append(float(seconds))

    def estimate(self: Self, specification: OperationSpec, candidate: str) -> float | None:
        values = self.samples.get(specification.key(), {}).get(candidate)
        return float(median(values)) if values else None

    def save(self: Self, path: str | PathLike[str]) -> None:
        with open(path, "w", encoding="utf-8") as output:
            json.dump({"schema_version": 1, "samples": self.samples}, output, indent=2, sort_keys=True)

    @classmethod
    def load(cls: type[Self], path: str | PathLike[str]) -> Self:
        with open(path, encoding="utf-8") as source:
            payload = json.load(source)
        if not isinstance(payload, dict) or payload.get("schema_version") != 1 or not isinstance(payload.get("samples"), dict):
            raise ValueError("unsupported cost model schema")
        model = cls()
        for key, per_candidate in payload["samples"].items():
            for candidate, values in per_candidate.items():
                for value in values:
                    if float(value) <= 0:
                        raise ValueError("cost samples must be positive")
                model.samples.setdefault(key, {})[candidate] = [float(v) for v in values]
        return model


class CapabilityRegistry:
    """Select the cheapest supported whole-operator implementation."""

    def __init__(self: Self, candidates: Iterable[ExecutionCandidate] = ()) -> None:
        self._candidates: list[ExecutionCandidate] = []
        for candidate in candidates:
            self.register(candidate)

    def register(self: Self, candidate: ExecutionCandidate) -> None:
        if any(existing.name == candidate.name for existing in self._candidates):
            raise ValueError(f"candidate {candidate.name!r} is already registered")
        self._candidates.append(candidate)

    def choose(
        self: Self, specification: OperationSpec, *, preference: Placement = Placement.AUTO, cost_model: CostModel | None = None
    ) -> PlannedExecution:
        eligible = [
            candidate
            for candidate in self._candidates
            if candidate.supported(specification)
            and (preference is Placement.AUTO or candidate.placement is preference)
            and not (
                preference is Placement.AUTO
                and candidate.requires_calibration
                and (cost_model is None or cost_model.estimate(specification, candidate.name) is None)
            )
        ]
        if not eligible:
            raise ValueError(f"no {preference.value} implementation supports {specification.name!r}")
        scored: list[tuple[float, str, ExecutionCandidate, bool]] = []
        for candidate in eligible:
            measured = None if cost_model is None else cost_model.estimate(specification, candidate.name)
            estimate = candidate.estimate_seconds(specification) if measured is None else measured
            if estimate <= 0:
                raise ValueError(f"candidate {candidate.name!r} produced a non-positive cost estimate")
            scored.append((estimate, candidate.name, candidate, measured is not None))
        estimate, _, candidate, calibrated = min(scored, key=lambda score: (score[0], score[1]))
        return PlannedExecution(candidate, estimate, calibrated)


__all__ = ["CapabilityRegistry", "CostModel", "ExecutionCandidate", "OperationSpec", "PartitionSpec", "Placement", "PlannedExecution"]
