"""Whole-operator placement (the drop-in surface of src/qpu_xla/scheduler/placement.py).

``Placement`` keeps the reference's values and adds ``CUDA``. A
``CapabilityRegistry`` holds named ``ExecutionCandidate`` implementations and
``choose`` ranks the ones that support an operation by cost: the median of the
``CostModel``'s measured samples for that exact operation and candidate when
there are any, the candidate's own estimate otherwise (ties go to the
alphabetically first name). Under ``AUTO``, candidates that require calibration
are only eligible once the cost model holds samples for them.

``CostModel`` keeps its samples per (operation name, dtype, shape, layout,
candidate) and persists them with a device/software ``fingerprint`` in the
reference's JSON form (``{"fingerprint": {...}, "records": [...]}``), so a model
calibrated and saved by either side loads on the other.
"""

from __future__ import annotations

import json
from collections.abc import Callable, Iterable
from dataclasses import dataclass, field
from enum import Enum
from os import PathLike
from statistics import median
from typing import Any, Self


class Placement(Enum):
    """A requested or selected whole-operator execution strategy."""

    AUTO = "auto"
    CPU = "cpu"
    QPU = "qpu"
    HYBRID = "hybrid"
    CUDA = "cuda"


def _check(condition: bool, message: str) -> None:
    if not condition:
        raise ValueError(message)


@dataclass(frozen=True, slots=True)
class PartitionSpec:
    """A disjoint split of one operator's units (rows or output columns) between two executors."""

    axis: str
    qpu_units: int
    total_units: int
    alignment: int = 1

    def __post_init__(self: Self) -> None:
        _check(bool(self.axis) and min(self.total_units, self.alignment) > 0, "hybrid partitions require an axis and positive sizes")
        _check(0 < self.qpu_units < self.total_units, "hybrid partitions must assign non-empty work to both CPU and QPU")
        _check(self.qpu_units % self.alignment == 0, "QPU partition units must satisfy the kernel alignment")


@dataclass(frozen=True, slots=True)
class OperationSpec:
    """Normalized operator identity for capabilities and cost samples."""

    name: str
    dtype: str
    shape: tuple[int, ...]
    layout: str = ""


@dataclass(frozen=True, slots=True)
class ExecutionCandidate:
    """One implementation with a capability predicate and a fallback cost estimate."""

    name: str
    placement: Placement
    supported: Callable[[OperationSpec], bool]
    estimate_seconds: Callable[[OperationSpec], float]
    partition: PartitionSpec | None = None
    requires_calibration: bool = False

    def __post_init__(self: Self) -> None:
        _check(self.placement is not Placement.AUTO, "execution candidates must name a concrete placement")
        hybrid = self.placement is Placement.HYBRID
        _check(not hybrid or self.partition is not None, "hybrid execution candidates require a partition")
        _check(hybrid or self.partition is None, "only hybrid execution candidates may carry a partition")


@dataclass(frozen=True, slots=True)
class PlannedExecution:
    candidate: ExecutionCandidate
    estimated_seconds: float
    calibrated: bool


_SampleKey = tuple[str, str, tuple[int, ...], str, str]


@dataclass(slots=True)
class CostModel:
    """Measured seconds per exact operation and candidate; the median drives placement."""

    fingerprint: dict[str, str] = field(default_factory=dict)
    _samples: dict[_SampleKey, list[float]] = field(default_factory=dict)

    @staticmethod
    def _key(specification: OperationSpec, candidate: str) -> _SampleKey:
        return (specification.name, specification.dtype, tuple(specification.shape), specification.layout, candidate)

    def record(self: Self, specification: OperationSpec, candidate_name: str, seconds: float) -> None:
        _check(seconds > 0, "cost samples must be positive seconds")
        self._samples.setdefault(self._key(specification, candidate_name), []).append(float(seconds))

    def estimate(self: Self, specification: OperationSpec, candidate_name: str) -> float | None:
        values = self._samples.get(self._key(specification, candidate_name))
        return float(median(values)) if values else None

    def to_dict(self: Self) -> dict[str, object]:
        fields = ("name", "dtype", "shape", "layout", "candidate")
        records = []
        for key, values in self._samples.items():
            entry: dict[str, object] = dict(zip(fields, key, strict=True))
            entry["shape"] = list(key[2])
            entry["seconds"] = list(values)
            records.append(entry)
        return {"fingerprint": dict(self.fingerprint), "records": records}

    def save(self: Self, path: str | PathLike[str]) -> None:
        with open(path, "w", encoding="utf-8") as output:
            json.dump(self.to_dict(), output, indent=2, sort_keys=True)

    @classmethod
    def load(cls: type[Self], path: str | PathLike[str]) -> Self:
        with open(path, encoding="utf-8") as source:
            payload: Any = json.load(source)
        _check(isinstance(payload, dict), "cost model JSON must contain an object")
        fingerprint = payload.get("fingerprint")
        _check(
            isinstance(fingerprint, dict) and all(isinstance(k, str) and isinstance(v, str) for k, v in fingerprint.items()),
            "cost model fingerprint must map strings to strings",
        )
        records = payload.get("records")
        _check(isinstance(records, list), "cost model records must be a list")
        model = cls(dict(fingerprint))
        for entry in records:
            _check(isinstance(entry, dict), "cost model record must be an object")
            model._load_record(entry)
        return model

    def _load_record(self: Self, entry: dict[str, Any]) -> None:
        texts = [entry.get(name) for name in ("name", "dtype", "layout", "candidate")]
        shape, seconds = entry.get("shape"), entry.get("seconds")

        def positive_numbers(values: Any, kinds: tuple[type, ...]) -> bool:
            return isinstance(values, list) and all(isinstance(v, kinds) and not isinstance(v, bool) and v > 0 for v in values)

        _check(
            all(isinstance(text, str) for text in texts) and positive_numbers(shape, (int,)) and positive_numbers(seconds, (int, float)),
            "cost model record has invalid fields",
        )
        name, dtype, layout, candidate = texts
        specification = OperationSpec(name, dtype, tuple(shape), layout)  # type: ignore[arg-type]
        for value in seconds:  # type: ignore[union-attr]
            self.record(specification, candidate, float(value))  # type: ignore[arg-type]


class CapabilityRegistry:
    """Selects the cheapest supported whole-operator implementation."""

    def __init__(self: Self, candidates: Iterable[ExecutionCandidate] = ()) -> None:
        self._by_name: dict[str, ExecutionCandidate] = {}
        for candidate in candidates:
            self.register(candidate)

    def register(self: Self, candidate: ExecutionCandidate) -> None:
        _check(candidate.name not in self._by_name, f"candidate {candidate.name!r} is already registered")
        self._by_name[candidate.name] = candidate

    def _eligible(self: Self, specification: OperationSpec, preference: Placement, cost_model: CostModel | None) -> list[ExecutionCandidate]:
        def admitted(candidate: ExecutionCandidate) -> bool:
            if preference is not Placement.AUTO:
                return candidate.placement is preference
            # automatic placement never picks an uncalibrated candidate that needs calibration
            return not candidate.requires_calibration or (
                cost_model is not None and cost_model.estimate(specification, candidate.name) is not None
            )

        return [c for c in self._by_name.values() if c.supported(specification) and admitted(c)]

    def choose(
        self: Self, specification: OperationSpec, *, preference: Placement = Placement.AUTO, cost_model: CostModel | None = None
    ) -> PlannedExecution:
        eligible = self._eligible(specification, preference, cost_model)
        _check(bool(eligible), f"no {preference.value} implementation supports {specification.name!r}")
        plans = []
        for candidate in eligible:
            measured = None if cost_model is None else cost_model.estimate(specification, candidate.name)
            cost = measured if measured is not None else candidate.estimate_seconds(specification)
            _check(cost > 0, f"candidate {candidate.name!r} produced a non-positive cost estimate")
            plans.append(PlannedExecution(candidate, cost, measured is not None))
        return min(plans, key=lambda plan: (plan.estimated_seconds, plan.candidate.name))


__all__ = ["CapabilityRegistry", "CostModel", "ExecutionCandidate", "OperationSpec", "PartitionSpec", "Placement", "PlannedExecution"]
