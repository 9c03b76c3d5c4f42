"""Candidate evidence records (src/qpu_xla/benchmark/candidates.py:13-295), with ``placement="cuda"``.

A record ties one kernel specialization (operation, dtype, layout, exact shape
class) to its numerical and timing evidence. ``CandidateRegistry.supported_for``
returns only "supported-win" records of one exact operation class; the JSON
archive (``save`` / ``load``, schema 3) persists every record, including slower
and quarantined ones.
"""

from __future__ import annotations

import json
from dataclasses import asdict, dataclass
from enum import Enum
from os import PathLike
from statistics import median
from typing import Any, Self

PLACEMENTS = frozenset({"cpu", "qpu", "hybrid", "cuda"})


class CandidateStatus(Enum):
    SUPPORTED_WIN = "supported-win"
    SAME_CONTRACT_WIN = "same-contract-win"
    EXPERIMENTAL_CORRECT_SLOWER = "experimental-correct-slower"
    QUARANTINED_INCORRECT = "quarantined-incorrect"
    REFERENCE_ONLY = "reference-only"


@dataclass(frozen=True, slots=True)
class CorrectnessEvidence:
    reference: str
    cases: int
    exact: bool
    max_abs_error: float
    mean_abs_error: float
    p99_abs_error: float
    max_relative_error: float
    saturation_count: int = 0
    nan_count: int = 0
    inf_count: int = 0

    def __post_init__(self: Self) -> None:
        if not self.reference or self.cases <= 0:
            raise ValueError("correctness evidence requires a reference and at least one case")
        errors = (self.max_abs_error, self.mean_abs_error, self.p99_abs_error, self.max_relative_error)
        counts = (self.saturation_count, self.nan_count, self.inf_count)
        if any(value < 0 for value in errors) or any(value < 0 for value in counts):
            raise ValueError("correctness errors and counts cannot be negative")


@dataclass(frozen=True, slots=True)
class PerformanceEvidence:
    cpu_reference: str
    cpu_seconds: tuple[float, ...]
    candidate_seconds: tuple[float, ...]
    fused_model_win: bool = False
    host_prep_seconds: tuple[float, ...] = ()
    kernel_seconds: tuple[float, ...] = ()
    cold_start_seconds: tuple[float, ...] = ()
    dequantization_seconds: tuple[float, ...] = ()
    same_contract_reference: str = ""
    same_contract_seconds: tuple[float, ...] = ()

    def __post_init__(self: Self) -> None:
        if not self.cpu_reference or not self.cpu_seconds or not self.candidate_seconds:
            raise ValueError("performance evidence requires both CPU and candidate samples")
        samples = (
            *self.cpu_seconds,
            *self.candidate_seconds,
            *self.host_prep_seconds,
            *self.kernel_seconds,
            *self.cold_start_seconds,
            *self.dequantization_seconds,
            *self.same_contract_seconds,
        )
        if any(value <= 0 for value in samples):
            raise ValueError("performance samples must be positive")
        if bool(self.same_contract_reference) != bool(self.same_contract_seconds):
            raise ValueError("same-contract performance requires both a reference and samples")

    @property
    def cpu_median_seconds(self: Self) -> float:
        return float(median(self.cpu_seconds))

    @property
    def candidate_median_seconds(self: Self) -> float:
        return float(median(self.candidate_seconds))

    @property
    def speedup(self: Self) -> float:
        return self.cpu_median_seconds / self.candidate_median_seconds

    @property
    def measured_win(self: Self) -> bool:
        """The reference's five-percent gate (candidates.py:97-100)."""
        return self.speedup >= 1.05 or self.fused_model_win

    @property
    def same_contract_speedup(self: Self) -> float | None:
        if not self.same_contract_seconds:
            return None
        return float(median(self.same_contract_seconds)) / self.candidate_median_seconds

    @property
    def same_contract_win(self: Self) -> bool:
        speedup = self.same_contract_speedup
        return speedup is not None and speedup >= 1.05


@dataclass(frozen=True, slots=True)
class PartitionEvidence:
    """A measured split: ``qpu_units`` is the accelerator's share (the CUDA shard on this build)."""

    axis: str
    qpu_units: int
    total_units: int
    alignment: int = 1

    def __post_init__(self: Self) -> None:
        if not self.axis or self.total_units <= 0 or self.alignment <= 0:
            raise ValueError("partition evidence requires an axis and positive sizes")
        if self.qpu_units <= 0 or self.qpu_units >= self.total_units:
            raise ValueError("partition evidence must retain work on both sides")
        if self.qpu_units % self.alignment:
            raise ValueError("partition evidence does not satisfy its alignment")


@dataclass(frozen=True, slots=True)
class CandidateRecord:
    name: str
    operation: str
    dtype: str
    layout: str
    shape_class: str
    source_hash: str
    status: CandidateStatus
    correctness: CorrectnessEvidence | None = None
    performance: PerformanceEvidence | None = None
    reason: str = ""
    placement: str = "cuda"
    kernels: tuple[str, ...] = ()
    partition: PartitionEvidence | None = None

    def __post_init__(self: Self) -> None:
        identity = (self.name, self.operation, self.dtype, self.layout, self.shape_class, self.source_hash)
        if any(not value for value in identity):
            raise ValueError("candidate identity fields must be non-empty")
        if self.placement not in PLACEMENTS:
            raise ValueError("candidate placement must be cpu, qpu, hybrid or cuda")
        if self.placement == "hybrid" and self.partition is None:
            raise ValueError("hybrid candidate records require partition evidence")
        if self.placement != "hybrid" and self.partition is not None:
            raise ValueError("only hybrid candidate records may include partition evidence")
        if self.status is CandidateStatus.SUPPORTED_WIN:
            if self.correctness is None or self.performance is None or not self.performance.measured_win:
                raise ValueError("supported candidates require correctness and a measured or fused win")
            if self.correctness.nan_count or self.correctness.inf_count:
                raise ValueError("supported candidates cannot produce NaN or Inf outputs")
        if self.status is CandidateStatus.SAME_CONTRACT_WIN:
            if self.correctness is None or self.performance is None or not self.performance.same_contract_win:
                raise ValueError("same-contract winners require correctness and a measured CPU win")
        if self.status is CandidateStatus.EXPERIMENTAL_CORRECT_SLOWER and self.correctness is None:
            raise ValueError("correct experimental candidates require correctness evidence")
        if self.status is CandidateStatus.QUARANTINED_INCORRECT and not self.reason:
            raise ValueError("quarantined candidates require a failure reason")


class CandidateRegistry:
    """Serializable archive that exposes only measured winners to placement."""

    def __init__(self: Self, records: tuple[CandidateRecord, ...] = ()) -> None:
        self._records: dict[str, CandidateRecord] = {}
        for record in records:
            self.register(record)

    @property
    def records(self: Self) -> tuple[CandidateRecord, ...]:
        return tuple(self._records.values())

    @property
    def supported(self: Self) -> tuple[CandidateRecord, ...]:
        return tuple(r for r in self._records.values() if r.status is CandidateStatus.SUPPORTED_WIN)

    def supported_for(self: Self, *, operation: str, dtype: str, layout: str, shape_class: str) -> tuple[CandidateRecord, ...]:
        return tuple(
            r
            for r in self.supported
            if r.operation == operation and r.dtype == dtype and r.layout == layout and r.shape_class == shape_class
        )

    def register(self: Self, record: CandidateRecord) -> None:
        if record.name in self._records:
            raise ValueError(f"candidate {record.name!r} is already registered")
        self._records[record.name] = record

    @classmethod
    def combine(cls: type[Self], *registries: CandidateRegistry) -> Self:
        return cls(tuple(record for registry in registries for record in registry.records))

    def to_dict(self: Self) -> dict[str, object]:
        payload: list[dict[str, object]] = []
        for record in self.records:
            item = asdict(record)
            item["status"] = record.status.value
            payload.append(item)
        return {"schema_version": 3, "records": payload}

    def save(self: Self, path: str | PathLike[str]) -> None:
        with open(path, "w", encoding="utf-8") as output:
            json.dump(self.to_dict(), output, indent=2, sort_keys=True)

    @classmethod
    def load(cls: type[Self], path: str | PathLike[str]) -> Self:
        with open(path, encoding="utf-8") as source:
            payload: Any = json.load(source)
        if not isinstance(payload, dict) or payload.get("schema_version") not in (1, 2, 3):
            raise ValueError("unsupported candidate registry schema")
        raw_records = payload.get("records")
        if not isinstance(raw_records, list):
            raise ValueError("candidate registry records must be a list")
        records: list[CandidateRecord] = []
        for raw in raw_records:
            if not isinstance(raw, dict):
                raise ValueError("candidate registry records must be objects")
            item = dict(raw)
            item.pop("quality", None)
            item["status"] = CandidateStatus(item["status"])
            if item.get("correctness") is not None:
                item["correctness"] = CorrectnessEvidence(**item["correctness"])
            if item.get("performance") is not None:
                perf = dict(item["performance"])
                for key, value in perf.items():
                    if isinstance(value, list):
                        perf[key] = tuple(value)
                item["performance"] = PerformanceEvidence(**perf)
            if item.get("partition") is not None:
                item["partition"] = PartitionEvidence(**item["partition"])
            item["kernels"] = tuple(item.get("kernels", ()))
            records.append(CandidateRecord(**item))
        return cls(tuple(records))


__all__ = [
    "CandidateRecord",
    "CandidateRegistry",
    "CandidateStatus",
    "CorrectnessEvidence",
    "PartitionEvidence",
    "PerformanceEvidence",
]
