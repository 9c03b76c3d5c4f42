"""Candidate evidence records (the drop-in surface of src/qpu_xla/benchmark/candidates.py).

A record ties one kernel specialization (operation, dtype, layout, exact shape
class) to the evidence behind its status; ``placement`` may also be ``"cuda"``.
Only ``supported-win`` records reach placement (``CandidateRegistry.supported_for``);
the JSON archive keeps every record, slower and quarantined ones included.

The record and evidence classes are frozen dataclasses whose field names are the
archive's JSON keys. Their checks are written as (condition, message) rules, and the
archive is read and written generically from the dataclass fields: nested evidence
objects become JSON objects and tuples become lists, and back.
"""

from __future__ import annotations

import dataclasses
import json
import typing
from dataclasses import dataclass
from enum import Enum
from os import PathLike
from statistics import median
from typing import Any, Self

PLACEMENTS = frozenset({"cpu", "qpu", "hybrid", "cuda"})
WIN_THRESHOLD = 1.05  # a measured win is at least 5 % faster than the comparison


class CandidateStatus(Enum):
    SUPPORTED_WIN = "supported-win"
    SAME_CONTRACT_WIN = "same-contract-win"
    EXPERIMENTAL_CORRECT_SLOWER = "experimental-correct-slower"
    QUARANTINED_INCORRECT = "quarantined-incorrect"
    REFERENCE_ONLY = "reference-only"


def _enforce(rules: tuple[tuple[bool, str], ...]) -> None:
    """Raise ValueError with the message of the first rule that does not hold."""
    for holds, message in rules:
        if not holds:
            raise ValueError(message)


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
        magnitudes = (self.max_abs_error, self.mean_abs_error, self.p99_abs_error, self.max_relative_error,
                      self.saturation_count, self.nan_count, self.inf_count)
        _enforce((
            (bool(self.reference) and self.cases > 0, "correctness evidence requires a reference and at least one case"),
            (min(magnitudes) >= 0, "correctness errors and counts cannot be negative"),
        ))

    @property
    def finite(self: Self) -> bool:
        return self.nan_count == 0 and self.inf_count == 0


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
        samples = [value for item in dataclasses.fields(self) if item.name.endswith("_seconds") for value in getattr(self, item.name)]
        _enforce((
            (bool(self.cpu_reference and self.cpu_seconds and self.candidate_seconds),
             "performance evidence requires both CPU and candidate samples"),
            (all(value > 0 for value in samples), "performance samples must be positive"),
            (bool(self.same_contract_reference) == bool(self.same_contract_seconds),
             "same-contract performance requires both a reference and samples"),
        ))

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
        return self.fused_model_win or self.speedup >= WIN_THRESHOLD

    @property
    def same_contract_speedup(self: Self) -> float | None:
        if not self.same_contract_seconds:
            return None
        return float(median(self.same_contract_seconds)) / self.candidate_median_seconds

    @property
    def same_contract_win(self: Self) -> bool:
        ratio = self.same_contract_speedup
        return ratio is not None and ratio >= WIN_THRESHOLD


@dataclass(frozen=True, slots=True)
class PartitionEvidence:
    """A measured split: ``qpu_units`` is the accelerator's share (the CUDA shard on this build)."""

    axis: str
    qpu_units: int
    total_units: int
    alignment: int = 1

    def __post_init__(self: Self) -> None:
        _enforce((
            (bool(self.axis) and min(self.total_units, self.alignment) > 0, "partition evidence requires an axis and positive sizes"),
            (0 < self.qpu_units < self.total_units, "partition evidence must retain work on both CPU and QPU"),
            (self.qpu_units % self.alignment == 0, "partition evidence does not satisfy its alignment"),
        ))


@dataclass(frozen=True, slots=True)
class QualityEvidence:
    """Error of a quantized format against its fp32 source-domain reference."""

    reference: str
    normalized_rmse: float
    cosine_similarity: float
    max_abs_error: float = 0.0
    mean_abs_error: float = 0.0
    p99_abs_error: float = 0.0
    nan_count: int = 0
    inf_count: int = 0
    top1_agreement: float | None = None

    def __post_init__(self: Self) -> None:
        errors = (self.normalized_rmse, self.max_abs_error, self.mean_abs_error, self.p99_abs_error)
        _enforce((
            (bool(self.reference) and min(errors) >= 0, "quality evidence requires a reference and non-negative NRMSE"),
            (-1.0 <= self.cosine_similarity <= 1.0, "quality cosine similarity must be within [-1, 1]"),
            (min(self.nan_count, self.inf_count) >= 0, "quality NaN and Inf counts cannot be negative"),
            (self.top1_agreement is None or 0.0 <= self.top1_agreement <= 1.0, "quality top-1 agreement must be within [0, 1]"),
        ))

    @property
    def passes_default_gate(self: Self) -> bool:
        """NRMSE at most 0.10, cosine similarity at least 0.99, and no NaN or Inf."""
        return self.normalized_rmse <= 0.10 and self.cosine_similarity >= 0.99 and self.nan_count == 0 and self.inf_count == 0


def _status_rules(record: CandidateRecord) -> tuple[tuple[bool, str], ...]:
    """The evidence each lifecycle state needs."""
    correct, timed = record.correctness, record.performance
    status = record.status
    if status is CandidateStatus.SUPPORTED_WIN:
        return (
            (correct is not None and timed is not None and timed.measured_win,
             "supported candidates require correctness and a measured or fused win"),
            (correct is None or correct.finite, "supported candidates cannot produce NaN or Inf outputs"),
        )
    if status is CandidateStatus.SAME_CONTRACT_WIN:
        return (
            (correct is not None and timed is not None and timed.same_contract_win,
             "same-contract winners require correctness and a measured W8A8 CPU win"),
            (correct is None or correct.finite, "same-contract winners cannot produce NaN or Inf outputs"),
        )
    if status is CandidateStatus.EXPERIMENTAL_CORRECT_SLOWER:
        return ((correct is not None, "correct experimental candidates require correctness evidence"),)
    if status is CandidateStatus.QUARANTINED_INCORRECT:
        return ((bool(record.reason), "quarantined candidates require a failure reason"),)
    return ()


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
    quality: QualityEvidence | None = None

    def __post_init__(self: Self) -> None:
        identity = (self.name, self.operation, self.dtype, self.layout, self.shape_class, self.source_hash)
        hybrid = self.placement == "hybrid"
        _enforce((
            (all(identity), "candidate identity fields must be non-empty"),
            (self.placement in PLACEMENTS, "candidate placement must be cpu, qpu, hybrid or cuda"),
            (not hybrid or self.partition is not None, "hybrid candidate records require partition evidence"),
            (hybrid or self.partition is None, "only hybrid candidate records may include partition evidence"),
        ))
        _enforce(_status_rules(self))

    def shape_key(self: Self) -> tuple[str, str, str, str]:
        """The exact operation class placement looks records up by."""
        return (self.operation, self.dtype, self.layout, self.shape_class)


# ---- archive (de)serialization, driven by the dataclass fields ---------------------------------


def _to_json(value: Any) -> Any:
    if isinstance(value, Enum):
        return value.value
    if dataclasses.is_dataclass(value):
        return {item.name: _to_json(getattr(value, item.name)) for item in dataclasses.fields(value)}
    if isinstance(value, tuple):
        return [_to_json(item) for item in value]
    return value


_NESTED: dict[str, type] = {}  # field name -> evidence class, filled below


def _from_json(cls: type, payload: dict[str, Any]) -> Any:
    """Build ``cls`` from a JSON object: nested evidence objects and enums are rebuilt, lists
    become tuples; unknown keys are an error (TypeError from the constructor)."""
    hints = typing.get_type_hints(cls)
    arguments: dict[str, Any] = {}
    for key, raw in payload.items():
        if key in _NESTED and raw is not None:
            arguments[key] = _from_json(_NESTED[key], raw)
        elif hints.get(key) is CandidateStatus:
            arguments[key] = CandidateStatus(raw)
        elif isinstance(raw, list):
            arguments[key] = tuple(raw)
        else:
            arguments[key] = raw
    return cls(**arguments)


_NESTED.update(correctness=CorrectnessEvidence, performance=PerformanceEvidence, partition=PartitionEvidence,
               quality=QualityEvidence)


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
        return tuple(record for record in self._records.values() if record.status is CandidateStatus.SUPPORTED_WIN)

    def supported_for(self: Self, *, operation: str, dtype: str, layout: str, shape_class: str) -> tuple[CandidateRecord, ...]:
        wanted = (operation, dtype, layout, shape_class)
        return tuple(record for record in self.supported if record.shape_key() == wanted)

    def register(self: Self, record: CandidateRecord) -> None:
        if record.name in self._records:
            raise ValueError(f"candidate {record.name!r} is already registered")
        self._records[record.name] = record

    @classmethod
    def combine(cls: type[Self], *registries: CandidateRegistry) -> Self:
        return cls(tuple(record for registry in registries for record in registry.records))

    def to_dict(self: Self) -> dict[str, object]:
        return {"schema_version": 3, "records": [_to_json(record) for record in self.records]}

    def save(self: Self, path: str | PathLike[str]) -> None:
        with open(path, "w", encoding="utf-8") as output:
            json.dump(self.to_dict(), output, indent=2, sort_keys=True)

    @classmethod
    def load(cls: type[Self], path: str | PathLike[str]) -> Self:
        with open(path, encoding="utf-8") as source:
            payload: Any = json.load(source)
        if not isinstance(payload, dict) or payload.get("schema_version") not in (1, 2, 3):
            raise ValueError("unsupported candidate registry schema")
        entries = payload.get("records")
        if not isinstance(entries, list):
            raise ValueError("candidate registry records must be a list")
        records = []
        for entry in entries:
            if not isinstance(entry, dict):
                raise ValueError("candidate registry records must be objects")
            try:
                records.append(_from_json(CandidateRecord, entry))
            except (KeyError, TypeError, ValueError) as error:
                raise ValueError("candidate registry contains an invalid record") from error
        return cls(tuple(records))


__all__ = [
    "CandidateRecord",
    "CandidateRegistry",
    "CandidateStatus",
    "CorrectnessEvidence",
    "PartitionEvidence",
    "PerformanceEvidence",
    "QualityEvidence",
]
