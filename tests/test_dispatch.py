"""The TinyLlama ``_linear`` routing (src/qpu_xla/models/tinyllama/accelerated.py:228-266) with
the ``cuda`` placement: host logic on CPU with stand-in plans, and one real projection on the GPU."""

from __future__ import annotations

from types import SimpleNamespace

import numpy as np
import pytest

from qpu_xla.candidates import CandidateRecord, CandidateRegistry, CandidateStatus, CorrectnessEvidence, PerformanceEvidence
from qpu_xla.dispatch import LINEAR_DTYPE, LINEAR_LAYOUT, LINEAR_OPERATION, LinearDispatch
from qpu_xla.placement import Placement


def record(shape_class: str) -> CandidateRecord:
    return CandidateRecord(
        name=f"cuda.w8a8_linear.{shape_class}",
        operation=LINEAR_OPERATION,
        dtype=LINEAR_DTYPE,
        layout=LINEAR_LAYOUT,
        shape_class=shape_class,
        source_hash="0" * 64,
        status=CandidateStatus.SUPPORTED_WIN,
        correctness=CorrectnessEvidence("oracle.w8a8_linear", 1, True, 0.0, 0.0, 0.0, 0.0),
        performance=PerformanceEvidence("numpy int32", (1.0,), (0.01,)),
    )


class StandInPlan:
    def __init__(self) -> None:
        self.calls: list[tuple] = []

    def execute(self, destination, source, *, queue, wait_for=()):  # type: ignore[no-untyped-def]
        self.calls.append((destination, source, queue, tuple(wait_for)))
        return "event"


def tensor(*shape: int) -> SimpleNamespace:
    return SimpleNamespace(shape=shape)


def test_auto_needs_a_supported_candidate_for_the_exact_shape() -> None:
    plan = StandInPlan()
    queue = object()
    dispatch = LinearDispatch({"q_proj": plan}, queue, candidates=CandidateRegistry((record("128x2048x2048"),)))  # type: ignore[arg-type]
    assert dispatch("q_proj", tensor(128, 2048), tensor(128, 2048), "dep") == "event"  # type: ignore[arg-type]
    assert plan.calls[-1][2] is queue and plan.calls[-1][3] == ("dep",)
    with pytest.raises(ValueError, match="no measured supported-win"):
        dispatch("q_proj", tensor(64, 2048), tensor(64, 2048), None)  # type: ignore[arg-type]
    with pytest.raises(KeyError):
        dispatch("o_proj", tensor(128, 2048), tensor(128, 2048), None)  # type: ignore[arg-type]


def test_explicit_cuda_placement_runs_any_shape_and_cpu_is_refused() -> None:
    plan = StandInPlan()
    dispatch = LinearDispatch({"k_proj": plan}, object(), placement=Placement.CUDA)  # type: ignore[arg-type]
    dispatch("k_proj", tensor(7, 256), tensor(7, 2048))  # type: ignore[arg-type]
    assert len(plan.calls) == 1 and plan.calls[0][3] == ()
    for placement in (Placement.CPU, Placement.QPU, Placement.HYBRID):
        with pytest.raises(ValueError, match="no path in this build"):
            LinearDispatch({}, object(), placement=placement)  # type: ignore[arg-type]


@pytest.mark.gpu
def test_tinyllama_projection_through_the_dispatch(cuda_device) -> None:  # type: ignore[no-untyped-def]
    from oracle import qpu_oracle as oracle
    from qpu_xla.quantization import PreparedW8A8Linear, QuantizedMatrixInt8

    rng = np.random.default_rng(228)
    weight = rng.standard_normal((256, 2048), dtype=np.float32) * 0.02  # k_proj, GQA 4 x 64
    values, scales = oracle.quantize_per_output_channel_int8(weight)
    source = rng.standard_normal((128, 2048), dtype=np.float32)
    with cuda_device.queue() as queue, PreparedW8A8Linear(cuda_device, QuantizedMatrixInt8(values, scales), max_batch=128) as plan:
        dispatch = LinearDispatch({"k_proj": plan}, queue, candidates=CandidateRegistry((record("128x2048x256"),)))
        src = cuda_device.tensor((128, 2048), np.float32)
        src.write(source)
        dst = cuda_device.tensor((128, 256), np.float32)
        dispatch("k_proj", dst, src).wait()
        np.testing.assert_array_equal(dst.numpy(), oracle.w8a8_linear(source, values, scales))
