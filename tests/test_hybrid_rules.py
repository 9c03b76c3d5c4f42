"""``PreparedW8A8Linear``'s hybrid-split entry points (src/qpu_xla/models/tinyllama/
quantization.py:350-391, 516-557, 664-750) on CPU: the argument rules against the plan's host-side
state, with the GPU submissions replaced by recorders. The GPU run of ``execute_hybrid`` is in
test_gpu_runtime.py; the other three reach the same ``execute`` / ``execute_prepared`` calls."""

from __future__ import annotations

from types import SimpleNamespace

import pytest

from qpu_xla.errors import DependencyError
from qpu_xla.quantization import PreparedW8A8Linear


def _plan(device: object) -> tuple[PreparedW8A8Linear, list[tuple[str, object]]]:
    plan = object.__new__(PreparedW8A8Linear)
    plan._closed = False
    plan._last_event = None
    plan._queue = None
    plan._cpu_queue = None
    plan.device = device
    plan.output_count = 512
    plan.max_batch = 64
    submitted: list[tuple[str, object]] = []

    def execute(destination: object, source: object, *, queue: object, wait_for: object = ()) -> str:
        submitted.append(("execute", queue))
        return "event"

    def execute_prepared(destination: object, *, batch: int, queue: object, wait_for: object = ()) -> str:
        submitted.append(("execute_prepared", queue))
        return "event"

    plan.execute = execute  # type: ignore[method-assign]
    plan.execute_prepared = execute_prepared  # type: ignore[method-assign]
    return plan, submitted


def test_hybrid_queue_rules() -> None:
    device = object()
    plan, submitted = _plan(device)
    gpu, cpu, other = (SimpleNamespace(device=device) for _ in range(3))
    foreign = SimpleNamespace(device=object())
    with pytest.raises(DependencyError, match="distinct"):
        plan.execute_hybrid(None, None, qpu_queue=gpu, cpu_queue=gpu, qpu_outputs=256)
    with pytest.raises(DependencyError, match="plan device"):
        plan.execute_hybrid(None, None, qpu_queue=gpu, cpu_queue=foreign, qpu_outputs=256)
    assert submitted == []
    # both parts go to the GPU queue; the CPU queue is bound but receives no work
    assert plan.execute_hybrid(None, None, qpu_queue=gpu, cpu_queue=cpu, qpu_outputs=256) == "event"
    assert submitted == [("execute", gpu)]
    with pytest.raises(DependencyError, match="first CPU queue"):
        plan.execute_hybrid(None, None, qpu_queue=gpu, cpu_queue=other, qpu_outputs=256)
    with pytest.raises(DependencyError, match="first QPU queue"):
        plan.execute_hybrid(None, None, qpu_queue=other, cpu_queue=cpu, qpu_outputs=256)
    plan._last_event = SimpleNamespace(done=False)
    with pytest.raises(RuntimeError, match="in-flight"):
        plan.execute_hybrid_rows(None, SimpleNamespace(shape=(64, 32)), qpu_queue=gpu, cpu_queue=cpu, qpu_rows=16)
    plan._closed = True
    with pytest.raises(RuntimeError, match="closed"):
        plan.execute_prepared_hybrid_outputs(None, batch=32, qpu_queue=gpu, cpu_queue=cpu, qpu_outputs=256)


def test_hybrid_unit_rules() -> None:
    device = object()
    plan, submitted = _plan(device)
    gpu, cpu = SimpleNamespace(device=device), SimpleNamespace(device=device)
    source = SimpleNamespace(shape=(48, 32))
    for qpu_outputs in (0, -16, 100, 512, 528):
        with pytest.raises(ValueError, match="qpu_outputs must be aligned"):
            plan.execute_hybrid(None, source, qpu_queue=gpu, cpu_queue=cpu, qpu_outputs=qpu_outputs)
        with pytest.raises(ValueError, match="qpu_outputs must be aligned"):
            plan.execute_prepared_hybrid_outputs(None, batch=32, qpu_queue=gpu, cpu_queue=cpu, qpu_outputs=qpu_outputs)
    for qpu_rows in (0, 8, 48, 64):
        with pytest.raises(ValueError, match="qpu_rows must be aligned"):
            plan.execute_hybrid_rows(None, source, qpu_queue=gpu, cpu_queue=cpu, qpu_rows=qpu_rows)
        with pytest.raises(ValueError, match="qpu_rows must be aligned"):
            plan.execute_prepared_hybrid_rows(None, batch=48, qpu_queue=gpu, cpu_queue=cpu, qpu_rows=qpu_rows)
    with pytest.raises(ValueError, match="rank-2"):
        plan.execute_hybrid_rows(None, SimpleNamespace(shape=(48,)), qpu_queue=gpu, cpu_queue=cpu, qpu_rows=16)
    for batch in (0, 65):
        with pytest.raises(ValueError, match="batch exceeds"):
            plan.execute_prepared_hybrid_rows(None, batch=batch, qpu_queue=gpu, cpu_queue=cpu, qpu_rows=16)
    assert submitted == []
    assert plan.execute_hybrid(None, source, qpu_queue=gpu, cpu_queue=cpu, qpu_outputs=496) == "event"
    assert plan.execute_hybrid_rows(None, source, qpu_queue=gpu, cpu_queue=cpu, qpu_rows=32) == "event"
    assert plan.execute_prepared_hybrid_rows(None, batch=48, qpu_queue=gpu, cpu_queue=cpu, qpu_rows=16) == "event"
    assert plan.execute_prepared_hybrid_outputs(None, batch=48, qpu_queue=gpu, cpu_queue=cpu, qpu_outputs=16) == "event"
    assert submitted == [("execute", gpu), ("execute", gpu), ("execute_prepared", gpu), ("execute_prepared", gpu)]
