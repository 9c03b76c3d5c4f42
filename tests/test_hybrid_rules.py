"""``PreparedW8A8Linear.execute_hybrid``'s argument rules (src/qpu_xla/models/tinyllama/
quantization.py:350-391) on CPU: the plan's host-side state only, with the GPU submission
replaced by a recorder. The GPU run of the same call is in test_gpu_runtime.py."""

from __future__ import annotations

from types import SimpleNamespace

import pytest

from qpu_xla.errors import DependencyError
from qpu_xla.quantization import PreparedW8A8Linear


def _plan(device: object) -> tuple[PreparedW8A8Linear, list[object]]:
    plan = object.__new__(PreparedW8A8Linear)
    plan._closed = False
    plan._last_event = None
    plan._cpu_queue = None
    plan.device = device
    plan.output_count = 512
    submitted: list[object] = []

    def execute(destination: object, source: object, *, queue: object, wait_for: object = ()) -> str:
        submitted.append(queue)
        return "event"

    plan.execute = execute  # type: ignore[method-assign]
    return plan, submitted


def test_hybrid_argument_rules() -> None:
    device = object()
    plan, submitted = _plan(device)
    gpu, cpu, other_cpu = (SimpleNamespace(device=device) for _ in range(3))
    foreign = SimpleNamespace(device=object())
    with pytest.raises(DependencyError, match="distinct"):
        plan.execute_hybrid(None, None, qpu_queue=gpu, cpu_queue=gpu, qpu_outputs=256)
    with pytest.raises(DependencyError, match="plan device"):
        plan.execute_hybrid(None, None, qpu_queue=gpu, cpu_queue=foreign, qpu_outputs=256)
    for qpu_outputs in (0, -16, 100, 512, 528):
        with pytest.raises(ValueError, match="aligned"):
            plan.execute_hybrid(None, None, qpu_queue=gpu, cpu_queue=cpu, qpu_outputs=qpu_outputs)
    assert submitted == []
    # both parts go to the GPU queue; the CPU queue is bound but receives no work
    assert plan.execute_hybrid(None, None, qpu_queue=gpu, cpu_queue=cpu, qpu_outputs=256) == "event"
    assert submitted == [gpu]
    with pytest.raises(DependencyError, match="first CPU queue"):
        plan.execute_hybrid(None, None, qpu_queue=gpu, cpu_queue=other_cpu, qpu_outputs=256)
    plan._last_event = SimpleNamespace(done=False)
    with pytest.raises(RuntimeError, match="in-flight"):
        plan.execute_hybrid(None, None, qpu_queue=gpu, cpu_queue=cpu, qpu_outputs=256)
    plan._closed = True
    with pytest.raises(RuntimeError, match="closed"):
        plan.execute_hybrid(None, None, qpu_queue=gpu, cpu_queue=cpu, qpu_outputs=256)
