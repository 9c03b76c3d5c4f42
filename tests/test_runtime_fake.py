"""Host-side runtime semantics on the fake backend, mirroring tests/test_qpu_xla_runtime.py and
tests/test_qpu_xla_scheduler.py of the reference: zero-copy views, ordering, dependencies,
failure and cancellation propagation, Chrome trace, hazards, placement and candidate records."""

from __future__ import annotations

import json
import threading
import time
from pathlib import Path

import numpy as np
import pytest

from qpu_xla import (
    AccessMode,
    AllocationError,
    BufferClosedError,
    DependencyError,
    Device,
    DeviceClosedError,
    EventCancelledError,
    EventStatus,
    EventTimeoutError,
    Kernel,
    KernelError,
    Placement,
)
from qpu_xla.candidates import (
    CandidateRecord,
    CandidateRegistry,
    CandidateStatus,
    CorrectnessEvidence,
    PartitionEvidence,
    PerformanceEvidence,
)
from qpu_xla.placement import CapabilityRegistry, CostModel, ExecutionCandidate, OperationSpec, PartitionSpec
from qpu_xla.quantization import CalibratedW8A8Linear, PreparedW8A8Linear, QuantizedMatrixInt8


def test_fake_tensors_are_zero_copy_views_with_slices() -> None:
    with Device.fake() as device:
        tensor = device.tensor((4, 6), np.float32)
        tensor.numpy()[:] = np.arange(24, dtype=np.float32).reshape(4, 6)
        view = tensor.slice((slice(1, 3), slice(2, 5)))
        assert view.shape == (2, 3)
        np.testing.assert_array_equal(view.numpy(), np.arange(24, dtype=np.float32).reshape(4, 6)[1:3, 2:5])
        view.numpy()[:] = -1
        assert tensor.numpy()[1, 2] == -1
        assert view.address == tensor.address + 1 * 24 + 2 * 4
        with pytest.raises(AllocationError):
            tensor.slice((slice(0, 4, 2), slice(None)))


def test_closed_buffers_and_devices_reject_use() -> None:
    device = Device.fake()
    tensor = device.tensor((4,), np.int32)
    tensor.buffer.close()
    with pytest.raises(BufferClosedError):
        tensor.numpy()
    reused = device.tensor((2,), np.int32)  # released allocations are reused
    assert reused.buffer.nbytes == 8
    device.close()
    with pytest.raises(DeviceClosedError):
        device.tensor((1,), np.float32)
    with pytest.raises(DeviceClosedError):
        device.queue()


def test_queue_runs_host_tasks_in_order_and_propagates_failures() -> None:
    with Device.fake() as device, device.queue() as queue:
        order: list[int] = []
        first = queue.host_task(lambda: order.append(1), name="first")
        second = queue.host_task(lambda: (_ for _ in ()).throw(RuntimeError("boom")), name="second")
        third = queue.host_task(lambda: order.append(3), name="third", wait_for=(first,))
        third.wait()
        with pytest.raises(RuntimeError, match="boom"):
            second.wait()
        assert order == [1, 3]
        assert second.status is EventStatus.FAILED and third.status is EventStatus.SUCCEEDED


def test_cross_queue_dependencies_and_cancellation() -> None:
    with Device.fake() as device, device.queue() as first, device.queue() as second:
        gate = threading.Event()
        blocker = first.host_task(lambda: gate.wait(5), name="blocker")
        dependent = second.host_task(lambda: None, wait_for=(blocker,), name="dependent")
        pending = first.host_task(lambda: None, name="pending")
        assert pending.cancel()
        with pytest.raises(EventTimeoutError):
            dependent.wait(timeout=0.05)
        gate.set()
        dependent.wait()
        with pytest.raises(EventCancelledError):
            pending.wait()


def test_failed_dependency_fails_its_dependents() -> None:
    with Device.fake() as device, device.queue() as queue:
        failing = queue.host_task(lambda: 1 / 0, name="failing")
        dependent = queue.host_task(lambda: None, wait_for=(failing,), name="dependent")
        with pytest.raises(ZeroDivisionError):
            dependent.wait()


def test_foreign_events_and_buffers_are_rejected() -> None:
    with Device.fake() as one, Device.fake() as two, one.queue() as q1, two.queue() as q2:
        event = q1.host_task(lambda: None)
        with pytest.raises(DependencyError):
            q2.host_task(lambda: None, wait_for=(event,))
        tensor = one.tensor((4,), np.float32)
        with pytest.raises(DependencyError):
            q2.host_task(lambda: None, buffers=(tensor.access(AccessMode.READ),))
        with pytest.raises(DependencyError):
            q2.host_task(lambda: None, wait_for=("not an event",))  # type: ignore[arg-type]


def test_kernels_on_the_fake_backend_fail_as_kernel_errors() -> None:
    from qpu_xla.kernels import CUDA_W8A8_GEMM_KERNEL

    with Device.fake() as device, device.queue() as queue:
        left = device.tensor((16, 16), np.int8)
        right = device.tensor((16, 16), np.int8)
        out = device.tensor((16, 16), np.int32)
        event = queue.submit(CUDA_W8A8_GEMM_KERNEL, (left, right, out))
        with pytest.raises(KernelError):
            event.wait()
        wrapped = queue.submit(Kernel("raises", lambda backend, args, grid, stream: (_ for _ in ()).throw(ValueError("x"))))
        with pytest.raises(KernelError):
            wrapped.wait()
        with pytest.raises(KernelError):
            queue.submit(CUDA_W8A8_GEMM_KERNEL, (left, right, out), grid=(0, 1, 1))


def test_chrome_trace_and_completed_counts(tmp_path: Path) -> None:
    with Device.fake() as device, device.queue() as queue:
        first = queue.host_task(lambda: time.sleep(0.001), name="a")
        second = queue.host_task(lambda: None, name="b", wait_for=(first,))
        second.wait()
        trace = queue.chrome_trace()["traceEvents"]
        names = {event["name"] for event in trace}
        assert {"a", "b", "dependency"} <= names
        path = tmp_path / "trace.json"
        queue.write_chrome_trace(path)
        assert json.loads(path.read_text())["traceEvents"]
        assert queue.consume_completed_event_counts() == {"host": 2}
        assert queue.consume_completed_event_counts() == {}


def test_hazard_ledger_reports_overlapping_writes() -> None:
    with Device.fake() as device, device.queue() as queue:
        tensor = device.tensor((8,), np.float32)
        gate = threading.Event()
        event = queue.host_task(lambda: gate.wait(5), buffers=(tensor.access(AccessMode.WRITE),))
        head = tensor.slice((slice(0, 4),))
        assert queue.hazards((head.access(AccessMode.READ),)) == [event]
        gate.set()
        event.wait()
        assert queue.hazards((head.access(AccessMode.READ),)) == []


def test_prepared_w8a8_linear_rejects_a_cpu_only_backend() -> None:
    """Like the reference (tests/test_qpu_xla_quantization.py:92-95): no CPU execution path."""
    values = np.ones((16, 16), dtype=np.int8)
    scales = np.ones(16, dtype=np.float32)
    with Device.fake() as device, pytest.raises(ValueError, match="CUDA"):
        PreparedW8A8Linear(device, QuantizedMatrixInt8(values, scales), max_batch=16)


def test_quantized_matrix_contract() -> None:
    with pytest.raises(ValueError):
        QuantizedMatrixInt8(np.ones((2, 3), dtype=np.int8), np.ones(3, dtype=np.float32))
    with pytest.raises(ValueError):
        QuantizedMatrixInt8(np.ones((2, 3), dtype=np.int8), np.array([1.0, 0.0], dtype=np.float32))
    matrix = QuantizedMatrixInt8(np.array([[1, -2]], dtype=np.int8), np.array([0.5], dtype=np.float32))
    np.testing.assert_array_equal(matrix.dequantize(), [[0.5, -1.0]])


def test_calibrated_linear_argument_checks_on_the_fake_device() -> None:
    values = np.ones((32, 16), dtype=np.int8)
    scales = np.ones(32, dtype=np.float32)
    with Device.fake() as device, device.queue() as queue:
        plan = CalibratedW8A8Linear(device, QuantizedMatrixInt8(values, scales), max_batch=32, candidates=CandidateRegistry())
        source = device.tensor((32, 16), np.float32)
        destination = device.tensor((32, 32), np.float32)
        with pytest.raises(ValueError, match="mutually exclusive"):
            plan.execute(destination, source, queue=queue, qpu_rows=16, qpu_outputs=16)
        with pytest.raises(ValueError, match="not available"):
            plan.execute(destination, source, queue=queue, placement=Placement.CPU)
        with pytest.raises(ValueError, match="CUDA backend"):
            plan.execute(destination, source, queue=queue)
        plan.close()


def correctness() -> CorrectnessEvidence:
    return CorrectnessEvidence("oracle", 1, True, 0.0, 0.0, 0.0, 0.0)


def test_candidate_registry_round_trip_and_exact_shape_lookup(tmp_path: Path) -> None:
    winning = CandidateRecord(
        "cuda-128x2048x2048", "linear", "w8a8-i32-fp32", "row-major-k", "128x2048x2048", "hash",
        CandidateStatus.SUPPORTED_WIN, correctness(), PerformanceEvidence("numpy", (0.1,), (0.001,)), placement="cuda",
    )
    slower = CandidateRecord(
        "cuda-slow", "linear", "w8a8-i32-fp32", "row-major-k", "128x2048x2048", "hash",
        CandidateStatus.EXPERIMENTAL_CORRECT_SLOWER, correctness(), PerformanceEvidence("numpy", (0.1,), (0.2,)),
    )
    hybrid = CandidateRecord(
        "hybrid", "linear", "w8a8-i32-fp32", "row-major-k", "128x2048x2048", "hash", CandidateStatus.SUPPORTED_WIN,
        correctness(), PerformanceEvidence("numpy", (0.1,), (0.05,)), placement="hybrid",
        partition=PartitionEvidence("outputs", 1024, 2048, 16),
    )
    registry = CandidateRegistry((winning, slower, hybrid))
    found = registry.supported_for(operation="linear", dtype="w8a8-i32-fp32", layout="row-major-k", shape_class="128x2048x2048")
    assert {record.name for record in found} == {"cuda-128x2048x2048", "hybrid"}
    path = tmp_path / "candidates.json"
    registry.save(path)
    loaded = CandidateRegistry.load(path)
    assert loaded.records == registry.records
    with pytest.raises(ValueError):
        CandidateRecord("x", "linear", "d", "l", "s", "h", CandidateStatus.SUPPORTED_WIN, correctness(), PerformanceEvidence("n", (1.0,), (1.0,)))
    with pytest.raises(ValueError):
        registry.register(winning)


def test_capability_registry_prefers_calibrated_cuda(tmp_path: Path) -> None:
    spec = OperationSpec("linear", "w8a8", (128, 2048, 2048))
    registry = CapabilityRegistry(
        (
            ExecutionCandidate("cpu", Placement.CPU, lambda s: True, lambda s: 0.5),
            ExecutionCandidate("cuda", Placement.CUDA, lambda s: True, lambda s: 1.0, requires_calibration=True),
        )
    )
    assert registry.choose(spec).candidate.name == "cpu"  # cuda needs calibration under AUTO
    model = CostModel()
    model.record(spec, "cuda", 1e-5)
    model.record(spec, "cuda", 2e-5)
    plan = registry.choose(spec, cost_model=model)
    assert plan.candidate.name == "cuda" and plan.calibrated and plan.estimated_seconds == pytest.approx(1.5e-5)
    path = tmp_path / "cost.json"
    model.save(path)
    assert CostModel.load(path).estimate(spec, "cuda") == pytest.approx(1.5e-5)
    assert registry.choose(spec, preference=Placement.CUDA).candidate.name == "cuda"
    with pytest.raises(ValueError):
        PartitionSpec("outputs", 0, 16)
    with pytest.raises(ValueError):
        ExecutionCandidate("h", Placement.HYBRID, lambda s: True, lambda s: 1.0)


def test_reference_style_three_argument_executors_run() -> None:
    """``Kernel(name, executor)`` with the reference's ``executor(backend, args, grid)`` form
    (src/qpu_xla/kernel.py:24-38) runs as submitted; this build's stream-aware form takes a fourth
    argument."""
    with Device.fake() as device, device.queue() as queue:
        calls: list[object] = []
        queue.submit(Kernel("three", lambda backend, args, grid: calls.append((args, grid))), ("a",), grid=(2, 3, 4)).wait()
        queue.submit(Kernel("four", lambda backend, args, grid, stream: calls.append((args, grid, stream))), ("b",)).wait()
        assert calls == [(("a",), (2, 3, 4)), (("b",), (1, 1, 1), None)]


def test_cost_model_reads_the_reference_file_format(tmp_path: Path) -> None:
    """A cost model saved in the reference's JSON form (fingerprint + records) loads and drives
    placement; malformed records are refused."""
    path = tmp_path / "reference-cost.json"
    path.write_text(json.dumps({
        "fingerprint": {"device": "b200"},
        "records": [{"name": "linear", "dtype": "w8a8", "shape": [1, 64, 64], "layout": "", "candidate": "cuda", "seconds": [3e-6, 1e-6, 2e-6]}],
    }))
    model = CostModel.load(path)
    assert model.fingerprint == {"device": "b200"}
    assert model.estimate(OperationSpec("linear", "w8a8", (1, 64, 64)), "cuda") == pytest.approx(2e-6)
    model.save(path)
    assert CostModel.load(path).to_dict() == model.to_dict()
    path.write_text(json.dumps({"fingerprint": {}, "records": [{"name": "x", "dtype": "d", "shape": [0], "layout": "", "candidate": "c", "seconds": [1.0]}]}))
    with pytest.raises(ValueError, match="invalid fields"):
        CostModel.load(path)


def test_candidate_records_keep_quality_evidence(tmp_path: Path) -> None:
    from qpu_xla.candidates import QualityEvidence

    quality = QualityEvidence("numpy-fp32", 0.02, 0.999, max_abs_error=0.1, top1_agreement=1.0)
    record = CandidateRecord(
        "q", "linear", "w8a8-i32-fp32", "row-major-k", "1x64x64", "hash", CandidateStatus.SUPPORTED_WIN, correctness(),
        PerformanceEvidence("numpy", (0.1,), (0.001,)), quality=quality,
    )
    path = tmp_path / "candidates.json"
    CandidateRegistry((record,)).save(path)
    assert CandidateRegistry.load(path).records == (record,)
    assert quality.passes_default_gate
    with pytest.raises(ValueError, match="cosine"):
        QualityEvidence("numpy-fp32", 0.02, 1.5)
