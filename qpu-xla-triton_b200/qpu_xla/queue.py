"""In-order queues and events over CUDA streams and CUDA events.

Same surface as src/qpu_xla/queue.py:23-393: ``Queue.submit(kernel, args, *,
grid, wait_for, buffers) -> Event``, ``Queue.host_task``, ``Event.wait(timeout)``
/ ``status`` / ``done`` / ``cancel``, the hazard ledger, Chrome-trace export and
``consume_completed_event_counts``. One worker thread per queue preserves
submission order, exactly as the reference's ``Queue._run`` (:376-393).

On the CUDA backend each queue owns one CUDA stream. A kernel submission
launches on that stream and its event completes when a CUDA event recorded
after the launch completes (no host round trip in between); a dependency on an
event of another queue becomes ``cudaStreamWaitEvent`` on the GPU. Host tasks
first wait (on the host) for the queue's earlier GPU work, so host code always
observes the results of the kernels submitted before it.
"""

from __future__ import annotations

import json
import time
from collections.abc import Callable, Iterable
from dataclasses import dataclass
from enum import Enum
from os import PathLike
from queue import Queue as ThreadQueue
from threading import Condition, Lock, Thread
from time import monotonic_ns
from typing import TYPE_CHECKING, Any, Self

from qpu_xla.errors import DependencyError, DeviceClosedError, EventCancelledError, EventTimeoutError
from qpu_xla.kernel import Kernel, LaunchConfig
from qpu_xla.memory import BufferAccess

if TYPE_CHECKING:
    from qpu_xla.device import Device


class EventStatus(Enum):
    PENDING = "pending"
    RUNNING = "running"
    SUCCEEDED = "succeeded"
    FAILED = "failed"
    CANCELLED = "cancelled"


class Event:
    """Completion state, failure propagation and timestamps of one submission."""

    def __init__(self: Self, queue: Queue, *, sequence: int, name: str, category: str, dependencies: tuple[Event, ...]) -> None:
        self._queue = queue
        self._sequence = sequence
        self._name = name
        self._category = category
        self._dependencies = dependencies
        self._condition = Condition()
        self._status = EventStatus.PENDING
        self._exception: BaseException | None = None
        self._submitted_ns = monotonic_ns()
        self._started_ns: int | None = None
        self._finished_ns: int | None = None
        # CUDA completion (kernel submissions): events recorded around the launch.
        self._launched = False
        self._cuda_start: Any = None
        self._cuda_end: Any = None
        self._device_ms: float | None = None

    @property
    def queue(self: Self) -> Queue:
        return self._queue

    @property
    def name(self: Self) -> str:
        return self._name

    @property
    def category(self: Self) -> str:
        return self._category

    @property
    def cuda_event(self: Self) -> Any:
        """The CUDA event recorded after this submission's launch (None for host tasks)."""
        return self._cuda_end

    @property
    def status(self: Self) -> EventStatus:
        self._poll_device()
        with self._condition:
            return self._status

    @property
    def submitted_ns(self: Self) -> int:
        return self._submitted_ns

    @property
    def started_ns(self: Self) -> int | None:
        with self._condition:
            return self._started_ns

    @property
    def finished_ns(self: Self) -> int | None:
        self._poll_device()
        with self._condition:
            return self._finished_ns

    @property
    def device_milliseconds(self: Self) -> float | None:
        """GPU time between the CUDA events around the launch, once complete."""
        self._poll_device()
        return self._device_ms

    @property
    def exception(self: Self) -> BaseException | None:
        with self._condition:
            return self._exception

    @property
    def done(self: Self) -> bool:
        self._poll_device()
        with self._condition:
            return self._status in {EventStatus.SUCCEEDED, EventStatus.FAILED, EventStatus.CANCELLED}

    def cancel(self: Self) -> bool:
        """Cancel a queued submission the worker has not started."""
        with self._condition:
            if self._status is not EventStatus.PENDING:
                return False
            self._status = EventStatus.CANCELLED
            self._finished_ns = monotonic_ns()
            self._condition.notify_all()
            return True

    def wait(self: Self, timeout: float | None = None) -> None:
        """Wait for completion; re-raise a cancellation or failure (queue.py:113-126)."""
        if timeout is not None and timeout < 0:
            raise ValueError("timeout must be non-negative or None")
        deadline = None if timeout is None else time.monotonic() + timeout
        with self._condition:
            ready = self._condition.wait_for(
                lambda: self._launched or self._status in {EventStatus.SUCCEEDED, EventStatus.FAILED, EventStatus.CANCELLED},
                timeout=timeout,
            )
            if not ready:
                raise EventTimeoutError("event did not complete before the timeout")
        if self._cuda_end is not None:
            delay = 2e-6
            while not self._poll_device():
                if deadline is not None and time.monotonic() > deadline:
                    raise EventTimeoutError("event did not complete before the timeout")
                time.sleep(delay)
                delay = min(delay * 2, 1e-3)
        with self._condition:
            if self._status is EventStatus.CANCELLED:
                raise EventCancelledError("event was cancelled")
            if self._status is EventStatus.FAILED:
                assert self._exception is not None
                raise self._exception

    # -- worker-side transitions ------------------------------------------------

    def _start(self: Self) -> bool:
        with self._condition:
            if self._status is EventStatus.CANCELLED:
                return False
            if self._status is not EventStatus.PENDING:
                raise RuntimeError("event cannot be started more than once")
            self._status = EventStatus.RUNNING
            self._started_ns = monotonic_ns()
            return True

    def _mark_launched(self: Self, start: Any, end: Any) -> None:
        with self._condition:
            self._cuda_start = start
            self._cuda_end = end
            self._launched = True
            self._condition.notify_all()

    def _poll_device(self: Self) -> bool:
        """Complete a launched kernel event once its CUDA event has completed."""
        with self._condition:
            if self._status is not EventStatus.RUNNING or not self._launched or self._cuda_end is None:
                return self._status is not EventStatus.RUNNING and self._status is not EventStatus.PENDING
        if not self._cuda_end.query():
            return False
        exception: BaseException | None = None
        try:
            self._queue._check_device_errors()
        except BaseException as exc:  # a kernel-side bounded wait expired
            exception = exc
        with self._condition:
            if self._status is EventStatus.RUNNING:
                if self._cuda_start is not None:
                    self._device_ms = float(self._cuda_start.elapsed_time(self._cuda_end))
                self._exception = exception
                self._status = EventStatus.FAILED if exception is not None else EventStatus.SUCCEEDED
                self._finished_ns = monotonic_ns()
                self._condition.notify_all()
        return True

    def _finish(self: Self, exception: BaseException | None = None) -> None:
        with self._condition:
            if self._status is EventStatus.CANCELLED:
                return
            self._exception = exception
            self._status = EventStatus.FAILED if exception is not None else EventStatus.SUCCEEDED
            self._finished_ns = monotonic_ns()
            self._condition.notify_all()

    def _wait_launched(self: Self) -> None:
        """Host wait until a kernel event is launched (or the event ends); re-raise its failure."""
        with self._condition:
            self._condition.wait_for(
                lambda: self._launched or self._status in {EventStatus.SUCCEEDED, EventStatus.FAILED, EventStatus.CANCELLED}
            )
            if self._status is EventStatus.CANCELLED:
                raise EventCancelledError("dependency was cancelled")
            if self._status is EventStatus.FAILED:
                assert self._exception is not None
                raise self._exception


@dataclass(slots=True)
class _Submission:
    event: Event
    action: Callable[[], None]
    dependencies: tuple[Event, ...]
    kernel: bool


class Queue:
    """A single-worker, in-order queue for CUDA kernels and declared host work."""

    def __init__(self: Self, device: Device) -> None:
        self._device = device
        self._stream: Any = None
        if device.is_cuda:
            import torch

            self._stream = torch.cuda.Stream(device=device.backend.torch_device)  # type: ignore[attr-defined]
        self._submissions: ThreadQueue[_Submission | None] = ThreadQueue()
        self._lock = Lock()
        self._closed = False
        self._tail: Event | None = None
        self._events: list[Event] = []
        self._next_sequence = 0
        self._live_accesses: list[tuple[BufferAccess, Event]] = []
        self._worker = Thread(target=self._run, name="qpu-xla-submit", daemon=True)
        self._worker.start()

    @property
    def device(self: Self) -> Device:
        return self._device

    @property
    def stream(self: Self) -> Any:
        """The torch CUDA stream of this queue (None on the fake backend)."""
        return self._stream

    @property
    def closed(self: Self) -> bool:
        with self._lock:
            return self._closed

    def submit(
        self: Self,
        kernel: Kernel,
        args: tuple[Any, ...] = (),
        *,
        grid: tuple[int, int, int] = (1, 1, 1),
        wait_for: Iterable[Event] = (),
        buffers: Iterable[BufferAccess] = (),
    ) -> Event:
        """Queue a kernel launch and return its completion event (queue.py:186-210)."""
        launch = LaunchConfig(tuple(grid))  # type: ignore[arg-type]
        backend = self._device.backend
        stream = self._stream

        def action() -> None:
            kernel.execute(backend, args, launch, stream)

        return self._enqueue(action, wait_for=wait_for, buffers=buffers, name=kernel.name, category="cuda", kernel=True)

    def host_task(
        self: Self,
        fn: Callable[[], None],
        *,
        wait_for: Iterable[Event] = (),
        buffers: Iterable[BufferAccess] = (),
        name: str | None = None,
    ) -> Event:
        """Queue host work with the same dependency and hazard declarations (queue.py:212-222)."""
        task_name = name if name is not None else str(getattr(fn, "__qualname__", "host_task"))
        return self._enqueue(fn, wait_for=wait_for, buffers=buffers, name=task_name, category="host", kernel=False)

    def _enqueue(
        self: Self,
        action: Callable[[], None],
        *,
        wait_for: Iterable[Event],
        buffers: Iterable[BufferAccess],
        name: str,
        category: str,
        kernel: bool,
    ) -> Event:
        declared = tuple(buffers)
        for access in declared:
            if access.buffer.device is not self._device:
                raise DependencyError("a buffer access belongs to a different device")
        with self._lock:
            if self._closed:
                raise DeviceClosedError("queue is closed")
            dependencies = self._normalize_dependencies(wait_for)
            # The in-order worker already serialises conflicting accesses on this
            # queue; the ledger keeps them for cross-queue diagnostics.
            self._live_accesses = [(access, event) for access, event in self._live_accesses if not event.done]
            event = Event(self, sequence=self._next_sequence, name=name, category=category, dependencies=dependencies)
            self._next_sequence += 1
            self._tail = event
            self._events.append(event)
            self._live_accesses.extend((access, event) for access in declared)
            self._submissions.put(_Submission(event, action, dependencies, kernel))
            return event

    def hazards(self: Self, accesses: Iterable[BufferAccess]) -> list[Event]:
        """Live events whose declared accesses conflict with ``accesses``."""
        wanted = tuple(accesses)
        with self._lock:
            return [event for access, event in self._live_accesses if not event.done and any(access.conflicts_with(other) for other in wanted)]

    def _normalize_dependencies(self: Self, wait_for: Iterable[Event]) -> tuple[Event, ...]:
        dependencies: list[Event] = []
        for event in wait_for:
            if not isinstance(event, Event):
                raise DependencyError("wait_for must contain Event instances")
            if event.queue.device is not self._device:
                raise DependencyError("event dependency belongs to a different device")
            if event not in dependencies:
                dependencies.append(event)
        return tuple(dependencies)

    def _check_device_errors(self: Self) -> None:
        """Raise if a kernel on this device reported an expired bounded wait."""
        backend = self._device.backend
        if getattr(backend, "kind", "") == "cuda" and self._stream is not None:
            backend.launch(self._stream, lambda native: native.synchronize())  # type: ignore[attr-defined]

    def _run(self: Self) -> None:
        while True:
            submission = self._submissions.get()
            if submission is None:
                self._submissions.task_done()
                return
            event = submission.event
            try:
                if event._start():
                    self._run_one(submission)
            except BaseException as exc:
                event._finish(exc)
            finally:
                self._submissions.task_done()

    def _run_one(self: Self, submission: _Submission) -> None:
        event = submission.event
        stream = self._stream
        if stream is None:
            for dependency in submission.dependencies:
                dependency.wait()
            submission.action()
            event._finish()
            return
        import torch

        if submission.kernel:
            for dependency in submission.dependencies:
                dependency._wait_launched()
                if dependency.cuda_event is not None:
                    stream.wait_event(dependency.cuda_event)
                else:
                    dependency.wait()
            start = torch.cuda.Event(enable_timing=True)
            end = torch.cuda.Event(enable_timing=True)
            with torch.cuda.stream(stream):
                start.record(stream)
                submission.action()
                end.record(stream)
            event._mark_launched(start, end)
        else:
            for dependency in submission.dependencies:
                dependency.wait()
            stream.synchronize()  # in-order: earlier kernels of this queue are complete
            submission.action()
            event._finish()

    def finish(self: Self, timeout: float | None = None) -> None:
        """Wait for every submitted event (failures are left on their events)."""
        with self._lock:
            events = tuple(self._events)
        for event in events:
            try:
                event.wait(timeout)
            except (EventCancelledError, EventTimeoutError):
                raise
            except BaseException:
                pass

    def chrome_trace(self: Self) -> dict[str, list[dict[str, object]]]:
        """Chrome Trace Event payload (queue.py:275-347): queue delay, execution and dependency flows.

        Kernel slices use the GPU time measured between the CUDA events around the launch.
        """
        with self._lock:
            events = tuple(self._events)
        trace: list[dict[str, object]] = []
        for event in events:
            started_ns = event.started_ns
            finished_ns = event.finished_ns
            if started_ns is None:
                continue
            submitted_us = event.submitted_ns / 1_000
            started_us = started_ns / 1_000
            if started_ns > event.submitted_ns:
                trace.append(
                    {"name": f"queue delay: {event.name}", "cat": "queue", "ph": "X", "pid": "qpu-xla", "tid": "submission",
                     "ts": submitted_us, "dur": started_us - submitted_us, "args": {"event": event._sequence}}
                )
            if finished_ns is not None:
                device_ms = event.device_milliseconds
                duration_us = device_ms * 1_000 if device_ms is not None else max(0, finished_ns - started_ns) / 1_000
                trace.append(
                    {"name": event.name, "cat": event._category, "ph": "X", "pid": "qpu-xla", "tid": event._category,
                     "ts": started_us, "dur": duration_us, "args": {"event": event._sequence, "status": event.status.value}}
                )
            for dependency in event._dependencies:
                dependency_finished_ns = dependency.finished_ns
                if dependency_finished_ns is None:
                    continue
                flow_id = f"{dependency._sequence}->{event._sequence}"
                trace.extend(
                    (
                        {"name": "dependency", "cat": "sync", "ph": "s", "pid": "qpu-xla", "tid": dependency._category,
                         "ts": dependency_finished_ns / 1_000, "id": flow_id},
                        {"name": "dependency", "cat": "sync", "ph": "f", "pid": "qpu-xla", "tid": event._category,
                         "ts": started_us, "id": flow_id},
                    )
                )
        return {"traceEvents": trace}

    def consume_completed_event_counts(self: Self) -> dict[str, int]:
        """Count and drop completed events by category, bounding profiling memory (queue.py:349-369)."""
        with self._lock:
            completed: list[Event] = []
            retained: list[Event] = []
            for event in self._events:
                (completed if event.done else retained).append(event)
            self._events = retained
            self._live_accesses = [(access, event) for access, event in self._live_accesses if not event.done]
        counts: dict[str, int] = {}
        for event in completed:
            counts[event._category] = counts.get(event._category, 0) + 1
        return counts

    def write_chrome_trace(self: Self, path: str | PathLike[str]) -> None:
        with open(path, "w", encoding="utf-8") as trace_file:
            json.dump(self.chrome_trace(), trace_file, separators=(",", ":"))

    def close(self: Self) -> None:
        """Stop accepting work and wait until submitted work has finished."""
        with self._lock:
            if self._closed:
                return
            self._closed = True
        self._submissions.put(None)
        self._worker.join()
        if self._stream is not None:
            self._stream.synchronize()

    def __enter__(self: Self) -> Self:
        return self

    def __exit__(self: Self, exc_type: object, exc_value: object, traceback: object) -> None:
        self.close()


__all__ = ["Event", "EventStatus", "Queue"]
