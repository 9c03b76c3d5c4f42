"""In-order queues and events over CUDA streams and CUDA events.

The drop-in surface of src/qpu_xla/queue.py: ``Queue.submit(kernel, args, *, grid,
wait_for, buffers) -> Event``, ``Queue.host_task``, ``Event.wait(timeout)`` /
``status`` / ``done`` / ``cancel``, buffer hazards, Chrome-trace export and
``consume_completed_event_counts``.

How it runs here. Each queue has one worker thread that takes submissions in order,
so a queue never reorders its own work. On the CUDA backend the queue also owns a
CUDA stream:

* a kernel submission is *launched* by the worker -- the executor enqueues its CUDA
  work on the stream between two CUDA events -- and its :class:`Event` completes when
  the second CUDA event has; the host never waits in between;
* a dependency on another queue's kernel becomes ``cudaStreamWaitEvent`` on the GPU
  (the worker only waits until that kernel has been launched);
* a host task first waits for the queue's earlier GPU work and for its dependencies,
  so host code sees the results of everything submitted before it.

Every declared buffer access of a submission that has not finished is kept in a
ledger indexed by allocation; ``Queue.hazards`` reports the events whose ranges
overlap a given access with at least one side writing.
"""

from __future__ import annotations

import itertools
import json
import threading
import time
from collections import Counter, defaultdict
from collections.abc import Callable, Iterable, Iterator
from enum import Enum
from os import PathLike
from queue import SimpleQueue
from time import monotonic_ns
from typing import TYPE_CHECKING, Any, NamedTuple, Self

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


_FINAL = frozenset({EventStatus.SUCCEEDED, EventStatus.FAILED, EventStatus.CANCELLED})


class Event:
    """One submission: its state, its failure, host timestamps and (kernels) GPU completion.

    Two latches carry the state to waiters: ``_launched`` opens once the submission's
    CUDA work is on the stream (or the event has ended without any), ``_ended`` once the
    event is final.
    """

    def __init__(self: Self, queue: Queue, *, sequence: int, name: str, category: str, dependencies: tuple[Event, ...]) -> None:
        self._queue = queue
        self._sequence = sequence
        self._name = name
        self._category = category
        self._dependencies = dependencies
        self._guard = threading.Lock()
        self._launched = threading.Event()
        self._ended = threading.Event()
        self._state = EventStatus.PENDING
        self._error: BaseException | None = None
        self._submitted_ns = monotonic_ns()
        self._started_ns: int | None = None
        self._finished_ns: int | None = None
        self._gpu_marks: tuple[Any, Any] | None = None  # CUDA events before / after the launch
        self._device_ms: float | None = None

    # -- read side ------------------------------------------------------------------

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
        marks = self._gpu_marks
        return None if marks is None else marks[1]

    @property
    def status(self: Self) -> EventStatus:
        self._refresh()
        return self._state

    @property
    def submitted_ns(self: Self) -> int:
        return self._submitted_ns

    @property
    def started_ns(self: Self) -> int | None:
        return self._started_ns

    @property
    def finished_ns(self: Self) -> int | None:
        self._refresh()
        return self._finished_ns

    @property
    def device_milliseconds(self: Self) -> float | None:
        """GPU time between the CUDA events around the launch, once complete."""
        self._refresh()
        return self._device_ms

    @property
    def exception(self: Self) -> BaseException | None:
        return self._error

    @property
    def done(self: Self) -> bool:
        self._refresh()
        return self._state in _FINAL

    def cancel(self: Self) -> bool:
        """Cancel the submission if its queue's worker has not started it."""
        return self._end(EventStatus.CANCELLED, None, only_from=EventStatus.PENDING)

    def wait(self: Self, timeout: float | None = None) -> None:
        """Block until the event ends; raise its failure, or EventCancelledError if cancelled."""
        if timeout is not None and timeout < 0:
            raise ValueError("timeout must be non-negative or None")
        deadline = None if timeout is None else time.monotonic() + timeout

        def remaining() -> float | None:
            return None if deadline is None else max(0.0, deadline - time.monotonic())

        if not self._launched.wait(remaining()):
            raise EventTimeoutError("event did not complete before the timeout")
        pause = 2e-6
        while not self._refresh():
            if deadline is not None and time.monotonic() >= deadline:
                raise EventTimeoutError("event did not complete before the timeout")
            time.sleep(pause)
            pause = min(2 * pause, 1e-3)
        self._raise_outcome(EventCancelledError("event was cancelled"))

    def _raise_outcome(self: Self, cancelled: BaseException) -> None:
        if self._state is EventStatus.CANCELLED:
            raise cancelled
        if self._state is EventStatus.FAILED:
            assert self._error is not None
            raise self._error

    # -- worker side ------------------------------------------------------------------

    def _end(self: Self, state: EventStatus, error: BaseException | None, *, only_from: EventStatus | None = None) -> bool:
        """Move to a final state (from ``only_from`` only, when given); False if that is not allowed."""
        with self._guard:
            if self._state in _FINAL or (only_from is not None and self._state is not only_from):
                return False
            self._state = state
            self._error = error
            self._finished_ns = monotonic_ns()
        self._launched.set()
        self._ended.set()
        return True

    def _begin(self: Self) -> bool:
        """PENDING -> RUNNING when the worker picks the submission up; False if it was cancelled."""
        with self._guard:
            if self._state is EventStatus.CANCELLED:
                return False
            if self._state is not EventStatus.PENDING:
                raise RuntimeError("event cannot be started more than once")
            self._state = EventStatus.RUNNING
            self._started_ns = monotonic_ns()
            return True

    def _on_stream(self: Self, before: Any, after: Any) -> None:
        """The submission's CUDA work is enqueued between ``before`` and ``after``."""
        self._gpu_marks = (before, after)
        self._launched.set()

    def _refresh(self: Self) -> bool:
        """Final yet? A launched kernel event becomes final when its closing CUDA event has completed."""
        if self._ended.is_set():
            return True
        marks = self._gpu_marks
        if marks is None or self._state is not EventStatus.RUNNING or not marks[1].query():
            return False
        try:
            self._queue._raise_device_errors()
        except BaseException as error:  # a kernel's bounded wait expired on the device
            self._end(EventStatus.FAILED, error)
            return True
        self._device_ms = float(marks[0].elapsed_time(marks[1]))
        self._end(EventStatus.SUCCEEDED, None)
        return True

    def _await_launch(self: Self) -> None:
        """Block until this dependency's GPU work is enqueued (or it ended); raise if it did not succeed."""
        self._launched.wait()
        if self._ended.is_set():
            self._raise_outcome(EventCancelledError("dependency was cancelled"))


class _Job(NamedTuple):
    event: Event
    run: Callable[[], None]
    dependencies: tuple[Event, ...]
    on_gpu: bool


class _Ledger:
    """Declared accesses of unfinished submissions, grouped by the allocation they touch."""

    def __init__(self: Self) -> None:
        self._by_block: dict[int, list[tuple[BufferAccess, Event]]] = defaultdict(list)

    def add(self: Self, accesses: Iterable[BufferAccess], event: Event) -> None:
        for access in accesses:
            self._by_block[id(access.buffer._block)].append((access, event))

    def conflicts(self: Self, accesses: Iterable[BufferAccess]) -> list[Event]:
        found: list[Event] = []
        for access in accesses:
            for held, event in self._by_block.get(id(access.buffer._block), ()):
                if event not in found and not event.done and access.conflicts_with(held):
                    found.append(event)
        return found

    def prune(self: Self) -> None:
        for key in list(self._by_block):
            live = [(access, event) for access, event in self._by_block[key] if not event.done]
            if live:
                self._by_block[key] = live
            else:
                del self._by_block[key]


class Queue:
    """A single-worker, in-order queue for CUDA kernels and declared host work."""

    def __init__(self: Self, device: Device) -> None:
        self._device = device
        self._stream: Any = None
        if device.is_cuda:
            import torch

            self._stream = torch.cuda.Stream(device=device.backend.torch_device)  # type: ignore[attr-defined]
        self._jobs: SimpleQueue[_Job | None] = SimpleQueue()
        self._lock = threading.Lock()
        self._closed = False
        self._history: list[Event] = []
        self._numbers = itertools.count()
        self._ledger = _Ledger()
        self._worker = threading.Thread(target=self._serve, name="qpu-xla-submit", daemon=True)
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
        return self._closed

    # -- submission ----------------------------------------------------------------------

    def submit(
        self: Self,
        kernel: Kernel,
        args: tuple[Any, ...] = (),
        *,
        grid: tuple[int, int, int] = (1, 1, 1),
        wait_for: Iterable[Event] = (),
        buffers: Iterable[BufferAccess] = (),
    ) -> Event:
        """Queue a kernel launch; the returned event completes with its GPU work."""
        launch = LaunchConfig(tuple(grid))  # type: ignore[arg-type]
        backend, stream = self._device.backend, self._stream
        return self._admit(
            lambda: kernel.execute(backend, args, launch, stream), wait_for, buffers, kernel.name, "cuda", on_gpu=True
        )

    def host_task(
        self: Self,
        fn: Callable[[], None],
        *,
        wait_for: Iterable[Event] = (),
        buffers: Iterable[BufferAccess] = (),
        name: str | None = None,
    ) -> Event:
        """Queue host work, ordered after this queue's earlier work and ``wait_for``."""
        label = name if name is not None else str(getattr(fn, "__qualname__", "host_task"))
        return self._admit(fn, wait_for, buffers, label, "host", on_gpu=False)

    def _admit(
        self: Self, run: Callable[[], None], wait_for: Iterable[Event], buffers: Iterable[BufferAccess],
        name: str, category: str, *, on_gpu: bool,
    ) -> Event:
        accesses = tuple(buffers)
        if any(access.buffer.device is not self._device for access in accesses):
            raise DependencyError("a buffer access belongs to a different device")
        with self._lock:
            if self._closed:
                raise DeviceClosedError("queue is closed")
            dependencies = self._own_dependencies(wait_for)
            event = Event(self, sequence=next(self._numbers), name=name, category=category, dependencies=dependencies)
            self._history.append(event)
            self._ledger.prune()
            self._ledger.add(accesses, event)
            self._jobs.put(_Job(event, run, dependencies, on_gpu))
        return event

    def _own_dependencies(self: Self, wait_for: Iterable[Event]) -> tuple[Event, ...]:
        """The distinct events of ``wait_for``, each checked to come from this device."""
        unique: dict[int, Event] = {}
        for event in wait_for:
            if not isinstance(event, Event):
                raise DependencyError("wait_for must contain Event instances")
            if event.queue.device is not self._device:
                raise DependencyError("event dependency belongs to a different device")
            unique.setdefault(id(event), event)
        return tuple(unique.values())

    def hazards(self: Self, accesses: Iterable[BufferAccess]) -> list[Event]:
        """Unfinished events of this queue whose declared ranges conflict with ``accesses``."""
        with self._lock:
            return self._ledger.conflicts(tuple(accesses))

    # -- worker ----------------------------------------------------------------------

    def _serve(self: Self) -> None:
        while (job := self._jobs.get()) is not None:
            try:
                if job.event._begin():
                    (self._launch if job.on_gpu and self._stream is not None else self._run_on_host)(job)
            except BaseException as error:
                job.event._end(EventStatus.FAILED, error)

    def _run_on_host(self: Self, job: _Job) -> None:
        for dependency in job.dependencies:
            dependency.wait()
        if self._stream is not None:
            self._stream.synchronize()  # this queue's earlier kernels are complete
        job.run()
        job.event._end(EventStatus.SUCCEEDED, None)

    def _launch(self: Self, job: _Job) -> None:
        import torch

        stream = self._stream
        for dependency in job.dependencies:
            dependency._await_launch()
            marker = dependency.cuda_event
            if marker is None:
                dependency.wait()  # a host task: it must have finished
            else:
                stream.wait_event(marker)
        before, after = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            before.record(stream)
            job.run()
            after.record(stream)
        job.event._on_stream(before, after)

    def _raise_device_errors(self: Self) -> None:
        """Raise if a kernel on this device recorded an expired bounded wait (CUDA backend)."""
        backend = self._device.backend
        if getattr(backend, "kind", "") == "cuda" and self._stream is not None:
            backend.launch(self._stream, lambda native: native.synchronize())  # type: ignore[attr-defined]

    # -- completion and profiling ----------------------------------------------------------

    def finish(self: Self, timeout: float | None = None) -> None:
        """Wait for every submitted event; failures stay on their events, a timeout or cancel raises."""
        with self._lock:
            pending = list(self._history)
        for event in pending:
            try:
                event.wait(timeout)
            except (EventCancelledError, EventTimeoutError):
                raise
            except BaseException:
                pass

    def chrome_trace(self: Self) -> dict[str, list[dict[str, object]]]:
        """Chrome Trace Event payload: queue delay and execution slices, and a flow per dependency.

        Kernel slices last the GPU time measured between the CUDA events around the launch.
        """
        with self._lock:
            events = list(self._history)
        return {"traceEvents": list(_trace_records(events))}

    def write_chrome_trace(self: Self, path: str | PathLike[str]) -> None:
        with open(path, "w", encoding="utf-8") as trace_file:
            json.dump(self.chrome_trace(), trace_file, separators=(",", ":"))

    def consume_completed_event_counts(self: Self) -> dict[str, int]:
        """Count finished events per category and forget them (bounds profiling memory)."""
        with self._lock:
            finished = [event for event in self._history if event.done]
            self._history = [event for event in self._history if not event.done]
            self._ledger.prune()
        return dict(Counter(event.category for event in finished))

    # -- lifetime ----------------------------------------------------------------------

    def close(self: Self) -> None:
        """Stop accepting work and wait until everything submitted has finished."""
        with self._lock:
            if self._closed:
                return
            self._closed = True
        self._jobs.put(None)
        self._worker.join()
        if self._stream is not None:
            self._stream.synchronize()

    def __enter__(self: Self) -> Self:
        return self

    def __exit__(self: Self, exc_type: object, exc_value: object, traceback: object) -> None:
        self.close()


_PROCESS = "qpu-xla"


def _trace_records(events: list[Event]) -> Iterator[dict[str, object]]:
    """Complete ('X') slices for the wait in the queue and for the work of every started event,
    and a start/finish ('s'/'f') flow pair from each finished dependency to its dependent."""
    for event in events:
        started = event.started_ns
        if started is None:
            continue
        if started > event.submitted_ns:
            yield {"name": f"queue delay: {event.name}", "cat": "queue", "ph": "X", "pid": _PROCESS, "tid": "submission",
                   "ts": event.submitted_ns / 1e3, "dur": (started - event.submitted_ns) / 1e3,
                   "args": {"event": event._sequence}}
        finished = event.finished_ns
        if finished is not None:
            gpu_ms = event.device_milliseconds
            span_us = gpu_ms * 1e3 if gpu_ms is not None else max(0, finished - started) / 1e3
            yield {"name": event.name, "cat": event.category, "ph": "X", "pid": _PROCESS, "tid": event.category,
                   "ts": started / 1e3, "dur": span_us, "args": {"event": event._sequence, "status": event.status.value}}
        for dependency in event._dependencies:
            ready = dependency.finished_ns
            if ready is None:
                continue
            link = f"{dependency._sequence}->{event._sequence}"
            yield {"name": "dependency", "cat": "sync", "ph": "s", "pid": _PROCESS, "tid": dependency.category,
                   "ts": ready / 1e3, "id": link}
            yield {"name": "dependency", "cat": "sync", "ph": "f", "pid": _PROCESS, "tid": event.category,
                   "ts": started / 1e3, "id": link}


__all__ = ["Event", "EventStatus", "Queue"]
