"""Exception hierarchy of the runtime; names and meanings follow src/qpu_xla/errors.py:1-37."""


class QpuXlaError(Exception):
    """Base class for all runtime failures."""


class DeviceClosedError(QpuXlaError):
    """An operation was attempted after its device was closed."""


class BufferClosedError(QpuXlaError):
    """An operation was attempted on a closed allocation."""


class AllocationError(QpuXlaError):
    """A buffer allocation or layout is invalid."""


class DependencyError(QpuXlaError):
    """An event dependency, queue or device pairing cannot be accepted."""


class EventTimeoutError(QpuXlaError):
    """Waiting for an event exceeded the requested timeout."""


class EventCancelledError(QpuXlaError):
    """The awaited event was cancelled."""


class KernelError(QpuXlaError):
    """A kernel could not be launched or failed while executing."""


class NativeError(KernelError):
    """A call into libqpucuda returned a non-OK status.

    ``status`` is the integer ``qpucuda_status`` (the same numbering as the
    reference's ``qpu_llama_status``, integrations/llama_cpp/include/qpu_llama_runtime.h:16-27).
    """

    def __init__(self, status: int, message: str) -> None:
        super().__init__(message)
        self.status = status
