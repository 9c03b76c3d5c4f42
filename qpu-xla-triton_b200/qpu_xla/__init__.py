"""qpu_xla on NVIDIA B200: the reference's quantized-linear path on CUDA (sm_100a).

Drop-in surface of yiannisha/qpu-xla-triton's ``qpu_xla`` for one path:
``Device``/``Buffer``/``Tensor`` on CUDA memory, ``Queue``/``Event`` on CUDA
streams and events, the W8A8 plans (``PreparedW8A8Linear``,
``CalibratedW8A8Linear``, ``quantize_per_output_channel_int8``), the GGML
Q4_0 x Q8_0 operator (``PreparedQ4_0Linear``), the ``cuda`` placement, and the
output-channel split across GPUs (``ShardedW8A8Linear``, ``ShardedQ4_0Linear``).
Import paths that were ``qpu_xla.models.tinyllama.quantization`` in the
reference are ``qpu_xla.quantization`` here; ``qpu_xla.kernels.ggml_q4_0`` and
``qpu_xla.kernels.gemm_int8`` map to ``qpu_xla.ggml`` and ``qpu_xla.kernels``.
"""

from qpu_xla.device import Device
from qpu_xla.errors import (
    AllocationError,
    BufferClosedError,
    DependencyError,
    DeviceClosedError,
    EventCancelledError,
    EventTimeoutError,
    KernelError,
    NativeError,
    QpuXlaError,
)
from qpu_xla.kernel import Kernel, LaunchConfig
from qpu_xla.memory import AccessMode, Buffer, BufferAccess, Tensor
from qpu_xla.placement import Placement
from qpu_xla.queue import Event, EventStatus, Queue

__version__ = "0.1.0"

__all__ = [
    "AccessMode",
    "AllocationError",
    "Buffer",
    "BufferAccess",
    "BufferClosedError",
    "DependencyError",
    "Device",
    "DeviceClosedError",
    "Event",
    "EventCancelledError",
    "EventStatus",
    "EventTimeoutError",
    "Kernel",
    "KernelError",
    "LaunchConfig",
    "NativeError",
    "Placement",
    "QpuXlaError",
    "Queue",
    "Tensor",
]
