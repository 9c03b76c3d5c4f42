"""ctypes binding of libqpucuda.so (the CUDA kernels and C-ABI in ``include/``).

The library is built in-tree by ``qpu-xla-triton_b200/build_native.py`` and
loaded from ``qpu_xla/_native/libqpucuda.so``. There is no fallback: when the
library is missing every operator raises, so a silent CPU path can never stand
in for the CUDA one.
"""

from __future__ import annotations

import ctypes
import os
import threading
from ctypes import POINTER, Structure, c_char, c_char_p, c_int, c_int32, c_size_t, c_uint8, c_uint32, c_uint64, c_void_p
from enum import IntEnum
from pathlib import Path

from qpu_xla.errors import AllocationError, DependencyError, EventTimeoutError, NativeError

LIBRARY_PATH = Path(__file__).resolve().parent / "_native" / "libqpucuda.so"


class Status(IntEnum):
    """``qpucuda_status``, numbered as ``qpu_llama_status`` (qpu_llama_runtime.h:16-27)."""

    OK = 0
    INVALID_ARGUMENT = 1
    DEVICE_UNAVAILABLE = 2
    CAPABILITY_MISSING = 3
    ALLOCATION_FAILED = 4
    IO_FAILED = 5
    SUBMISSION_FAILED = 6
    TIMEOUT = 7
    HASH_MISMATCH = 8
    INTERNAL_ERROR = 9


class FailurePoint(IntEnum):
    """``qpucuda_failure_point`` (host-side fault injection bits, qpu_llama_runtime.h:29-36)."""

    NONE = 0
    DEVICE_OPEN = 1 << 0
    ALLOCATION = 1 << 1
    SUBMISSION = 1 << 2
    WAIT = 1 << 3
    SOURCE_HASH = 1 << 4


class ContextConfig(Structure):
    _fields_ = [("device_ordinal", c_int32), ("timeout_ns", c_uint64), ("failure_mask", c_uint32), ("stream", c_void_p)]


class Capabilities(Structure):
    _fields_ = [
        ("device_name", c_char * 128),
        ("device_ordinal", c_int32),
        ("compute_capability_major", c_int32),
        ("compute_capability_minor", c_int32),
        ("multiprocessor_count", c_int32),
        ("global_memory_bytes", c_uint64),
        ("l2_cache_bytes", c_uint64),
        ("supports_tcgen05", c_uint8),
    ]


class Q40LinearDesc(Structure):
    _fields_ = [
        ("weights", c_void_p),
        ("weight_size", c_size_t),
        ("input_columns", c_uint32),
        ("output_columns", c_uint32),
        ("rows", c_uint32),
        ("resident_column_start", c_uint32),
        ("resident_column_count", c_uint32),
        ("weight_mode", c_int),
        ("workgroups_per_supergroup", c_uint32),
        ("expected_source_hash", c_char_p),
    ]


class Q40Execution(Structure):
    _fields_ = [
        ("activation", c_void_p),
        ("activation_size", c_size_t),
        ("activation_offset", c_size_t),
        ("destination", c_void_p),
        ("destination_size", c_size_t),
        ("destination_offset", c_size_t),
        ("column_start", c_uint32),
        ("column_count", c_uint32),
        ("rows", c_uint32),
        ("activation_interleave", c_uint32),
    ]


class Q40Timing(Structure):
    _fields_ = [
        (name, c_uint64)
        for name in (
            "input_access_ns",
            "input_pack_ns",
            "input_sync_ns",
            "input_copy_ns",
            "submit_ns",
            "wait_ns",
            "submit_wait_ns",
            "output_sync_ns",
            "output_copy_ns",
            "complete_ns",
        )
    ]


class W8A8LinearDesc(Structure):
    _fields_ = [
        ("weight_values", c_void_p),
        ("weight_scales", c_void_p),
        ("bias", c_void_p),
        ("input_features", c_uint32),
        ("output_features", c_uint32),
        ("max_batch", c_uint32),
        ("resident_output_start", c_uint32),
        ("resident_output_count", c_uint32),
        ("memory", c_int),
    ]


class W8A8Execution(Structure):
    _fields_ = [
        ("source", c_void_p),
        ("source_size", c_size_t),
        ("destination", c_void_p),
        ("destination_size", c_size_t),
        ("rows", c_uint32),
    ]


class MatrixLayout(Structure):
    """``qpucuda_matrix_layout``: element (r, c) at (r // rows_per_batch) * batch_stride
    + (r % rows_per_batch) * row_stride + c * column_stride elements from the base."""

    _fields_ = [
        ("rows_per_batch", c_uint64),
        ("batch_stride", c_uint64),
        ("row_stride", c_uint64),
        ("column_stride", c_uint64),
    ]


class GgmlTensor(Structure):
    """``qpucuda_ggml_tensor``: the ggml_tensor fields the MUL_MAT offload reads."""

    _fields_ = [
        ("type", ctypes.c_int32),
        ("cpu_repack", ctypes.c_int32),
        ("ne", ctypes.c_int64 * 4),
        ("nb", c_size_t * 4),
        ("data", c_void_p),
        ("identity", c_void_p),
    ]


class GgmlStats(Structure):
    """``qpucuda_ggml_stats``."""

    _fields_ = [
        ("dispatch_count", c_uint64),
        ("weight_cache_hits", c_uint64),
        ("weight_cache_misses", c_uint64),
        ("input_copy_ns", c_uint64),
        ("submit_wait_ns", c_uint64),
        ("output_copy_ns", c_uint64),
        ("complete_ns", c_uint64),
        ("rows", c_uint32),
    ]


GGML_TYPE_F32 = 0
GGML_TYPE_Q4_0 = 2

MEMORY_HOST = 0
MEMORY_DEVICE = 1

_S = c_int  # qpucuda_status
_P = c_void_p

# name -> (restype, argtypes); every function declared in include/*.h.
SIGNATURES: dict[str, tuple[object, list[object]]] = {
    # qpucuda_runtime.h
    "qpucuda_context_create": (_S, [POINTER(ContextConfig), POINTER(c_void_p)]),
    "qpucuda_context_destroy": (None, [_P]),
    "qpucuda_context_last_error": (c_char_p, [_P]),
    "qpucuda_context_capabilities": (_S, [_P, POINTER(Capabilities)]),
    "qpucuda_context_set_failure_mask": (None, [_P, c_uint32]),
    "qpucuda_context_set_stream": (_S, [_P, _P]),
    "qpucuda_context_stream": (_P, [_P]),
    "qpucuda_context_library_stream": (_P, [_P]),
    "qpucuda_context_synchronize": (_S, [_P]),
    "qpucuda_context_poisoned": (c_int, [_P]),
    "qpucuda_context_probe_wait_expiry": (_S, [_P, c_uint64]),
    "qpucuda_status_string": (c_char_p, [c_int]),
    "qpucuda_build_info": (c_char_p, []),
    # qpucuda_kernels.h
    "qpucuda_quantize_rows_int8": (_S, [_P, _P, c_size_t, c_uint32, c_uint32, c_uint32, _P, c_size_t, _P]),
    "qpucuda_w8a8_gemm_s32": (_S, [_P, _P, c_size_t, _P, c_size_t, c_uint32, c_uint32, c_uint32, _P, c_size_t]),
    "qpucuda_w8a8_gemm_dequantize": (
        _S,
        [_P, _P, c_size_t, _P, c_size_t, c_uint32, c_uint32, c_uint32, _P, _P, _P, _P, c_size_t],
    ),
    "qpucuda_w8a8_dequantize": (_S, [_P, _P, c_size_t, c_uint32, c_uint32, _P, _P, _P, _P, c_size_t]),
    "qpucuda_w8a8_gemv": (
        _S,
        [_P, _P, c_size_t, _P, c_size_t, c_uint32, c_uint32, c_uint32, _P, c_size_t, _P, _P, _P, _P, c_size_t],
    ),
    "qpucuda_ggml_q4_0_q8_0_linear": (
        _S,
        [_P, _P, c_uint32, c_uint32, _P, c_uint32, _P, c_size_t, c_uint32, c_uint32, c_uint32],
    ),
    "qpucuda_quantize_q8_0": (_S, [_P, _P, c_size_t, c_uint32, c_uint32, _P]),
    "qpucuda_quantize_q4_0": (_S, [_P, _P, c_size_t, c_uint32, c_uint32, _P]),
    "qpucuda_im2col_nchw_f32": (_S, [_P, _P] + [c_uint32] * 14 + [_P, c_size_t]),
    # qpucuda_w8a8.h
    "qpucuda_w8a8_linear_prepare": (_S, [_P, POINTER(W8A8LinearDesc), POINTER(c_void_p)]),
    "qpucuda_w8a8_linear_destroy": (None, [_P]),
    "qpucuda_w8a8_linear_resident_bytes": (c_size_t, [_P]),
    "qpucuda_w8a8_linear_execute": (_S, [_P, POINTER(W8A8Execution)]),
    "qpucuda_w8a8_linear_execute_direct": (_S, [_P, POINTER(W8A8Execution)]),
    "qpucuda_w8a8_linear_submit_direct": (_S, [_P, POINTER(W8A8Execution), POINTER(c_void_p)]),
    "qpucuda_w8a8_submission_wait": (_S, [_P]),
    "qpucuda_w8a8_submission_destroy": (None, [_P]),
    "qpucuda_w8a8_linear_execute_device": (_S, [_P, _P, c_size_t, c_uint32, _P, c_size_t]),
    "qpucuda_w8a8_linear_execute_prepared_device": (_S, [_P, _P, c_size_t, _P, c_uint32, _P, c_size_t]),
    "qpucuda_w8a8_linear_execute_device_layout": (_S, [_P, _P, POINTER(MatrixLayout), c_uint32, _P, POINTER(MatrixLayout)]),
    "qpucuda_w8a8_linear_scratch": (_S, [_P, POINTER(c_void_p), POINTER(c_size_t), POINTER(c_void_p)]),
    "qpucuda_w8a8_linear_execute_static": (
        _S,
        [_P, _P, c_size_t, c_uint32, _P, c_size_t, _P, _P, c_uint32, c_uint32, _P, c_size_t],
    ),
    # qpucuda_peer.h
    "qpucuda_peer_buffer_create": (_S, [_P, c_size_t, POINTER(c_void_p), c_char_p]),
    "qpucuda_peer_buffer_open": (_S, [_P, c_char_p, POINTER(c_void_p)]),
    "qpucuda_peer_buffer_close": (_S, [_P, _P]),
    "qpucuda_peer_buffer_destroy": (_S, [_P, _P]),
    "qpucuda_w8a8_linear_execute_device_fanout": (_S, [_P, _P, c_size_t, c_uint32, _P, POINTER(c_void_p), c_uint32, c_size_t]),
    "qpucuda_peer_copy_rows": (_S, [_P, _P, c_size_t, _P, c_size_t, c_size_t, c_size_t, _P]),
    # qpucuda_q4_0.h
    "qpucuda_q4_0_linear_prepare": (_S, [_P, POINTER(Q40LinearDesc), POINTER(c_void_p)]),
    "qpucuda_q4_0_linear_destroy": (None, [_P]),
    "qpucuda_q4_0_linear_execute": (_S, [_P, POINTER(Q40Execution), POINTER(Q40Timing)]),
    "qpucuda_q4_0_linear_submit": (_S, [_P, POINTER(Q40Execution), POINTER(c_void_p)]),
    "qpucuda_q4_0_submission_wait": (_S, [_P, POINTER(Q40Timing)]),
    "qpucuda_q4_0_submission_cpu_fallback": (_S, [_P]),
    "qpucuda_q4_0_submission_destroy": (None, [_P]),
    "qpucuda_q4_0_linear_resident_bytes": (c_size_t, [_P]),
    "qpucuda_q4_0_linear_execute_device": (_S, [_P, _P, c_uint32, _P, c_size_t, c_uint32, c_uint32, c_uint32]),
    "qpucuda_q4_0_linear_execute_f32_device": (
        _S,
        [_P, _P, c_size_t, c_uint32, _P, c_size_t, c_uint32, c_uint32, c_uint32],
    ),
    "qpucuda_q4_0_kernel_source_hash": (c_char_p, []),
    # qpucuda_ggml.h
    "qpucuda_ggml_supports_mul_mat": (
        c_int,
        [POINTER(GgmlTensor), POINTER(GgmlTensor), POINTER(GgmlTensor), c_uint32, c_uint32],
    ),
    "qpucuda_ggml_unpack_q4_0x4": (_S, [_P, c_size_t, c_uint32, c_uint32, _P, c_size_t]),
    "qpucuda_ggml_backend_create": (_S, [_P, c_uint32, c_uint32, POINTER(c_void_p)]),
    "qpucuda_ggml_backend_destroy": (None, [_P]),
    "qpucuda_ggml_mul_mat": (_S, [_P, POINTER(GgmlTensor), POINTER(GgmlTensor), POINTER(GgmlTensor)]),
    "qpucuda_ggml_backend_forget": (None, [_P, _P]),
    "qpucuda_ggml_backend_stats": (_S, [_P, POINTER(GgmlStats)]),
}

_LOCK = threading.Lock()
_LIBRARY: ctypes.CDLL | None = None


def library_path() -> Path:
    """Path of the native library (``QPU_XLA_NATIVE_LIB`` overrides the in-tree location)."""
    override = os.environ.get("QPU_XLA_NATIVE_LIB")
    return Path(override) if override else LIBRARY_PATH


def load() -> ctypes.CDLL:
    """Load libqpucuda.so once and declare every C signature; raise if it is absent."""
    global _LIBRARY
    with _LOCK:
        if _LIBRARY is not None:
            return _LIBRARY
        path = library_path()
        if not path.exists():
            raise NativeError(
                int(Status.CAPABILITY_MISSING),
                f"libqpucuda.so is not built at {path}; run qpu-xla-triton_b200/build_native.py "
                "(the CUDA path has no CPU fallback)",
            )
        library = ctypes.CDLL(str(path))
        for name, (restype, argtypes) in SIGNATURES.items():
            function = getattr(library, name)
            function.restype = restype
            function.argtypes = argtypes
        _LIBRARY = library
        return library


def status_string(status: int) -> str:
    return load().qpucuda_status_string(int(status)).decode()


def raise_for_status(status: int, context: int | None = None, what: str = "libqpucuda") -> None:
    """Translate a non-OK ``qpucuda_status`` into the runtime's exceptions."""
    if status == Status.OK:
        return
    library = load()
    detail = ""
    if context:
        raw = library.qpucuda_context_last_error(context)
        detail = raw.decode(errors="replace") if raw else ""
    message = f"{what}: {status_string(status)}" + (f" ({detail})" if detail else "")
    if status == Status.INVALID_ARGUMENT:
        raise ValueError(message)
    if status == Status.TIMEOUT:
        raise EventTimeoutError(message)
    if status == Status.ALLOCATION_FAILED:
        raise AllocationError(message)
    if status == Status.INTERNAL_ERROR and "in-flight" in detail:
        raise RuntimeError(message)
    if status == Status.DEVICE_UNAVAILABLE:
        raise DependencyError(message)
    raise NativeError(int(status), message)


class NativeContext:
    """One ``qpucuda_context``: a CUDA device, the stream work is issued on, failure mask and timeout."""

    def __init__(self, device_ordinal: int, *, timeout_ns: int = 0, failure_mask: int = 0, stream: int | None = None):
        self._library = load()
        config = ContextConfig(device_ordinal, timeout_ns, failure_mask, stream)
        handle = c_void_p()
        status = self._library.qpucuda_context_create(ctypes.byref(config), ctypes.byref(handle))
        raise_for_status(status, None, "qpucuda_context_create")
        self.handle: int = int(handle.value)  # type: ignore[arg-type]
        self.device_ordinal = device_ordinal
        self.lock = threading.RLock()
        self._closed = False

    @property
    def library(self) -> ctypes.CDLL:
        return self._library

    def check(self, status: int, what: str) -> None:
        raise_for_status(status, self.handle, what)

    def set_stream(self, stream: int | None) -> None:
        """Issue on ``stream`` (a cudaStream_t; 0/None is CUDA's legacy default stream)."""
        self.check(self._library.qpucuda_context_set_stream(self.handle, stream or None), "qpucuda_context_set_stream")

    def use_library_stream(self) -> None:
        """Issue on the library-owned non-blocking stream (the host-buffer entry points use it)."""
        self.set_stream(self._library.qpucuda_context_library_stream(self.handle))

    def set_failure_mask(self, mask: int) -> None:
        self._library.qpucuda_context_set_failure_mask(self.handle, int(mask))

    def synchronize(self) -> None:
        self.check(self._library.qpucuda_context_synchronize(self.handle), "qpucuda_context_synchronize")

    @property
    def poisoned(self) -> bool:
        return bool(self._library.qpucuda_context_poisoned(self.handle))

    def last_error(self) -> str:
        raw = self._library.qpucuda_context_last_error(self.handle)
        return raw.decode(errors="replace") if raw else ""

    def capabilities(self) -> Capabilities:
        result = Capabilities()
        self.check(self._library.qpucuda_context_capabilities(self.handle, ctypes.byref(result)), "capabilities")
        return result

    def close(self) -> None:
        if not self._closed:
            self._library.qpucuda_context_destroy(self.handle)
            self._closed = True

    def __del__(self) -> None:  # pragma: no cover - interpreter shutdown order
        try:
            self.close()
        except Exception:
            pass


def header_function_names(include_dir: Path) -> list[str]:
    """Every ``qpucuda_*`` function declared in ``include_dir/*.h`` (for the export check)."""
    import re

    names: list[str] = []
    pattern = re.compile(r"^[A-Za-z_][\w\s\*]*?\b(qpucuda_\w+)\s*\(", re.MULTILINE)
    for header in sorted(include_dir.glob("*.h")):
        text = re.sub(r"/\*.*?\*/", "", header.read_text(), flags=re.DOTALL)
        names.extend(match.group(1) for match in pattern.finditer(text))
    return sorted(set(names))


__all__ = [
    "Capabilities",
    "ContextConfig",
    "FailurePoint",
    "NativeContext",
    "Q40Execution",
    "Q40LinearDesc",
    "Q40Timing",
    "SIGNATURES",
    "Status",
    "W8A8Execution",
    "MatrixLayout",
    "W8A8LinearDesc",
    "header_function_names",
    "load",
    "raise_for_status",
]
