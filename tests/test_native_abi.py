"""libqpucuda.so loads on any host and exports every function include/*.h declares.

No kernel is launched here: calls either reject their arguments before touching
CUDA or, without a GPU, report QPUCUDA_DEVICE_UNAVAILABLE.
"""

from __future__ import annotations

import ctypes

import pytest

from conftest import REPO, cuda_available
from qpu_xla import _native


def test_library_is_built_in_tree() -> None:
    assert _native.library_path().exists(), "run qpu-xla-triton_b200/build_native.py"
    assert _native.library_path().is_relative_to(REPO)


def test_every_declared_function_is_exported_and_bound() -> None:
    library = _native.load()
    declared = _native.header_function_names(REPO / "include")
    assert len(declared) >= 35
    missing = [name for name in declared if not hasattr(library, name)]
    assert missing == []
    assert sorted(_native.SIGNATURES) == declared


def test_status_strings_follow_the_reference_numbering() -> None:
    expected = {
        0: "ok",
        1: "invalid argument",
        2: "device unavailable",
        3: "capability missing",
        4: "allocation failed",
        5: "I/O failed",
        6: "submission failed",
        7: "timeout",
        8: "hash mismatch",
        9: "internal error",
    }
    for status, text in expected.items():
        assert _native.status_string(status) == text
    assert _native.load().qpucuda_build_info().decode().endswith("sm_100a")


def test_null_arguments_are_rejected_without_a_device() -> None:
    library = _native.load()
    handle = ctypes.c_void_p()
    assert library.qpucuda_context_create(None, None) == _native.Status.INVALID_ARGUMENT
    assert library.qpucuda_q4_0_linear_prepare(None, None, ctypes.byref(handle)) == _native.Status.INVALID_ARGUMENT
    assert library.qpucuda_q4_0_linear_submit(None, None, ctypes.byref(handle)) == _native.Status.INVALID_ARGUMENT
    assert library.qpucuda_q4_0_submission_wait(None, None) == _native.Status.INVALID_ARGUMENT
    assert library.qpucuda_q4_0_submission_cpu_fallback(None) == _native.Status.INVALID_ARGUMENT
    assert library.qpucuda_w8a8_linear_prepare(None, None, ctypes.byref(handle)) == _native.Status.INVALID_ARGUMENT
    assert library.qpucuda_w8a8_linear_execute(None, None) == _native.Status.INVALID_ARGUMENT
    assert library.qpucuda_quantize_rows_int8(None, None, 0, 0, 0, 0, None, 0, None) == _native.Status.INVALID_ARGUMENT
    # NULL-safe destroys (qpu_llama_q4_0.c:449-459, :924-932).
    library.qpucuda_q4_0_linear_destroy(None)
    library.qpucuda_q4_0_submission_destroy(None)
    library.qpucuda_w8a8_linear_destroy(None)
    library.qpucuda_context_destroy(None)
    assert library.qpucuda_q4_0_linear_resident_bytes(None) == 0
    assert library.qpucuda_context_last_error(None) == b"no context"


@pytest.mark.skipif(cuda_available(), reason="checks the GPU-less path")
def test_context_reports_device_unavailable_without_a_gpu() -> None:
    library = _native.load()
    handle = ctypes.c_void_p()
    assert library.qpucuda_context_create(None, ctypes.byref(handle)) == _native.Status.DEVICE_UNAVAILABLE
    assert handle.value is None


def test_injected_device_open_failure_is_reported_before_any_cuda_call() -> None:
    library = _native.load()
    handle = ctypes.c_void_p()
    config = _native.ContextConfig(0, 0, int(_native.FailurePoint.DEVICE_OPEN), None)
    assert library.qpucuda_context_create(ctypes.byref(config), ctypes.byref(handle)) == _native.Status.DEVICE_UNAVAILABLE


def test_q4_0_kernel_source_hash_is_the_sha256_of_the_kernel_source() -> None:
    import hashlib

    csrc = REPO / "qpu-xla-triton_b200" / "csrc"
    sources = ("q4_0_gemv.cu", "q4_0_mx_sm100.cu")  # the kernels a prepared Q4_0 linear runs
    digest = hashlib.sha256(b"".join((csrc / name).read_bytes() for name in sources)).hexdigest()
    assert _native.load().qpucuda_q4_0_kernel_source_hash().decode() == digest
