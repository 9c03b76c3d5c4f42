"""The GGML MUL_MAT offload on the GPU (include/qpucuda_ggml.h): the node-level work of the
reference's llama.cpp backend (integrations/llama_cpp/backend/ggml-qpu.cpp:319-360, 539-620)
against the oracle, its weight cache, CPU_REPACK weights and its failure paths."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

from oracle import qpu_oracle as oracle
from qpu_xla import Device, _native
from qpu_xla.ggml import GgmlMulMatBackend, ggml_tensor_view

pytestmark = pytest.mark.gpu

Q4_0_TOLERANCE = 1e-4  # rows <= 4 (matvec: per-lane partial sums added in a tree)


def _inputs(rows: int, k: int, n: int, seed: int) -> tuple[np.ndarray, np.ndarray]:
    rng = np.random.default_rng(seed)
    activation = rng.standard_normal((rows, k)).astype(np.float32)
    weight = oracle.quantize_q4_0((rng.standard_normal((n, k)) * 0.02).astype(np.float32))
    return activation, weight


def _expected(activation: np.ndarray, weight: np.ndarray) -> np.ndarray:
    """compute_q4_0_mul_mat: quantize_row_q8_0 of each row, then the Q4_0 x Q8_0 linear."""
    q8 = oracle.quantize_q8_0(activation)
    if activation.shape[0] > 4:
        return oracle.q4_0_q8_0_linear_mx(q8, weight)  # the reference's MX program arithmetic
    return oracle.q4_0_q8_0_linear(q8, weight)


@pytest.mark.parametrize("rows", (1, 4, 16, 37))
def test_mul_mat_matches_the_reference(cuda_device: Device, rows: int) -> None:
    from gpu_helpers import max_relative_error

    activation, weight = _inputs(rows, 1024, 272, seed=rows)
    with GgmlMulMatBackend(cuda_device) as backend:
        got = backend.mul_mat(weight, activation)
        assert backend.stats["rows"] == rows and backend.stats["dispatch_count"] == 1
    expected = _expected(activation, weight)
    if rows > 4:
        np.testing.assert_array_equal(got, expected)
    else:
        assert max_relative_error(got, expected) <= Q4_0_TOLERANCE


def test_weight_cache_follows_get_or_prepare_linear(cuda_device: Device) -> None:
    activation, weight = _inputs(4, 512, 64, seed=5)
    with GgmlMulMatBackend(cuda_device) as backend:
        one = backend.mul_mat(weight, activation[:1])
        assert (backend.stats["weight_cache_misses"], backend.stats["weight_cache_hits"]) == (1, 0)
        np.testing.assert_array_equal(backend.mul_mat(weight, activation[:1]), one)
        assert (backend.stats["weight_cache_misses"], backend.stats["weight_cache_hits"]) == (1, 1)
        four = backend.mul_mat(weight, activation)  # more rows than the cached plan: re-prepared
        assert (backend.stats["weight_cache_misses"], backend.stats["weight_cache_hits"]) == (2, 1)
        np.testing.assert_array_equal(four[:1], one)
        backend.mul_mat(weight, activation[:2])  # fewer rows: the 4-row plan serves it
        assert (backend.stats["weight_cache_misses"], backend.stats["weight_cache_hits"]) == (2, 2)
        backend.forget(weight.ctypes.data)
        backend.mul_mat(weight, activation[:2])
        assert backend.stats["weight_cache_misses"] == 3
        assert backend.stats["dispatch_count"] == 5
        # the same cache key on another weight (a tensor reallocated at a reused address): a new plan
        other = oracle.quantize_q4_0(np.random.default_rng(6).standard_normal((64, 512)).astype(np.float32) * 0.02)
        got = backend.mul_mat(other, activation[:2], identity=weight.ctypes.data)
        assert backend.stats["weight_cache_misses"] == 4
        from gpu_helpers import max_relative_error

        assert max_relative_error(got, _expected(activation[:2], other)) <= Q4_0_TOLERANCE


def test_cpu_repack_weights(cuda_device: Device) -> None:
    activation, weight = _inputs(8, 768, 96, seed=8)
    packed = oracle.pack_q4_0x4(weight)
    with GgmlMulMatBackend(cuda_device) as backend:
        native = backend.mul_mat(weight, activation)
        repacked = backend.mul_mat(packed, activation, cpu_repack=True, output_columns=96)
    np.testing.assert_array_equal(repacked, native)
    np.testing.assert_array_equal(native, _expected(activation, weight))


def test_unsupported_node_and_failure_paths() -> None:
    """Unsupported nodes are refused before any work; an injected wait failure returns TIMEOUT,
    leaves the destination as it was and poisons the context (a private one)."""
    from gpu_helpers import Native

    native = Native()
    backend = ctypes.c_void_p()
    try:
        lib = native.lib
        assert lib.qpucuda_ggml_backend_create(native.handle, 1, 8, ctypes.byref(backend)) == _native.Status.OK
        activation, weight = _inputs(2, 256, 32, seed=2)
        destination = np.full((2, 32), -777.0, dtype=np.float32)
        views = [
            ggml_tensor_view(weight, _native.GGML_TYPE_Q4_0),
            ggml_tensor_view(activation, _native.GGML_TYPE_F32),
            ggml_tensor_view(destination, _native.GGML_TYPE_F32),
        ]
        native.context.set_stream(lib.qpucuda_context_library_stream(native.handle))

        def run() -> int:
            return int(lib.qpucuda_ggml_mul_mat(backend, *(ctypes.byref(v) for v in views)))

        views[0].ne[0] = 48  # K % 32 != 0
        assert run() == _native.Status.INVALID_ARGUMENT
        views[0].ne[0] = 256
        assert np.all(destination == -777.0)
        native.context.set_failure_mask(int(_native.FailurePoint.ALLOCATION))
        assert run() == _native.Status.ALLOCATION_FAILED
        native.context.set_failure_mask(int(_native.FailurePoint.WAIT))
        assert run() == _native.Status.TIMEOUT
        assert np.all(destination == -777.0), "wait failure exposed partial output"
        native.context.set_failure_mask(0)
        assert native.context.poisoned
        assert run() == _native.Status.IO_FAILED
    finally:
        lib.qpucuda_ggml_backend_destroy(backend)
        native.close()
