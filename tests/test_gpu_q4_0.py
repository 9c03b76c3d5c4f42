"""GGML Q4_0 x Q8_0 parity on the GPU through the C-ABI.

Tolerances: integer block dots are exact; the fp32 sum over blocks is reduced in
a different order than the reference's sequential sum, so outputs are held to
the reference's own test tolerance (rtol 2e-6, atol 2e-5 on its hardware-test
inputs, tests/test_qpu_xla_ggml_q4_0.py:80) and to the north-star bound of
1e-4 max-rel on the TinyLlama and Llama shapes. Codecs and quantizers are bit-exact.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

from oracle import qpu_oracle as oracle
from qpu_xla import _native, workloads

pytestmark = pytest.mark.gpu

Q4_0_TOLERANCE = 1e-4  # north-star bound, max-rel


@pytest.fixture(scope="module")
def native():  # type: ignore[no-untyped-def]
    from gpu_helpers import Native

    context = Native()
    yield context
    context.close()


def prepare(native, weights: np.ndarray, *, rows: int, start: int = 0, count: int | None = None, source_hash: bytes | None = None):  # type: ignore[no-untyped-def]
    weights = np.ascontiguousarray(weights)
    outputs, blocks, _ = weights.shape
    count = outputs - start if count is None else count
    desc = _native.Q40LinearDesc(
        weights.ctypes.data, weights.nbytes, blocks * 32, outputs, rows, start, count, 0, 0,
        source_hash if source_hash is not None else native.lib.qpucuda_q4_0_kernel_source_hash(),
    )
    handle = ctypes.c_void_p()
    status = native.call("qpucuda_q4_0_linear_prepare", ctypes.byref(desc), ctypes.byref(handle))
    return status, handle.value


def execute_host(native, handle, activation: np.ndarray, destination: np.ndarray, column_start: int, column_count: int, rows: int = 0, interleave: int = 0) -> int:  # type: ignore[no-untyped-def]
    execution = _native.Q40Execution(
        activation.ctypes.data, activation.nbytes, 0, destination.ctypes.data, destination.nbytes, 0,
        column_start, column_count, rows, interleave,
    )
    timing = _native.Q40Timing()
    return int(native.lib.qpucuda_q4_0_linear_execute(handle, ctypes.byref(execution), ctypes.byref(timing)))


def test_native_known_answer_test_and_fault_paths() -> None:
    """integrations/llama_cpp/tests/qpu_llama_q4_0_smoke.c:10-145 on the CUDA operator."""
    from gpu_helpers import Native
    from test_oracle_golden import native_kat_inputs

    native = Native()
    try:
        activation, weights, expected = native_kat_inputs()
        activation = np.ascontiguousarray(activation.reshape(34))
        status, handle = prepare(native, weights, rows=1, start=16, count=16, source_hash=b"0" * 64)
        assert status == _native.Status.HASH_MISMATCH and handle is None
        native.context.set_failure_mask(int(_native.FailurePoint.ALLOCATION))
        status, handle = prepare(native, weights, rows=1, start=16, count=16)
        native.context.set_failure_mask(0)
        assert status == _native.Status.ALLOCATION_FAILED and handle is None
        status, handle = prepare(native, weights, rows=1, start=16, count=16)
        assert status == _native.Status.OK
        destination = np.full(32, 123456.0, dtype=np.float32)
        assert execute_host(native, handle, activation, destination, 16, 16) == _native.Status.OK
        assert np.all(destination[:16] == 123456.0), "columns outside the window were modified"
        np.testing.assert_array_equal(destination[16:], expected[16:].astype(np.float32))
        destination[16:] = -777.0
        native.context.set_failure_mask(int(_native.FailurePoint.SUBMISSION))
        assert execute_host(native, handle, activation, destination, 16, 16) == _native.Status.SUBMISSION_FAILED
        native.context.set_failure_mask(0)
        assert np.all(destination[16:] == -777.0)
        native.context.set_failure_mask(int(_native.FailurePoint.WAIT))
        assert execute_host(native, handle, activation, destination, 16, 16) == _native.Status.TIMEOUT
        native.context.set_failure_mask(0)
        assert np.all(destination[16:] == -777.0), "wait failure exposed partial output"
        assert native.lib.qpucuda_q4_0_linear_resident_bytes(handle) > 0
        native.lib.qpucuda_q4_0_linear_destroy(handle)
    finally:
        native.close()


def test_argument_rules_follow_the_reference(native) -> None:  # type: ignore[no-untyped-def]
    """qpu_llama_q4_0.c:205-225 and :465-495."""
    rng = np.random.default_rng(3)
    weights = oracle.quantize_q4_0(rng.standard_normal((64, 64), dtype=np.float32))
    status, _ = prepare(native, weights, rows=1, start=8, count=16)
    assert status == _native.Status.INVALID_ARGUMENT  # unaligned window
    status, _ = prepare(native, weights, rows=1, start=48, count=32)
    assert status == _native.Status.INVALID_ARGUMENT  # window past the matrix
    status, _ = prepare(native, weights, rows=4 * 65535 + 1)
    assert status == _native.Status.INVALID_ARGUMENT  # past the reference's row limit
    for mode in (1, 2):  # COLUMN_W8, ROWCOL_W8A8: re-quantized modes are not built
        desc = _native.Q40LinearDesc(weights.ctypes.data, weights.nbytes, 64, 64, 16, 0, 64, mode, 0, native.lib.qpucuda_q4_0_kernel_source_hash())
        handle = ctypes.c_void_p()
        assert native.call("qpucuda_q4_0_linear_prepare", ctypes.byref(desc), ctypes.byref(handle)) == _native.Status.CAPABILITY_MISSING
    status, handle = prepare(native, weights, rows=4, start=16, count=32)
    assert status == _native.Status.OK
    activation = np.zeros((4, 2, 34), dtype=np.uint8)
    destination = np.zeros((4, 64), dtype=np.float32)
    assert execute_host(native, handle, activation, destination, 0, 16) == _native.Status.INVALID_ARGUMENT
    assert execute_host(native, handle, activation, destination, 16, 48) == _native.Status.INVALID_ARGUMENT
    assert execute_host(native, handle, activation, destination, 16, 16, rows=5) == _native.Status.INVALID_ARGUMENT
    assert execute_host(native, handle, activation, destination, 16, 16, interleave=2) == _native.Status.INVALID_ARGUMENT
    assert execute_host(native, handle, activation[:3], destination, 16, 16) == _native.Status.INVALID_ARGUMENT
    assert execute_host(native, handle, activation, destination, 16, 16) == _native.Status.OK
    submission = ctypes.c_void_p()
    execution = _native.Q40Execution(activation.ctypes.data, activation.nbytes, 0, destination.ctypes.data, destination.nbytes, 0, 16, 16, 0, 0)
    assert native.lib.qpucuda_q4_0_linear_submit(handle, ctypes.byref(execution), ctypes.byref(submission)) == _native.Status.OK
    second = ctypes.c_void_p()
    assert native.lib.qpucuda_q4_0_linear_submit(handle, ctypes.byref(execution), ctypes.byref(second)) == _native.Status.INTERNAL_ERROR
    assert native.lib.qpucuda_q4_0_submission_cpu_fallback(submission) == _native.Status.INVALID_ARGUMENT
    assert native.lib.qpucuda_q4_0_submission_wait(submission, None) == _native.Status.OK
    native.lib.qpucuda_q4_0_submission_destroy(submission)
    native.lib.qpucuda_q4_0_linear_destroy(handle)


def test_reference_hardware_test_inputs_and_sentinel(native, golden: dict) -> None:  # type: ignore[no-untyped-def]
    """tests/test_qpu_xla_ggml_q4_0.py:47-80 through the single-kernel entry point:
    weight columns [16, 32) into destination columns [16, 32); columns [0, 16) keep the sentinel."""
    import torch

    ref = golden["q4_0_reference"]
    activation = torch.from_numpy(ref["hw_activation"]).cuda()
    weight = torch.from_numpy(np.ascontiguousarray(ref["hw_weight"][16:])).cuda()
    destination = torch.full((4, 32), 123456.0, dtype=torch.float32, device="cuda")
    native.check("qpucuda_ggml_q4_0_q8_0_linear", activation.data_ptr(), 4, 5, weight.data_ptr(), 16, destination.data_ptr(), 32, 0, 16, 16)
    native.sync()
    actual = destination.cpu().numpy()
    np.testing.assert_array_equal(actual[:, :16], np.float32(123456.0))
    np.testing.assert_allclose(actual[:, 16:], ref["hw_expected"][:, 16:], rtol=2e-6, atol=2e-5)


@pytest.mark.parametrize("shape", workloads.TINYLLAMA_Q4_0_SHAPES, ids=lambda s: s.name)
@pytest.mark.parametrize("rows", (1, 4))
def test_tinyllama_ffn_matvec_matches_the_reference(native, shape, rows: int, golden: dict) -> None:  # type: ignore[no-untyped-def]
    import torch

    from gpu_helpers import max_relative_error

    ref = golden["q4_0_reference"]
    key = f"{shape.name}_m{rows}"
    source, weight = workloads.q4_0_case(shape, rows)
    weight_blocks = oracle.quantize_q4_0(weight)
    # quantizers on the GPU are bit-exact with the oracle
    np.testing.assert_array_equal(native.quantize_blocks(torch.from_numpy(source).cuda(), "q8_0").cpu().numpy(), ref[f"{key}_activation"])
    np.testing.assert_array_equal(native.quantize_blocks(torch.from_numpy(weight).cuda(), "q4_0").cpu().numpy(), weight_blocks)
    status, handle = prepare(native, weight_blocks, rows=rows)
    assert status == _native.Status.OK
    try:
        # host C-ABI path
        destination = np.full((rows, shape.out_features), np.nan, dtype=np.float32)
        assert execute_host(native, handle, ref[f"{key}_activation"], destination, 0, shape.out_features) == _native.Status.OK
        assert max_relative_error(destination, ref[f"{key}_expected"]) <= Q4_0_TOLERANCE
        np.testing.assert_allclose(destination, ref[f"{key}_expected"], rtol=1e-4, atol=1e-4 * float(np.abs(ref[f"{key}_expected"]).max()))
        # device path, fused fp32 -> Q8_0 -> matvec
        src = torch.from_numpy(source).cuda()
        out = torch.full((rows, shape.out_features), float("nan"), dtype=torch.float32, device="cuda")
        native.context.set_stream(torch.cuda.current_stream().cuda_stream)
        native.context.check(
            native.lib.qpucuda_q4_0_linear_execute_f32_device(handle, src.data_ptr(), src.stride(0), rows, out.data_ptr(), out.stride(0), 0, shape.out_features, 0),
            "execute_f32_device",
        )
        native.sync()
        np.testing.assert_array_equal(out.cpu().numpy(), destination)  # same kernel, same order
    finally:
        native.lib.qpucuda_q4_0_linear_destroy(handle)


def interleave_q8_0x4(native_blocks: np.ndarray, interleave: int) -> np.ndarray:
    """Rows 0..3 as CPU_REPACK block_q8_0x4 groups (the layout qpu_llama_q4_0.c:153-190 reads)."""
    rows, blocks, _ = native_blocks.shape
    assert rows == 4
    out = np.empty((blocks, 4 * 34), dtype=np.uint8)
    for block in range(blocks):
        group = out[block]
        for row in range(4):
            group[row * 2 : row * 2 + 2] = native_blocks[row, block, :2]
        values = group[8:]
        for row in range(4):
            for index in range(32):
                values[(index // interleave) * 4 * interleave + row * interleave + index % interleave] = native_blocks[row, block, 2 + index]
    return np.ascontiguousarray(out.reshape(1, blocks, 4 * 34))


@pytest.mark.parametrize("interleave", (4, 8))
def test_cpu_repack_interleaved_activations(native, interleave: int, golden: dict) -> None:  # type: ignore[no-untyped-def]
    ref = golden["q4_0_reference"]
    source, weight = workloads.q4_0_case(workloads.TINYLLAMA_Q4_0_SHAPES[0], 4)
    weight_blocks = oracle.quantize_q4_0(weight)
    activation = ref["ffn_up_m4_activation"]
    status, handle = prepare(native, weight_blocks, rows=4)
    assert status == _native.Status.OK
    try:
        plain = np.zeros((4, 5632), dtype=np.float32)
        assert execute_host(native, handle, activation, plain, 0, 5632) == _native.Status.OK
        packed = np.zeros((4, 5632), dtype=np.float32)
        assert execute_host(native, handle, interleave_q8_0x4(activation, interleave), packed, 0, 5632, interleave=interleave) == _native.Status.OK
        np.testing.assert_array_equal(packed, plain)
    finally:
        native.lib.qpucuda_q4_0_linear_destroy(handle)


@pytest.mark.parametrize(("k", "n"), [(20512, 96), (28672, 144)])
@pytest.mark.parametrize("rows", (1, 2, 3, 4))
def test_long_reductions_over_windows(native, k: int, n: int, rows: int) -> None:  # type: ignore[no-untyped-def]
    """Long reductions (641 and 896 blocks: the K-split kernel at M = 1, with a partial last trip
    at 641) over a resident window and an execution window inside it (both on the reference's
    16-column grid) written at an odd output offset; every written column is checked and the
    columns around the window stay untouched."""
    import torch

    from gpu_helpers import max_relative_error

    source, weight = workloads.torch_linear_inputs(rows, k, n, seed=11, weight_std=0.02, device="cuda")
    weight_blocks = native.quantize_blocks(weight, "q4_0").cpu().numpy()
    activation = native.quantize_blocks(source, "q8_0")
    start, count = 16, n - 32
    status, handle = prepare(native, weight_blocks, rows=4, start=start, count=count)
    assert status == _native.Status.OK
    try:
        column_start, column_count, out_start = start + 16, count - 16, 3
        out = torch.full((rows, out_start + column_count + 1), float("nan"), dtype=torch.float32, device="cuda")
        native.context.set_stream(torch.cuda.current_stream().cuda_stream)
        native.context.check(
            native.lib.qpucuda_q4_0_linear_execute_device(
                handle, activation.data_ptr(), rows, out.data_ptr(), out.shape[1], column_start, column_count, out_start
            ),
            "execute_device",
        )
        native.sync()
        got = out.cpu().numpy()
        expected = oracle.q4_0_q8_0_linear(activation.cpu().numpy(), weight_blocks[column_start : column_start + column_count])
        assert max_relative_error(got[:, out_start : out_start + column_count], expected) <= Q4_0_TOLERANCE
        assert np.isnan(got[:, :out_start]).all() and np.isnan(got[:, out_start + column_count :]).all()
        # fp32 rows quantized inside the kernel: bit-identical to quantize-then-execute, also from
        # rows whose stride is not a multiple of 4 floats (scalar loads)
        for pad in (0, 1):
            padded = torch.empty((rows, k + pad), dtype=torch.float32, device="cuda")
            padded[:, :k].copy_(source)
            fused = torch.full_like(out, float("nan"))
            native.context.check(
                native.lib.qpucuda_q4_0_linear_execute_f32_device(
                    handle, padded.data_ptr(), padded.stride(0), rows, fused.data_ptr(), fused.shape[1], column_start, column_count, out_start
                ),
                "execute_f32_device",
            )
            native.sync()
            np.testing.assert_array_equal(fused.cpu().numpy(), got)
    finally:
        native.lib.qpucuda_q4_0_linear_destroy(handle)


@pytest.mark.parametrize("shape", workloads.LLAMA2_70B_FFN + workloads.LLAMA2_7B_FFN, ids=lambda s: f"{s.name}_{s.in_features}x{s.out_features}")
def test_decode_full_size_columns_sample(native, shape) -> None:  # type: ignore[no-untyped-def]
    """M=1 decode at the 70B / 7B shapes: the full output is computed, a column sample is checked
    against the oracle (each output column depends only on its own weight row)."""
    import torch

    from gpu_helpers import max_relative_error

    source, weight = workloads.torch_linear_inputs(1, shape.in_features, shape.out_features, seed=5, weight_std=0.02, device="cuda")
    weight_blocks = native.quantize_blocks(weight, "q4_0").cpu().numpy()
    activation = native.quantize_blocks(source, "q8_0")
    status, handle = prepare(native, weight_blocks, rows=1)
    assert status == _native.Status.OK
    try:
        out = torch.empty((1, shape.out_features), dtype=torch.float32, device="cuda")
        native.context.set_stream(torch.cuda.current_stream().cuda_stream)
        native.context.check(
            native.lib.qpucuda_q4_0_linear_execute_device(handle, activation.data_ptr(), 1, out.data_ptr(), shape.out_features, 0, shape.out_features, 0),
            "execute_device",
        )
        native.sync()
        sample = np.sort(np.random.default_rng(1).choice(shape.out_features, 96, replace=False))
        expected = oracle.q4_0_q8_0_linear(activation.cpu().numpy(), weight_blocks[sample])
        assert max_relative_error(out.cpu().numpy()[:, sample], expected) <= Q4_0_TOLERANCE
    finally:
        native.lib.qpucuda_q4_0_linear_destroy(handle)


@pytest.mark.parametrize(
    "rows,k,n,start,count",
    [
        (5, 2048, 96, 16, 64),  # fewest MX rows, one partial 16-row tile
        (20, 2048, 256, 0, 256),  # a 32-row tile
        (64, 4128, 160, 0, 160),  # 129 blocks: a partial last K stage
        (100, 5632, 2048, 512, 1024),  # ragged rows, a column window
        (300, 8192, 384, 128, 256),  # several row tiles, a partial column tile
        (1000, 4096, 528, 16, 512),  # 8 row tiles of 128 (ragged last), 4 column tiles from column 16
        # calls that give the tcgen05 kernel a tile per SM (fewer go to the mma.sync kernel)
        (16, 1024, 19200, 0, 19200),  # 16-row tiles (two CTAs per SM)
        (30, 1024, 19456, 256, 19200),  # 32-row tiles, ragged rows, a column window
        (64, 2048, 19200, 0, 19200),  # 64-row tiles
        (300, 1056, 9600, 0, 9600),  # 128-row tiles, ragged rows, 33 blocks: a partial last K stage
    ],
)
def test_mx_rows_match_the_reference_program(native, rows: int, k: int, n: int, start: int, count: int) -> None:  # type: ignore[no-untyped-def]
    """Rows > 4 (the reference's MX path) on the tensor cores through every entry point: bit for bit
    against the reference program's arithmetic (oracle.q4_0_q8_0_linear_mx) and within the stated
    tolerance of ggml_q4_0_q8_0_reference (oracle.q4_0_q8_0_linear)."""
    import torch

    from gpu_helpers import max_relative_error

    source, weight = workloads.torch_linear_inputs(rows, k, n, seed=rows + k, weight_std=0.02, device="cuda")
    weight_blocks = native.quantize_blocks(weight, "q4_0").cpu().numpy()
    activation = native.quantize_blocks(source, "q8_0")
    activation_host = np.ascontiguousarray(activation.cpu().numpy())
    status, handle = prepare(native, weight_blocks, rows=rows, start=start, count=count)
    assert status == _native.Status.OK
    try:
        window = slice(start, start + count)
        expected = oracle.q4_0_q8_0_linear_mx(activation_host, weight_blocks[window])
        assert max_relative_error(expected, oracle.q4_0_q8_0_linear(activation_host, weight_blocks[window])) <= Q4_0_TOLERANCE
        native.context.set_stream(torch.cuda.current_stream().cuda_stream)
        device_out = torch.full((rows, count + 3), float("nan"), dtype=torch.float32, device="cuda")
        native.context.check(
            native.lib.qpucuda_q4_0_linear_execute_device(handle, activation.data_ptr(), rows, device_out.data_ptr(), count + 3, start, count, 2),
            "execute_device",
        )
        fused_out = torch.full((rows, count), float("nan"), dtype=torch.float32, device="cuda")
        native.context.check(
            native.lib.qpucuda_q4_0_linear_execute_f32_device(handle, source.data_ptr(), source.stride(0), rows, fused_out.data_ptr(), count, start, count, 0),
            "execute_f32_device",
        )
        native.sync()
        got = device_out.cpu().numpy()
        np.testing.assert_array_equal(got[:, 2 : 2 + count], expected)
        assert np.isnan(got[:, :2]).all() and np.isnan(got[:, 2 + count :]).all()
        np.testing.assert_array_equal(fused_out.cpu().numpy(), expected)
        host = np.full((rows, n), np.nan, dtype=np.float32)
        assert execute_host(native, handle, activation_host, host, start, count) == _native.Status.OK
        np.testing.assert_array_equal(host[:, window], expected)
        if rows % 4 == 0:
            grouped = np.concatenate([interleave_q8_0x4(activation_host[r : r + 4], 8) for r in range(0, rows, 4)], axis=0)
            packed = np.full((rows, n), np.nan, dtype=np.float32)
            assert execute_host(native, handle, grouped, packed, start, count, interleave=8) == _native.Status.OK
            np.testing.assert_array_equal(packed[:, window], expected)
        submission = ctypes.c_void_p()
        execution = _native.Q40Execution(activation_host.ctypes.data, activation_host.nbytes, 0, host.ctypes.data, host.nbytes, 0, start, count, rows, 0)
        assert native.lib.qpucuda_q4_0_linear_submit(handle, ctypes.byref(execution), ctypes.byref(submission)) == _native.Status.OK
        assert native.lib.qpucuda_q4_0_submission_cpu_fallback(submission) == _native.Status.CAPABILITY_MISSING
        assert native.lib.qpucuda_q4_0_submission_wait(submission, None) == _native.Status.OK
        native.lib.qpucuda_q4_0_submission_destroy(submission)
    finally:
        native.lib.qpucuda_q4_0_linear_destroy(handle)
