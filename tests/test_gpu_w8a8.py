"""W8A8 parity on the GPU: every kernel through the C-ABI against the reference-pinned oracle.

int8 activations and int32 accumulators must be bit-exact; fp32 outputs are
held to bit-exactness as well (the reference's own fused-dequant test demands
``assert_array_equal``, tests/test_qpu_xla_gemm_int8.py:92); the north-star
tolerance, max-rel <= 1e-5, is asserted alongside as the contract bound.
"""

from __future__ import annotations

import ctypes
import hashlib

import numpy as np
import pytest

from oracle import qpu_oracle as oracle
from qpu_xla import _native, workloads

pytestmark = pytest.mark.gpu

W8A8_TOLERANCE = 1e-5  # north-star bound on max-rel error after dequant


@pytest.fixture(scope="module")
def native():  # type: ignore[no-untyped-def]
    from gpu_helpers import Native

    context = Native()
    yield context
    context.close()


def sha256(array: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(array).tobytes()).hexdigest()


@pytest.mark.parametrize(
    "rows,cols,padded",
    [
        (64, 64, 64), (512, 512, 512), (17, 20, 32), (1, 2048, 2048), (2048, 5632, 5632), (3, 28672, 28672),
        (2, 40000, 40000), (5, 33, 48),
        # many rows: register-cached kernel up to ~14.5K columns, bulk-staged kernel above
        (297, 1024, 1040), (300, 16384, 16384), (600, 28672, 28688), (4096, 8192, 8192), (296, 14592, 14592),
        (2048, 2048, 2048), (100, 1500, 1504), (64, 996, 1008),
    ],
)
def test_row_quantizer_is_bit_exact(native, rows: int, cols: int, padded: int) -> None:  # type: ignore[no-untyped-def]
    import torch

    rng = np.random.default_rng(rows * 7 + cols)
    x = rng.standard_normal((rows, cols), dtype=np.float32)
    x[0, :3] = [0.0, 1e-9, -1e-9]
    if rows > 1:
        x[1] = 0.0  # all-zero row -> the 1/127 floor
    q, scales = native.quantize_rows(torch.from_numpy(x).cuda(), padded)
    expected_q, expected_scales = oracle.quantize_rows_int8(x)
    np.testing.assert_array_equal(scales.cpu().numpy(), expected_scales)
    q_host = q.cpu().numpy()
    np.testing.assert_array_equal(q_host[:, :cols], expected_q)
    assert np.all(q_host[:, cols:] == 0)


def test_bulk_row_quantizer_on_strided_rows_of_mixed_scale(native) -> None:  # type: ignore[no-untyped-def]
    """Bulk-staged kernel over a 16-byte aligned strided view, with rows that hit the clamp, the
    scale floor, exact halves and a negative maximum."""
    import torch

    rng = np.random.default_rng(17)
    rows, cols, stride = 400, 16384, 16388
    full = rng.standard_normal((rows, stride), dtype=np.float32)
    full *= rng.uniform(1e-4, 1e4, (rows, 1)).astype(np.float32)
    full[2, :cols] = 0.0
    full[3, :cols] = -5.0
    full[4, :cols] = np.arange(cols, dtype=np.float32) * np.float32(0.5) - np.float32(300.0)
    full[5, :cols] = np.float32(127.0) * (np.arange(cols, dtype=np.float32) % np.float32(255.0) - np.float32(127.0)) / np.float32(254.0)
    view = torch.from_numpy(full).cuda()[:, :cols]
    q, scales = native.quantize_rows(view, cols + 16)
    expected_q, expected_scales = oracle.quantize_rows_int8(np.ascontiguousarray(full[:, :cols]))
    np.testing.assert_array_equal(scales.cpu().numpy(), expected_scales)
    q_host = q.cpu().numpy()
    np.testing.assert_array_equal(q_host[:, :cols], expected_q)
    assert np.all(q_host[:, cols:] == 0)


def test_row_quantizer_strided_rows(native) -> None:  # type: ignore[no-untyped-def]
    import torch

    rng = np.random.default_rng(5)
    full = rng.standard_normal((6, 100), dtype=np.float32)
    view = torch.from_numpy(full).cuda()[:, 3:67]  # unaligned base, stride 100
    q, scales = native.quantize_rows(view, 64)
    expected_q, expected_scales = oracle.quantize_rows_int8(np.ascontiguousarray(full[:, 3:67]))
    np.testing.assert_array_equal(q.cpu().numpy(), expected_q)
    np.testing.assert_array_equal(scales.cpu().numpy(), expected_scales)


@pytest.mark.parametrize(
    "m,k,n",
    [(16, 16, 16), (32, 64, 32), (128, 128, 256), (300, 2048, 600), (1024, 1024, 1024), (129, 4096, 257), (4096, 512, 512)],
)
def test_gemm_int32_accumulators_are_exact(native, m: int, k: int, n: int) -> None:  # type: ignore[no-untyped-def]
    """tests/test_qpu_xla_gemm_int8.py:28-54 at the reference's shapes and beyond (ragged M, N)."""
    from gpu_helpers import padded_int8

    rng = np.random.default_rng(91 + k)
    left = rng.integers(-127, 128, size=(m, k), dtype=np.int8)
    right = rng.integers(-127, 128, size=(n, k), dtype=np.int8)
    acc = native.gemm_s32(padded_int8(left), padded_int8(right))
    np.testing.assert_array_equal(acc.cpu().numpy(), oracle.int8_accumulate(left, right))


def test_gemm_extreme_values_reach_the_int32_bound(native) -> None:  # type: ignore[no-untyped-def]
    from gpu_helpers import padded_int8

    k = 28672  # the largest reduction of the benchmark shapes: K * 127^2 < 2^31
    left = np.full((130, k), 127, dtype=np.int8)
    left[1::2] = -127
    right = np.full((260, k), -127, dtype=np.int8)
    acc = native.gemm_s32(padded_int8(left), padded_int8(right)).cpu().numpy()
    np.testing.assert_array_equal(acc, oracle.int8_accumulate(left, right))
    assert acc.min() == -k * 127 * 127


def test_gemm_rejects_overflowing_reductions(native) -> None:  # type: ignore[no-untyped-def]
    import torch

    k = 133168  # K * 127^2 > INT32_MAX (gemm_int8.py:298)
    a = torch.zeros((16, k), dtype=torch.int8, device="cuda")
    acc = torch.zeros((16, 16), dtype=torch.int32, device="cuda")
    status = native.call("qpucuda_w8a8_gemm_s32", a.data_ptr(), k, a.data_ptr(), k, 16, 16, k, acc.data_ptr(), 16)
    assert status == _native.Status.INVALID_ARGUMENT


def test_fused_dequant_matches_fp32_epilogue_bit_exactly(native) -> None:  # type: ignore[no-untyped-def]
    """tests/test_qpu_xla_gemm_int8.py:57-92 (32x64x48), then with bias and at larger shapes."""
    from gpu_helpers import padded_int8, to_cuda

    for (p, q, r), seed in (((32, 64, 48), 1765), ((640, 1024, 768), 3), ((200, 2048, 5632), 4)):
        rng = np.random.default_rng(seed)
        left = rng.integers(-127, 128, size=(p, q), dtype=np.int8)
        right = rng.integers(-127, 128, size=(r, q), dtype=np.int8)
        row_scales = rng.uniform(0.001, 0.1, size=p).astype(np.float32)
        col_scales = rng.uniform(0.001, 0.1, size=r).astype(np.float32)
        bias = rng.standard_normal(r).astype(np.float32)
        acc = oracle.int8_accumulate(left, right)
        out = native.gemm_dequantize(padded_int8(left), padded_int8(right), to_cuda(row_scales), to_cuda(col_scales)).cpu().numpy()
        np.testing.assert_array_equal(out, oracle.w8a8_dequantize(acc, row_scales, col_scales))
        out_bias = native.gemm_dequantize(padded_int8(left), padded_int8(right), to_cuda(row_scales), to_cuda(col_scales), to_cuda(bias)).cpu().numpy()
        np.testing.assert_array_equal(out_bias, oracle.w8a8_dequantize(acc, row_scales, col_scales, bias))


def test_standalone_dequantize_matches_epilogue(native) -> None:  # type: ignore[no-untyped-def]
    """tests/test_qpu_xla_w8a8_epilogue.py:13-36 (the reference allows 1e-6; this is bit-exact)."""
    from gpu_helpers import to_cuda

    rng = np.random.default_rng(13)
    acc = rng.integers(-(2**26), 2**26, size=(48, 80), dtype=np.int32)
    row_scales = rng.uniform(1e-3, 1e-1, size=48).astype(np.float32)
    col_scales = rng.uniform(1e-3, 1e-1, size=80).astype(np.float32)
    bias = rng.standard_normal(80).astype(np.float32)
    out = native.dequantize(to_cuda(acc), to_cuda(row_scales), to_cuda(col_scales), to_cuda(bias)).cpu().numpy()
    np.testing.assert_array_equal(out, oracle.w8a8_dequantize(acc, row_scales, col_scales, bias))


@pytest.mark.parametrize("k,n", [(16, 16), (512, 512), (1536, 512), (28672, 8192), (28672, 1024), (28672, 256), (4112, 16), (1040, 1000)])
@pytest.mark.parametrize("m", [1, 3, 5, 8])
def test_gemv_is_exact(native, m: int, k: int, n: int) -> None:  # type: ignore[no-untyped-def]
    """tests/test_qpu_xla_gemv_int8.py:13-33 shapes, plus M = 3, 8, the 70B down projection and
    narrower long-K matrices (its 8-GPU column shard and below); K = 4112 and 1040 leave the last
    K slice ragged, N = 1000 a partial 16-column group."""
    from gpu_helpers import padded_int8, to_cuda

    rng = np.random.default_rng(190 + k + m)
    source = rng.integers(-127, 128, size=(m, k), dtype=np.int8)
    weight = rng.integers(-127, 128, size=(n, k), dtype=np.int8)
    acc = native.gemv(padded_int8(source), padded_int8(weight)).cpu().numpy()
    expected = oracle.int8_accumulate(source, weight)
    np.testing.assert_array_equal(acc, expected)
    row_scales = rng.uniform(1e-3, 1e-1, size=m).astype(np.float32)
    col_scales = rng.uniform(1e-3, 1e-1, size=n).astype(np.float32)
    out = native.gemv(padded_int8(source), padded_int8(weight), to_cuda(row_scales), to_cuda(col_scales)).cpu().numpy()
    np.testing.assert_array_equal(out, oracle.w8a8_dequantize(expected, row_scales, col_scales))


def run_prepared(native, values, scales, bias, source, *, start=0, count=0):  # type: ignore[no-untyped-def]
    """prepare + device execute through the C-ABI; returns the fp32 output."""
    import torch

    rows = source.shape[0]
    handle = native.w8a8_prepare(values, scales, bias, max_batch=rows, start=start, count=count)
    try:
        columns = count if count else values.shape[0] - start
        src = torch.from_numpy(source).cuda()
        out = torch.full((rows, columns), float("nan"), dtype=torch.float32, device="cuda")
        native.context.set_stream(torch.cuda.current_stream().cuda_stream)
        status = native.lib.qpucuda_w8a8_linear_execute_device(handle, src.data_ptr(), src.stride(0), rows, out.data_ptr(), out.stride(0))
        native.context.check(status, "execute_device")
        native.sync()
        return out.cpu().numpy()
    finally:
        native.lib.qpucuda_w8a8_linear_destroy(handle)


@pytest.mark.parametrize("size", (64, 512))
def test_square_cases_match_the_reference_golden_output(native, size: int, golden: dict) -> None:  # type: ignore[no-untyped-def]
    ref = golden[f"w8a8_square_{size}"]
    case = workloads.square_case(size)
    out = run_prepared(native, ref["weight_values"], ref["weight_scales"], ref.get("bias"), case.source)
    np.testing.assert_array_equal(out, ref["output"])


@pytest.mark.parametrize("shape", workloads.TINYLLAMA_LAYER, ids=lambda s: s.name)
@pytest.mark.parametrize("tokens", workloads.TINYLLAMA_TOKENS)
def test_tinyllama_projections_match_the_reference(native, shape, tokens: int, golden: dict) -> None:  # type: ignore[no-untyped-def]
    case = workloads.tinyllama_case(shape, tokens)
    values, scales = oracle.quantize_per_output_channel_int8(case.weight)
    out = run_prepared(native, values, scales, None, case.source)
    if tokens in (1, 128):
        assert sha256(out) == str(golden["w8a8_tinyllama"][f"{shape.name}_m{tokens}_output"])
    else:
        expected = oracle.w8a8_linear(case.source, values, scales)
        np.testing.assert_array_equal(out, expected)


def test_reference_odd_shapes_and_decode_gemv(native) -> None:  # type: ignore[no-untyped-def]
    """tests/test_qpu_xla_quantization.py:167-183 (17x20 -> 19) and :349-367 (M=1, 512x512)."""
    for seed, (m, k, n) in ((731, (17, 20, 19)), (1731, (1, 512, 512)), (1907, (31, 20, 19))):
        rng = np.random.default_rng(seed)
        source = rng.standard_normal((m, k), dtype=np.float32)
        values, scales = oracle.quantize_per_output_channel_int8(rng.standard_normal((n, k), dtype=np.float32))
        out = run_prepared(native, values, scales, None, source)
        expected = oracle.w8a8_linear(source, values, scales)
        np.testing.assert_allclose(out, expected, atol=1e-6, rtol=1e-6)  # the reference's tolerance
        np.testing.assert_array_equal(out, expected)


@pytest.mark.parametrize(
    "k,n,max_batch,batches",
    [
        (4112, 1000, 128, (128, 17, 100)),  # one row block; 33 K stages: uneven slices
        (2064, 256, 512, (300, 512, 130, 9)),  # one column tile, several row blocks per slice
    ],
)
def test_split_k_batches_match_the_reference(native, k: int, n: int, max_batch: int, batches: tuple[int, ...]) -> None:  # type: ignore[no-untyped-def]
    """Batches whose output tiles leave most SMs idle run the GEMM in K slices into the plan's
    int32 workspace and add them in a second launch. One plan, several batch sizes in a row (later
    calls must not see an earlier call's partial rows), with bias: bit for bit against the oracle."""
    import torch

    rng = np.random.default_rng(5150 + n)
    values, scales = oracle.quantize_per_output_channel_int8(rng.standard_normal((n, k), dtype=np.float32) * 0.05)
    bias = rng.standard_normal(n, dtype=np.float32) * 0.1
    handle = native.w8a8_prepare(values, scales, bias, max_batch=max_batch)
    try:
        native.context.set_stream(torch.cuda.current_stream().cuda_stream)
        for rows in batches:
            source = rng.standard_normal((rows, k), dtype=np.float32)
            src = torch.from_numpy(source).cuda()
            out = torch.full((rows, n), float("nan"), dtype=torch.float32, device="cuda")
            status = native.lib.qpucuda_w8a8_linear_execute_device(handle, src.data_ptr(), src.stride(0), rows, out.data_ptr(), out.stride(0))
            native.context.check(status, "execute_device")
            native.sync()
            np.testing.assert_array_equal(out.cpu().numpy(), oracle.w8a8_linear(source, values, scales, bias))
    finally:
        native.lib.qpucuda_w8a8_linear_destroy(handle)


def test_resident_output_window_is_a_disjoint_column_split(native) -> None:  # type: ignore[no-untyped-def]
    """The reference's output split (execute_hybrid, quantization.py:350-514) as two resident windows."""
    case = workloads.linear_inputs(40, 96, 600, seed=21, weight_std=0.05, bias=True)
    values, scales = oracle.quantize_per_output_channel_int8(case.weight)
    expected = oracle.w8a8_linear(case.source, values, scales, case.bias)
    head = run_prepared(native, values, scales, case.bias, case.source, start=0, count=256)
    tail = run_prepared(native, values, scales, case.bias, case.source, start=256, count=344)
    np.testing.assert_array_equal(np.concatenate([head, tail], axis=1), expected)


@pytest.mark.parametrize("shape", workloads.LLAMA2_70B_FFN + workloads.LLAMA2_7B_FFN, ids=lambda s: f"{s.name}_{s.in_features}x{s.out_features}")
def test_sharded_case_full_size_rows_and_columns_sample(native, shape) -> None:  # type: ignore[no-untyped-def]
    """M=4096 at the 70B/7B FFN shapes. Rows are quantized independently, so any row
    subset of the full-size output must equal the oracle on those rows, bit for bit;
    the full int32 GEMM also gets a column checksum (sum over N of the output) check."""
    import torch

    rows = workloads.SHARDED_PREFILL_TOKENS
    source, weight = workloads.torch_linear_inputs(rows, shape.in_features, shape.out_features, seed=4, weight_std=0.02, device="cuda")
    values_t, scales_t = native.quantize_rows(weight)
    values, scales = values_t.cpu().numpy(), scales_t.cpu().numpy()
    handle = native.w8a8_prepare(values, scales, None, max_batch=rows)
    try:
        out = torch.empty((rows, shape.out_features), dtype=torch.float32, device="cuda")
        native.context.set_stream(torch.cuda.current_stream().cuda_stream)
        native.context.check(
            native.lib.qpucuda_w8a8_linear_execute_device(handle, source.data_ptr(), source.stride(0), rows, out.data_ptr(), out.stride(0)),
            "execute_device",
        )
        native.sync()
        sample = np.r_[0:3, 127:131, rows - 3 : rows, np.random.default_rng(0).choice(rows, 40, replace=False)]
        src_host = source[torch.from_numpy(sample).cuda()].cpu().numpy()
        expected = oracle.w8a8_linear(src_host, values, scales)
        np.testing.assert_array_equal(out[torch.from_numpy(sample).cuda()].cpu().numpy(), expected)
        assert torch.isfinite(out).all()
    finally:
        native.lib.qpucuda_w8a8_linear_destroy(handle)


@pytest.mark.parametrize("rows", (512, 2500), ids=("one-slice", "pipelined-slices"))
def test_host_buffer_execute_and_injected_failures(rows: int) -> None:
    """qpucuda_w8a8_linear_execute with host buffers; FAIL_SUBMISSION and FAIL_WAIT leave the
    destination untouched, and a failed wait poisons the context (qpu_llama_runtime.c:688-727).
    2500 rows take the pipelined path (row slices of 1024 on separate copy streams)."""
    from gpu_helpers import Native

    native = Native()
    try:
        case = workloads.square_case(512)
        values, scales = oracle.quantize_per_output_channel_int8(case.weight)
        source = np.ascontiguousarray(np.tile(case.source, ((rows + 511) // 512, 1))[:rows])
        source[512:] *= np.float32(1.5)
        handle = native.w8a8_prepare(values, scales, case.bias, max_batch=rows)
        destination = np.full((rows, 512), -777.0, dtype=np.float32)

        def execute() -> int:
            execution = _native.W8A8Execution(source.ctypes.data, source.nbytes, destination.ctypes.data, destination.nbytes, rows)
            return int(native.lib.qpucuda_w8a8_linear_execute(handle, ctypes.byref(execution)))

        assert execute() == _native.Status.OK
        np.testing.assert_array_equal(destination, oracle.w8a8_linear(source, values, scales, case.bias))
        destination[:] = -777.0
        native.context.set_failure_mask(int(_native.FailurePoint.SUBMISSION))
        assert execute() == _native.Status.SUBMISSION_FAILED
        assert np.all(destination == -777.0)
        native.context.set_failure_mask(int(_native.FailurePoint.WAIT))
        assert execute() == _native.Status.TIMEOUT
        assert np.all(destination == -777.0), "wait failure exposed partial output"
        native.context.set_failure_mask(0)
        assert native.context.poisoned
        assert execute() == _native.Status.IO_FAILED
        native.lib.qpucuda_w8a8_linear_destroy(handle)
    finally:
        native.close()


def test_injected_allocation_failure_leaves_no_plan() -> None:
    from gpu_helpers import Native

    native = Native()
    native.context.set_failure_mask(int(_native.FailurePoint.ALLOCATION))
    try:
        values = np.ones((32, 32), dtype=np.int8)
        scales = np.ones(32, dtype=np.float32)
        desc = _native.W8A8LinearDesc(values.ctypes.data, scales.ctypes.data, None, 32, 32, 4, 0, 0, _native.MEMORY_HOST)
        handle = ctypes.c_void_p()
        status = native.call("qpucuda_w8a8_linear_prepare", ctypes.byref(desc), ctypes.byref(handle))
        assert status == _native.Status.ALLOCATION_FAILED and handle.value is None
    finally:
        native.close()
