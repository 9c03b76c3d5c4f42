"""The W8A8 linear entry point that allocates nothing, against the prepared linear.

``qpucuda_w8a8_linear_execute_static`` serves callers that cannot call
cudaMalloc while they run the operator (its activation scratch is a fixed
device array inside the library). Its output must equal the prepared linear's
(``qpucuda_w8a8_linear_execute_device``) bit for bit, the tolerance of every
W8A8 test here, on two calls in a row -- the second call finds the first call's
contents still in the shared array. This file is collected last on purpose.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

from oracle import qpu_oracle as oracle
from qpu_xla import _native, workloads

pytestmark = pytest.mark.gpu


def run_pair(native, plan: int, weight, weight_scales, bias, k: int, n: int, rows: int, seed: int):  # type: ignore[no-untyped-def]
    """One prepared-linear call and one no-allocation call on the same source; returns both outputs."""
    import torch

    source = torch.from_numpy(np.random.default_rng(seed).standard_normal((rows, k), dtype=np.float32)).cuda()
    expected = torch.full((rows, n), float("nan"), dtype=torch.float32, device="cuda")
    actual = torch.full((rows, n), float("nan"), dtype=torch.float32, device="cuda")
    native.context.set_stream(torch.cuda.current_stream().cuda_stream)
    native.context.check(
        native.lib.qpucuda_w8a8_linear_execute_device(plan, source.data_ptr(), source.stride(0), rows, expected.data_ptr(), expected.stride(0)),
        "qpucuda_w8a8_linear_execute_device",
    )
    native.check(
        "qpucuda_w8a8_linear_execute_static",
        source.data_ptr(), source.stride(0), rows, weight.data_ptr(), weight.stride(0),
        weight_scales.data_ptr(), bias.data_ptr(), k, n, actual.data_ptr(), actual.stride(0),
    )
    native.sync()
    return actual.cpu().numpy(), expected.cpu().numpy()


def test_static_scratch_linear_matches_the_prepared_linear_twice_in_a_row() -> None:
    """Rows 384 and 200 take the CTA-pair GEMM, 64 the single-CTA GEMM, 5 the GEMV; each call
    finds the previous call's contents in the shared array. A last call with a smaller K that is
    not a multiple of 16 (1000, padded to 1008) reads padding bytes that the earlier K = 2048
    calls left non-zero, so it also checks that the padding is rewritten."""
    import torch

    from gpu_helpers import Native, padded_int8

    native = Native()
    try:
        plans = []
        for k, n in ((2048, 768), (1000, 272)):
            case = workloads.linear_inputs(1, k, n, seed=41 + k, weight_std=0.02, bias=True)
            values, scales = oracle.quantize_per_output_channel_int8(case.weight)
            plans.append((k, n, padded_int8(values), torch.from_numpy(scales).cuda(), torch.from_numpy(case.bias).cuda(),
                          native.w8a8_prepare(values, scales, case.bias, max_batch=512)))
        try:
            calls = [(0, 384, 42), (0, 200, 43), (0, 64, 44), (0, 5, 45), (1, 300, 46)]
            for index, rows, seed in calls:
                k, n, weight, weight_scales, bias, plan = plans[index]
                actual, expected = run_pair(native, plan, weight, weight_scales, bias, k, n, rows, seed)
                np.testing.assert_array_equal(actual, expected)
        finally:
            for *_, plan in plans:
                native.lib.qpucuda_w8a8_linear_destroy(plan)
    finally:
        native.close()


def test_static_scratch_linear_allocates_nothing_after_its_set_up() -> None:
    """After the first call (the set-up: symbol lookup, every kernel loaded), further calls on the
    GEMM and GEMV paths leave the device's free memory exactly as it was."""
    import torch

    from gpu_helpers import Native, padded_int8

    native = Native()
    try:
        k, n = 2048, 512
        case = workloads.linear_inputs(1, k, n, seed=47, weight_std=0.02, bias=True)
        values, scales = oracle.quantize_per_output_channel_int8(case.weight)
        weight, weight_scales, bias = padded_int8(values), torch.from_numpy(scales).cuda(), torch.from_numpy(case.bias).cuda()
        sources = {rows: torch.randn((rows, k), dtype=torch.float32, device="cuda") for rows in (1, 96, 512)}
        outputs = {rows: torch.empty((rows, n), dtype=torch.float32, device="cuda") for rows in sources}

        def call(rows: int) -> None:
            native.check(
                "qpucuda_w8a8_linear_execute_static",
                sources[rows].data_ptr(), k, rows, weight.data_ptr(), weight.stride(0),
                weight_scales.data_ptr(), bias.data_ptr(), k, n, outputs[rows].data_ptr(), n,
            )

        call(1)  # the set-up call
        native.sync()
        torch.cuda.synchronize()
        free_before = torch.cuda.mem_get_info()[0]
        for rows in (512, 96, 1):  # paths the set-up call did not launch
            call(rows)
        native.sync()
        assert torch.cuda.mem_get_info()[0] == free_before
    finally:
        native.close()


def test_static_scratch_linear_rejects_batches_beyond_its_fixed_size() -> None:
    from gpu_helpers import Native

    native = Native()
    try:
        rows, k, n = 4096, 8192, 256  # 32 MiB of int8 activations > the 16 MiB array
        dummy = ctypes.c_void_p(256)  # never dereferenced: the size check comes first
        status = native.call(
            "qpucuda_w8a8_linear_execute_static", dummy, k, rows, dummy, k, dummy, None, k, n, dummy, n
        )
        assert status == _native.Status.INVALID_ARGUMENT
        assert "fixed" in native.context.last_error()
    finally:
        native.close()
