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


def test_static_scratch_linear_matches_the_prepared_linear_twice_in_a_row() -> None:
    import torch

    from gpu_helpers import Native, padded_int8

    native = Native()
    try:
        k, n = 2048, 768
        case = workloads.linear_inputs(1, k, n, seed=41, weight_std=0.02, bias=True)
        values, scales = oracle.quantize_per_output_channel_int8(case.weight)
        weight = padded_int8(values)
        weight_scales = torch.from_numpy(scales).cuda()
        bias = torch.from_numpy(case.bias).cuda()
        plan = native.w8a8_prepare(values, scales, case.bias, max_batch=512)
        try:
            for rows, seed in ((384, 42), (200, 43), (5, 44)):
                source = torch.from_numpy(np.random.default_rng(seed).standard_normal((rows, k), dtype=np.float32)).cuda()
                expected = torch.full((rows, n), float("nan"), dtype=torch.float32, device="cuda")
                actual = torch.full((rows, n), float("nan"), dtype=torch.float32, device="cuda")
                native.context.set_stream(torch.cuda.current_stream().cuda_stream)
                native.context.check(
                    native.lib.qpucuda_w8a8_linear_execute_device(
                        plan, source.data_ptr(), source.stride(0), rows, expected.data_ptr(), expected.stride(0)
                    ),
                    "qpucuda_w8a8_linear_execute_device",
                )
                native.check(
                    "qpucuda_w8a8_linear_execute_static",
                    source.data_ptr(), source.stride(0), rows, weight.data_ptr(), weight.stride(0),
                    weight_scales.data_ptr(), bias.data_ptr(), k, n, actual.data_ptr(), actual.stride(0),
                )
                native.sync()
                np.testing.assert_array_equal(actual.cpu().numpy(), expected.cpu().numpy())
        finally:
            native.lib.qpucuda_w8a8_linear_destroy(plan)
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
