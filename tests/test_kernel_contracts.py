"""The kernel handles' ``supports_*`` predicates (gemm_int8.py:224-268, ggml_q4_0.py:725-761
contracts) on CPU: they return a bool and never raise, for tensors of a fake device (not CUDA) and
for arguments that are not tensors at all; a CUDA kernel submitted on a fake device fails its
event with ``KernelError`` instead of running anywhere else."""

from __future__ import annotations

import numpy as np
import pytest

from qpu_xla import Device, KernelError
from qpu_xla import kernels


def test_predicates_return_false_off_cuda_and_never_raise() -> None:
    with Device.fake() as device:
        q = device.tensor((16, 32), np.int8)
        w = device.tensor((48, 32), np.int8)
        acc = device.tensor((16, 48), np.int32)
        out = device.tensor((16, 48), np.float32)
        row = device.tensor((16,), np.float32)
        col = device.tensor((48,), np.float32)
        x = device.tensor((16, 32), np.float32)
        one = device.tensor((1, 32), np.int8)
        activation = device.tensor((4, 2, 34), np.uint8)
        blocks = device.tensor((32, 2, 18), np.uint8)
        q4_out = device.tensor((4, 32), np.float32)
        cases = [
            (kernels.supports_quantize_rows_int8, (x, q, row)),
            (kernels.supports_w8a8_gemm, (q, w, acc)),
            (kernels.supports_w8a8_gemm_dequantize, (q, w, row, col, out)),
            (kernels.supports_w8a8_dequantize, (acc, row, col, out)),
            (kernels.supports_w8a8_gemv, (one, w, device.tensor((1, 48), np.float32))),
            (kernels.supports_ggml_q4_0_q8_0_linear, (activation, blocks, q4_out, 0, 0, 32)),
        ]
        for predicate, args in cases:
            assert predicate(*args) is False, predicate.__name__
            garbage = tuple(None if not isinstance(a, int) else a for a in args)
            assert predicate(*garbage) is False, predicate.__name__


def test_cuda_kernels_fail_their_event_on_a_fake_device() -> None:
    with Device.fake() as device, device.queue() as queue:
        x = device.tensor((16, 32), np.float32)
        q = device.tensor((16, 32), np.int8)
        row = device.tensor((16,), np.float32)
        event = queue.submit(kernels.CUDA_QUANTIZE_ROWS_INT8_KERNEL, (x, q, row))
        with pytest.raises(KernelError):
            event.wait()
