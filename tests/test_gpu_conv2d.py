"""W8A8 convolution plan on the GPU (src/qpu_xla/ops/conv2d_w8a8.py:22-305).

Every case must equal the reference's per-group dynamic W8A8 convolution bit for bit: the
reference test's own inputs and outputs (tests/golden/conv2d_w8a8.npz, recorded from
tests/test_qpu_xla_conv2d_w8a8.py:14-130), then larger pointwise, strided, dilated, grouped and
depthwise cases against the oracle, with batches whose pixel count is not a multiple of 32 so
that warps straddle a batch boundary in the NCHW epilogue.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import qpu_oracle as oracle

pytestmark = pytest.mark.gpu


def run_plan(device, source: np.ndarray, weight: np.ndarray, *, stride: int | tuple[int, int], padding: int | tuple[int, int], dilation: int | tuple[int, int] = 1, groups: int = 1) -> np.ndarray:  # type: ignore[no-untyped-def]
    from qpu_xla.conv2d_w8a8 import Conv2dW8A8Plan

    with device.queue() as queue, Conv2dW8A8Plan(device, source_shape=source.shape, weight=weight, stride=stride, padding=padding, dilation=dilation, groups=groups) as plan:
        src = device.tensor(source.shape, np.float32)
        src.write(source)
        dst = device.tensor(plan.destination_shape, np.float32)
        dst.write(np.full(plan.destination_shape, np.nan, dtype=np.float32))
        plan.execute(dst, src, queue=queue).wait()
        return np.array(dst.numpy(), copy=True)


def test_reference_cases(cuda_device, golden: dict) -> None:  # type: ignore[no-untyped-def]
    conv = golden["conv2d_w8a8"]
    for name in conv["case_names"]:
        stride, padding, groups = (int(v) for v in conv[f"{name}_params"])
        actual = run_plan(cuda_device, conv[f"{name}_source"], conv[f"{name}_weight"], stride=stride, padding=padding, groups=groups)
        np.testing.assert_array_equal(actual, conv[f"{name}_expected"], err_msg=str(name))


@pytest.mark.parametrize(
    "source_shape,weight_shape,stride,padding,dilation,groups",
    [
        ((2, 64, 15, 15), (128, 64, 1, 1), 1, 0, 1, 1),  # pointwise, NCHW pixels read in place
        ((3, 96, 7, 7), (192, 48, 1, 1), 1, 0, 1, 2),  # grouped pointwise, 49 pixels per image
        ((2, 16, 20, 18), (40, 16, 3, 3), 2, 2, 2, 1),  # strided, dilated, padded 3x3 via im2col
        ((1, 32, 9, 9), (32, 1, 3, 3), 1, 1, 1, 32),  # depthwise 3x3 as 32 per-group GEMMs
        ((4, 8, 6, 5), (24, 4, 2, 3), (1, 2), (0, 1), (2, 1), 2),  # rectangular everything
        ((1, 40, 33, 31), (300, 40, 1, 1), 1, 0, 1, 1),  # pointwise with > 256 output channels
    ],
)
def test_against_the_oracle(cuda_device, source_shape, weight_shape, stride, padding, dilation, groups) -> None:  # type: ignore[no-untyped-def]
    rng = np.random.default_rng(sum(source_shape) + sum(weight_shape))
    source = rng.standard_normal(source_shape, dtype=np.float32)
    weight = np.ascontiguousarray(rng.standard_normal(weight_shape, dtype=np.float32) * 0.1)
    pair = lambda v: (v, v) if isinstance(v, int) else v  # noqa: E731
    expected = oracle.conv2d_w8a8(source, weight, stride=pair(stride), padding=pair(padding), dilation=pair(dilation), groups=groups)
    actual = run_plan(cuda_device, source, weight, stride=stride, padding=padding, dilation=dilation, groups=groups)
    np.testing.assert_array_equal(actual, expected)


def test_plan_contract(cuda_device) -> None:  # type: ignore[no-untyped-def]
    from qpu_xla.conv2d_w8a8 import Conv2dW8A8Plan

    weight = np.ones((4, 2, 1, 1), dtype=np.float32)
    with pytest.raises(ValueError, match="channels do not align"):
        Conv2dW8A8Plan(cuda_device, source_shape=(1, 3, 4, 4), weight=weight, groups=2)
    with pytest.raises(ValueError, match="empty output"):
        Conv2dW8A8Plan(cuda_device, source_shape=(1, 4, 2, 2), weight=np.ones((4, 4, 3, 3), dtype=np.float32))
    with cuda_device.queue() as queue, Conv2dW8A8Plan(cuda_device, source_shape=(1, 4, 4, 4), weight=weight, groups=2) as plan:
        wrong = cuda_device.tensor((1, 4, 4, 5), np.float32)
        out = cuda_device.tensor(plan.destination_shape, np.float32)
        with pytest.raises(ValueError, match="planned topology"):
            plan.execute(out, wrong, queue=queue)
