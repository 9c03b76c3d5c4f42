"""The W8A8 convolution plan's host-side geometry (src/qpu_xla/ops/conv2d.py:17-39, 82-90) on
CPU: output sizes against torch's own convolution and the oracle's im2col, the pointwise 1x1
condition and the parameter rules."""

from __future__ import annotations

import itertools

import numpy as np
import pytest

from oracle import qpu_oracle as oracle
from qpu_xla.conv2d_w8a8 import _pair, is_pointwise_1x1, output_hw


@pytest.mark.parametrize(
    "height,width,kernel,stride,padding,dilation",
    [
        (7, 5, (3, 3), (1, 1), (1, 1), (1, 1)),
        (9, 11, (3, 2), (2, 3), (0, 1), (1, 2)),
        (4, 4, (1, 1), (1, 1), (0, 0), (1, 1)),
        (16, 8, (5, 5), (2, 2), (2, 2), (1, 1)),
        (6, 13, (2, 4), (3, 1), (1, 0), (2, 1)),
    ],
)
def test_output_size_matches_torch_and_the_oracle_im2col(height, width, kernel, stride, padding, dilation) -> None:  # type: ignore[no-untyped-def]
    import torch

    expected = torch.nn.functional.conv2d(
        torch.zeros(1, 1, height, width), torch.zeros(1, 1, *kernel), stride=stride, padding=padding, dilation=dilation
    ).shape[2:]
    assert output_hw(height, width, kernel[0], kernel[1], stride, padding, dilation) == tuple(expected)
    source = np.zeros((2, 3, height, width), dtype=np.float32)
    lowered = oracle.im2col_nchw(source, kernel, stride=stride, padding=padding, dilation=dilation)
    assert lowered.shape[0] == 2 * expected[0] * expected[1]


@pytest.mark.parametrize(
    "kernel,stride,padding,dilation",
    [((3, 3), (1, 1), (1, 1), (1, 1)), ((3, 2), (2, 3), (0, 1), (1, 2)), ((2, 4), (3, 1), (1, 0), (2, 1))],
)
def test_oracle_im2col_matches_torch_unfold(kernel, stride, padding, dilation) -> None:  # type: ignore[no-untyped-def]
    """The oracle's im2col (rows (b, oh, ow), columns (c, i, j), zeros in the padding) against
    torch's independent unfold, value for value."""
    import torch

    source = np.random.default_rng(3).standard_normal((2, 3, 9, 11)).astype(np.float32)
    unfolded = torch.nn.functional.unfold(torch.from_numpy(source), kernel, dilation=dilation, padding=padding, stride=stride)
    expected = unfolded.transpose(1, 2).reshape(-1, unfolded.shape[1]).numpy()
    np.testing.assert_array_equal(oracle.im2col_nchw(source, kernel, stride=stride, padding=padding, dilation=dilation), expected)


def test_empty_output_is_rejected() -> None:
    with pytest.raises(ValueError, match="empty output"):
        output_hw(2, 2, 3, 3, (1, 1), (0, 0), (1, 1))
    with pytest.raises(ValueError, match="empty output"):
        output_hw(5, 5, 3, 3, (1, 1), (0, 0), (3, 3))


def test_pointwise_condition() -> None:
    ones = ((1, 1), (1, 1), (0, 0), (1, 1))
    assert is_pointwise_1x1(1, 1, *ones[1:])
    for kernel, stride, padding, dilation in itertools.product(((1, 1), (1, 3), (3, 1)), ((1, 1), (2, 1)), ((0, 0), (0, 1)), ((1, 1), (1, 2))):
        expected = kernel == (1, 1) and stride == (1, 1) and padding == (0, 0) and dilation == (1, 1)
        assert is_pointwise_1x1(kernel[0], kernel[1], stride, padding, dilation) == expected


def test_parameter_pairs() -> None:
    assert _pair(2, name="stride") == (2, 2)
    assert _pair((1, 3), name="stride") == (1, 3)
    assert _pair(0, name="padding") == (0, 0)
    with pytest.raises(ValueError, match="padding"):
        _pair((1, -1), name="padding")
    with pytest.raises(ValueError, match="dilation"):
        _pair((1, 2, 3), name="dilation")  # type: ignore[arg-type]
