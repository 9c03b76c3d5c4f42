"""Host-side rules of the merged W8A8 plan: stacking along the output channels and the argument
checks that run before any device work (no GPU needed)."""

from __future__ import annotations

import numpy as np
import pytest

from qpu_xla.quantization import MergedW8A8Linear, QuantizedMatrixInt8, concatenate_output_channels


def _weight(rows: int, cols: int, seed: int) -> QuantizedMatrixInt8:
    rng = np.random.default_rng(seed)
    values = rng.integers(-127, 128, size=(rows, cols), dtype=np.int8)
    scales = (rng.random(rows).astype(np.float32) + np.float32(0.5)) / np.float32(127.0)
    return QuantizedMatrixInt8(values, scales)


def test_concatenation_stacks_rows_and_keeps_each_scale() -> None:
    a, b, c = _weight(8, 32, 1), _weight(3, 32, 2), _weight(5, 32, 3)
    merged = concatenate_output_channels([a, b, c])
    assert merged.shape == (16, 32)
    np.testing.assert_array_equal(merged.values[8:11], b.values)
    np.testing.assert_array_equal(merged.scales[11:], c.scales)
    np.testing.assert_array_equal(merged.dequantize()[:8], a.dequantize())


def test_concatenation_rejects_mismatched_widths_and_empty_lists() -> None:
    with pytest.raises(ValueError, match="share the input width"):
        concatenate_output_channels([_weight(4, 32, 1), _weight(4, 48, 2)])
    with pytest.raises(ValueError, match="at least one"):
        concatenate_output_channels([])


def test_merged_plan_checks_biases_before_touching_the_device() -> None:
    weights = [_weight(4, 32, 1), _weight(2, 32, 2)]
    with pytest.raises(ValueError, match="every section or for none"):
        MergedW8A8Linear(None, weights, max_batch=4, biases=[np.zeros(4, np.float32), None])  # type: ignore[arg-type, list-item]
    with pytest.raises(ValueError, match="every section or for none"):
        MergedW8A8Linear(None, weights, max_batch=4, biases=[np.zeros(4, np.float32)])  # type: ignore[arg-type]
    with pytest.raises(ValueError, match="one fp32 value per output feature"):
        MergedW8A8Linear(None, weights, max_batch=4, biases=[np.zeros(4, np.float32), np.zeros(3, np.float32)])  # type: ignore[arg-type]
    with pytest.raises(ValueError, match="share the input width"):
        MergedW8A8Linear(None, [weights[0], _weight(2, 16, 3)], max_batch=4)  # type: ignore[arg-type]
