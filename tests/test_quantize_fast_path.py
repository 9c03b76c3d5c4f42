"""The row quantizer's division-free rounding rule, checked on the CPU in IEEE float32.

The CUDA row quantizer computes q = rint(x / scale) (quantization.py:156-171) as
rint(x * RN(1 / scale)) wherever that product lies farther than 2^-15 from a half-integer,
and with the IEEE division elsewhere. NumPy float32 arithmetic rounds to nearest like the
GPU's __fmul_rn / __frcp_rn / __fdiv_rn, so the rule can be checked here exhaustively on
inputs built to sit on, and just beside, every half-integer the clamp range can reach.
"""

from __future__ import annotations

import numpy as np

WINDOW = np.float32(0.5) - np.float32(2.0**-15)


def _check(x: np.ndarray, scale: np.float32) -> int:
    inverse = np.float32(1.0) / scale
    product = x * inverse
    fast = np.abs(product - np.rint(product)) <= WINDOW
    exact = np.rint(x / scale)
    assert np.array_equal(np.rint(product)[fast], exact[fast])
    return int(np.count_nonzero(~fast))


def test_reciprocal_product_rounds_like_the_division_outside_the_window() -> None:
    rng = np.random.default_rng(2024)
    fallbacks = 0
    total = 0
    for _ in range(200):
        amax = np.float32(rng.uniform(1e-3, 1e4))
        scale = max(amax / np.float32(127.0), np.float32(1.0 / 127.0))
        halves = np.arange(-127, 127, dtype=np.float32) + np.float32(0.5)
        # values at and within a few ulps of every half-integer quotient, plus random values
        near = (halves[:, None] * scale).astype(np.float32)
        offsets = np.arange(-8, 9, dtype=np.int32)
        bits = near.view(np.int32) + offsets[None, :]
        x = np.concatenate([bits.view(np.float32).ravel(), rng.uniform(-amax, amax, 4096).astype(np.float32)])
        x = x[np.abs(x) <= amax]
        fallbacks += _check(x, scale)
        total += x.size
    # the window catches the near-half inputs, and only those: random values almost never fall back
    assert 0 < fallbacks < total


def test_random_rows_fall_back_rarely() -> None:
    rng = np.random.default_rng(7)
    x = rng.standard_normal(1 << 20).astype(np.float32)
    scale = max(np.abs(x).max() / np.float32(127.0), np.float32(1.0 / 127.0))
    assert _check(x, np.float32(scale)) < x.size * 2e-4
