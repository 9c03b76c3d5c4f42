"""Projection shapes and seeded synthetic inputs of the quantized-linear path.

Shapes follow the reference's workload manifest (src/qpu_xla/workloads.py:108-123,
TinyLlama h2048 / kv 4x64 / inter 5632) and the Llama-2 7B / 70B FFN shapes of the
sharded case. No dataset is involved anywhere: every input is drawn from a
seeded ``numpy.random.default_rng`` (or ``torch.Generator`` for the large sharded
case) with the distributions the benchmark configurations state.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import numpy.typing as npt


@dataclass(frozen=True, slots=True)
class LinearShape:
    name: str
    in_features: int  # K
    out_features: int  # N


TINYLLAMA_LAYER: tuple[LinearShape, ...] = (
    LinearShape("q_proj", 2048, 2048),
    LinearShape("k_proj", 2048, 256),
    LinearShape("v_proj", 2048, 256),
    LinearShape("o_proj", 2048, 2048),
    LinearShape("gate_proj", 2048, 5632),
    LinearShape("up_proj", 2048, 5632),
    LinearShape("down_proj", 5632, 2048),
)
TINYLLAMA_TOKENS: tuple[int, ...] = (1, 128, 2048)

TINYLLAMA_Q4_0_SHAPES: tuple[LinearShape, ...] = (
    LinearShape("ffn_up", 2048, 5632),
    LinearShape("ffn_down", 5632, 2048),
)

LLAMA2_70B_FFN: tuple[LinearShape, ...] = (
    LinearShape("gate_proj", 8192, 28672),
    LinearShape("up_proj", 8192, 28672),
    LinearShape("down_proj", 28672, 8192),
)
LLAMA2_7B_FFN: tuple[LinearShape, ...] = (
    LinearShape("gate_proj", 4096, 11008),
    LinearShape("up_proj", 4096, 11008),
    LinearShape("down_proj", 11008, 4096),
)
SHARDED_PREFILL_TOKENS = 4096

# Seeds per configuration: 0 for the 64^3 case, then 1, 2, 3, ... in configuration order.
SEED_SQUARE_64 = 0
SEED_SQUARE_512 = 1
SEED_TINYLLAMA = 2
SEED_Q4_0 = 3
SEED_SHARDED = 4

WEIGHT_STD_SQUARE = 0.05
WEIGHT_STD_LLAMA = 0.02
BIAS_STD = 0.1


@dataclass(frozen=True, slots=True)
class LinearInputs:
    source: npt.NDArray[np.float32]
    weight: npt.NDArray[np.float32]
    bias: npt.NDArray[np.float32] | None


def linear_inputs(rows: int, in_features: int, out_features: int, *, seed: int, weight_std: float, bias: bool = False) -> LinearInputs:
    """Draw X ~ N(0, 1) [rows, K], then W ~ N(0, std) [N, K], then (optionally) b ~ N(0, 0.1) [N] from one generator."""
    rng = np.random.default_rng(seed)
    source = rng.standard_normal((rows, in_features), dtype=np.float32)
    weight = (rng.standard_normal((out_features, in_features), dtype=np.float32) * np.float32(weight_std)).astype(np.float32)
    bias_values = (rng.standard_normal(out_features, dtype=np.float32) * np.float32(BIAS_STD)).astype(np.float32) if bias else None
    return LinearInputs(source, weight, bias_values)


def square_case(size: int) -> LinearInputs:
    """The reference's square W8A8 cases: 64^3 without bias (seed 0), 512^3 with bias (seed 1)."""
    if size == 64:
        return linear_inputs(64, 64, 64, seed=SEED_SQUARE_64, weight_std=WEIGHT_STD_SQUARE, bias=False)
    if size == 512:
        return linear_inputs(512, 512, 512, seed=SEED_SQUARE_512, weight_std=WEIGHT_STD_SQUARE, bias=True)
    raise ValueError("square cases are 64 and 512")


def tinyllama_case(shape: LinearShape, tokens: int) -> LinearInputs:
    """One TinyLlama projection at ``tokens`` rows; the seed is derived from the config seed and the shape."""
    index = TINYLLAMA_LAYER.index(shape)
    return linear_inputs(tokens, shape.in_features, shape.out_features, seed=SEED_TINYLLAMA * 1000 + index * 10 + TINYLLAMA_TOKENS.index(tokens), weight_std=WEIGHT_STD_LLAMA)


def q4_0_case(shape: LinearShape, rows: int) -> tuple[npt.NDArray[np.float32], npt.NDArray[np.float32]]:
    """fp32 activations ~N(0,1) [rows, K] and weights ~N(0, 0.02) [N, K] for the Q4_0 x Q8_0 matvec."""
    index = TINYLLAMA_Q4_0_SHAPES.index(shape)
    inputs = linear_inputs(rows, shape.in_features, shape.out_features, seed=SEED_Q4_0 * 1000 + index * 10 + rows, weight_std=WEIGHT_STD_LLAMA)
    return inputs.source, inputs.weight


def torch_linear_inputs(rows: int, in_features: int, out_features: int, *, seed: int, weight_std: float, device: object) -> tuple[object, object]:
    """Large sharded case on the GPU: identical on every rank for the same seed (torch's CUDA generator)."""
    import torch

    generator = torch.Generator(device=device)
    generator.manual_seed(seed)
    source = torch.randn((rows, in_features), generator=generator, device=device, dtype=torch.float32)
    weight = torch.randn((out_features, in_features), generator=generator, device=device, dtype=torch.float32) * weight_std
    return source, weight


__all__ = [
    "LLAMA2_70B_FFN",
    "LLAMA2_7B_FFN",
    "LinearInputs",
    "LinearShape",
    "SHARDED_PREFILL_TOKENS",
    "TINYLLAMA_LAYER",
    "TINYLLAMA_Q4_0_SHAPES",
    "TINYLLAMA_TOKENS",
    "linear_inputs",
    "q4_0_case",
    "square_case",
    "tinyllama_case",
    "torch_linear_inputs",
]
