"""Generate ``tests/golden/gguf_quants.npz``: Q4_0 and Q8_0 blocks from ggml-org's gguf-py.

The float -> Q4_0 weight quantizer and the float -> Q8_0 activation quantizer of this
path live in llama.cpp (``quantize_row_q4_0`` / ``quantize_row_q8_0``), which the
reference calls but does not vendor (call sites:
integrations/llama_cpp/tests/qpu_ggml_backend_smoke.cpp:119 for Q4_0 and
integrations/llama_cpp/backend/ggml-qpu.cpp:556 for Q8_0; llama.cpp pinned at
91d2fc387529940230555abd297a8b5e99737d3f by scripts/bootstrap_llama_cpp.py:27, absent
here). ggml-org publishes a NumPy restatement of both in its ``gguf`` package
(``gguf.quants.Q4_0.quantize_blocks``, ``gguf.quants.Q8_0.quantize_blocks``; version
0.19.0 is installed in this container), which it documents as bit-exact with
ggml-quants.c's scalar ``quantize_row_q4_0_ref`` / ``quantize_row_q8_0_ref``. This
script runs those functions on seeded inputs and records inputs and blocks:

* ``q4_0_input`` / ``q4_0_blocks`` -- N(0, 0.02) weights (the north-star weight
  distribution) followed by crafted blocks: all zeros, a +a/-a magnitude tie (the first
  index wins), a negative extreme, the -max element that lands on code 16 and clamps
  to 15, fp16-subnormal and large scales;
* ``q8_0_input`` / ``q8_0_blocks`` -- N(0, 1) activations followed by crafted blocks
  (all zeros, tiny and large magnitudes);
* ``q8_0_tie_input`` / ``q8_0_tie_blocks_roundf`` -- a block whose scale is exactly 1,
  so every x * (1/d) is x itself and the half-integers are exact ties.

Ties are where the two llama.cpp Q8_0 forms differ: the scalar reference (and
gguf-py) rounds half away from zero (``roundf``); the NEON form that runs on the
reference's own platform (aarch64) converts with round-to-nearest-even
(``vcvtnq_s32_f32``), as does the reference's in-repo restatement
(examples/benchmark_llama_cpp_qpu_persistent_q4.py:42-54, ``np.rint``). The tests check
this build's quantizers against gguf-py everywhere except exact ties, and hold ties to
round-half-even.

Run: ``python tests/golden/make_gguf_golden.py`` (needs the ``gguf`` package; the GPU
box only reads the .npz).
"""

from __future__ import annotations

import importlib.metadata
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def q4_0_inputs() -> np.ndarray:
    rng = np.random.default_rng(1901)
    normal = (rng.standard_normal((32, 256), dtype=np.float32) * np.float32(0.02)).astype(np.float32)
    crafted = np.zeros((6, 32), dtype=np.float32)
    crafted[1] = rng.uniform(-0.5, 0.5, 32).astype(np.float32)
    crafted[1, 3], crafted[1, 20] = np.float32(0.75), np.float32(-0.75)  # magnitude tie: index 3 wins
    crafted[2] = rng.uniform(-1.0, 1.0, 32).astype(np.float32)
    crafted[2, 7] = np.float32(-3.0)  # negative extreme: d > 0
    crafted[3] = rng.uniform(-1.0, 1.0, 32).astype(np.float32)
    crafted[3, 0], crafted[3, 31] = np.float32(2.0), np.float32(-2.0)  # -max lands on 16.5 -> code 15
    crafted[4] = (rng.standard_normal(32).astype(np.float32) * np.float32(1e-6)).astype(np.float32)  # fp16-subnormal d
    crafted[5] = (rng.standard_normal(32).astype(np.float32) * np.float32(900.0)).astype(np.float32)  # large d
    # row 0 stays all zeros: d = -0.0, id = 0, every code 8
    return np.concatenate([normal, np.pad(crafted, ((0, 0), (0, 256 - 32)))], axis=0).astype(np.float32)


def q8_0_inputs() -> np.ndarray:
    rng = np.random.default_rng(1902)
    normal = rng.standard_normal((16, 256), dtype=np.float32)
    crafted = np.zeros((3, 256), dtype=np.float32)
    crafted[1, :32] = (rng.standard_normal(32).astype(np.float32) * np.float32(1e-5)).astype(np.float32)
    crafted[2, :32] = (rng.standard_normal(32).astype(np.float32) * np.float32(3000.0)).astype(np.float32)
    return np.concatenate([normal, crafted], axis=0).astype(np.float32)


def q8_0_tie_inputs() -> np.ndarray:
    block = np.array([127.0, -127.0, 0.5, -0.5, 1.5, -1.5, 2.5, -2.5, 3.5, -3.5, 100.5, -100.5, 126.5, -126.5]
                     + [float(v) for v in range(-9, 9)], dtype=np.float32)
    return block.reshape(1, 32)


def blocks(quant: type, values: np.ndarray) -> np.ndarray:
    rows, columns = values.shape
    flat = np.ascontiguousarray(values.reshape(-1, 32))
    return np.asarray(quant.quantize_blocks(flat), dtype=np.uint8).reshape(rows, columns // 32, -1)


def main() -> int:
    from gguf.quants import Q4_0, Q8_0

    version = importlib.metadata.version("gguf")
    q4_input = q4_0_inputs()
    q8_input = q8_0_inputs()
    tie_input = q8_0_tie_inputs()
    np.savez_compressed(
        HERE / "gguf_quants.npz",
        gguf_version=np.array(version),
        q4_0_input=q4_input,
        q4_0_blocks=blocks(Q4_0, q4_input),
        q8_0_input=q8_input,
        q8_0_blocks=blocks(Q8_0, q8_input),
        q8_0_tie_input=tie_input,
        q8_0_tie_blocks_roundf=blocks(Q8_0, tie_input),
    )
    print(f"wrote {HERE / 'gguf_quants.npz'} from gguf {version}")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
