"""The Q4_0 / Q8_0 quantizers pinned to ggml-org's gguf-py restatement of llama.cpp.

llama.cpp's ``quantize_row_q4_0`` and ``quantize_row_q8_0`` are third-party code the
reference calls but does not vendor (qpu_ggml_backend_smoke.cpp:119, ggml-qpu.cpp:556).
``tests/golden/gguf_quants.npz`` holds the blocks gguf-py 0.19.0 produces
(``tests/golden/make_gguf_golden.py``); the oracle must reproduce them byte for byte,
except that at exact Q8_0 ties it rounds half to even, as the reference's platform (the
aarch64 NEON form, ``vcvtnq_s32_f32``) and its in-repo restatement (``np.rint``,
examples/benchmark_llama_cpp_qpu_persistent_q4.py:42-54) do, where gguf-py's scalar form
rounds half away from zero.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import qpu_oracle as oracle


def test_q4_0_quantizer_matches_gguf_byte_for_byte(golden: dict) -> None:
    ref = golden["gguf_quants"]
    np.testing.assert_array_equal(oracle.quantize_q4_0(ref["q4_0_input"]), ref["q4_0_blocks"])


def test_q8_0_quantizer_matches_gguf_byte_for_byte(golden: dict) -> None:
    ref = golden["gguf_quants"]
    np.testing.assert_array_equal(oracle.quantize_q8_0(ref["q8_0_input"]), ref["q8_0_blocks"])


def test_q8_0_ties_round_half_to_even(golden: dict) -> None:
    ref = golden["gguf_quants"]
    values = ref["q8_0_tie_input"]
    ours = oracle.quantize_q8_0(values)
    roundf = ref["q8_0_tie_blocks_roundf"]
    np.testing.assert_array_equal(ours[..., :2], roundf[..., :2])  # the scale (exactly 1.0)
    ours_q = ours[0, 0, 2:].view(np.int8).astype(np.int32)
    roundf_q = roundf[0, 0, 2:].view(np.int8).astype(np.int32)
    tie = (np.abs(values[0]) % 1.0) == 0.5
    assert tie.sum() == 12
    np.testing.assert_array_equal(ours_q[~tie], roundf_q[~tie])
    np.testing.assert_array_equal(ours_q[tie], np.rint(values[0][tie]).astype(np.int32))
    assert np.all(roundf_q[tie] == np.sign(values[0][tie]) * np.floor(np.abs(values[0][tie]) + 0.5))


def test_fixture_is_what_gguf_produces() -> None:
    """The committed fixture regenerates from the installed gguf-py (skipped where it is absent)."""
    pytest.importorskip("gguf")
    import importlib.util
    from pathlib import Path

    path = Path(__file__).resolve().parent / "golden" / "make_gguf_golden.py"
    spec = importlib.util.spec_from_file_location("make_gguf_golden", path)
    assert spec is not None and spec.loader is not None
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    from gguf.quants import Q4_0, Q8_0

    with np.load(path.parent / "gguf_quants.npz") as ref:
        np.testing.assert_array_equal(module.blocks(Q4_0, module.q4_0_inputs()), ref["q4_0_blocks"])
        np.testing.assert_array_equal(module.blocks(Q8_0, module.q8_0_inputs()), ref["q8_0_blocks"])
        np.testing.assert_array_equal(module.blocks(Q8_0, module.q8_0_tie_inputs()), ref["q8_0_tie_blocks_roundf"])
