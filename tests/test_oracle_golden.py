"""Pin the CPU oracle to the reference: golden vectors produced by the reference itself
(tests/golden/make_golden.py) and the reference's native known-answer test."""

from __future__ import annotations

import hashlib

import numpy as np
import pytest

from oracle import qpu_oracle as oracle
from qpu_xla import workloads
from qpu_xla.ggml import pack_ggml_q4_0_blocks, pack_ggml_q8_0_blocks, unpack_ggml_q4_0_blocks, unpack_ggml_q8_0_blocks


def sha256(array: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(array).tobytes()).hexdigest()


@pytest.mark.parametrize("size", (64, 512))
def test_oracle_w8a8_matches_reference_bit_for_bit(size: int, golden: dict) -> None:
    case = workloads.square_case(size)
    ref = golden[f"w8a8_square_{size}"]
    assert sha256(case.source) == str(ref["source_sha256"]), "seeded inputs drifted from the golden run"
    weight_values, weight_scales = oracle.quantize_per_output_channel_int8(case.weight)
    np.testing.assert_array_equal(weight_values, ref["weight_values"])
    np.testing.assert_array_equal(weight_scales, ref["weight_scales"])
    activation_values, activation_scales = oracle.quantize_rows_int8(case.source)
    np.testing.assert_array_equal(activation_values, ref["activation_values"])
    np.testing.assert_array_equal(activation_scales, ref["activation_scales"])
    accumulation = oracle.int8_accumulate(activation_values, weight_values)
    np.testing.assert_array_equal(accumulation, ref["accumulation"])
    np.testing.assert_array_equal(oracle.int8_accumulate_int32(activation_values, weight_values), ref["accumulation"])
    output = oracle.w8a8_linear(case.source, weight_values, weight_scales, case.bias)
    np.testing.assert_array_equal(output, ref["output"])


@pytest.mark.parametrize("shape", workloads.TINYLLAMA_LAYER, ids=lambda s: s.name)
@pytest.mark.parametrize("tokens", (1, 128))
def test_oracle_tinyllama_projections_match_reference_digests(shape: workloads.LinearShape, tokens: int, golden: dict) -> None:
    digests = golden["w8a8_tinyllama"]
    key = f"{shape.name}_m{tokens}"
    case = workloads.tinyllama_case(shape, tokens)
    assert sha256(case.source) == str(digests[f"{key}_source"])
    weight_values, weight_scales = oracle.quantize_per_output_channel_int8(case.weight)
    assert sha256(weight_values) == str(digests[f"{key}_weight_values"])
    output = oracle.w8a8_linear(case.source, weight_values, weight_scales)
    assert sha256(output) == str(digests[f"{key}_output"])


def test_oracle_q4_0_matches_reference_on_its_hardware_test_inputs(golden: dict) -> None:
    ref = golden["q4_0_reference"]
    expected = oracle.q4_0_q8_0_linear(ref["hw_activation"], ref["hw_weight"])
    np.testing.assert_array_equal(expected, ref["hw_expected"])


@pytest.mark.parametrize("shape", workloads.TINYLLAMA_Q4_0_SHAPES, ids=lambda s: s.name)
@pytest.mark.parametrize("rows", (1, 4))
def test_oracle_q8_0_quantizer_and_block_dot_match_reference(shape: workloads.LinearShape, rows: int, golden: dict) -> None:
    ref = golden["q4_0_reference"]
    key = f"{shape.name}_m{rows}"
    source, weight = workloads.q4_0_case(shape, rows)
    activation = oracle.quantize_q8_0(source)
    np.testing.assert_array_equal(activation, ref[f"{key}_activation"])
    weight_blocks = oracle.quantize_q4_0(weight)
    assert sha256(weight_blocks) == str(ref[f"{key}_weight_sha256"])
    np.testing.assert_array_equal(oracle.q4_0_q8_0_linear(activation, weight_blocks), ref[f"{key}_expected"])


def test_codecs_match_reference_on_extreme_codes(golden: dict) -> None:
    ref = golden["codec_extremes"]
    for pack4, pack8, unpack4, unpack8 in (
        (oracle.pack_q4_0_blocks, oracle.pack_q8_0_blocks, oracle.unpack_q4_0_blocks, oracle.unpack_q8_0_blocks),
        (pack_ggml_q4_0_blocks, pack_ggml_q8_0_blocks, unpack_ggml_q4_0_blocks, unpack_ggml_q8_0_blocks),
    ):
        q4 = pack4(ref["q4_scales"], ref["q4_codes"])
        np.testing.assert_array_equal(q4, ref["q4_blocks"])
        scales, values = unpack4(q4)
        np.testing.assert_array_equal(scales, ref["q4_decoded_scales"])
        np.testing.assert_array_equal(values, ref["q4_decoded_values"])
        q8 = pack8(ref["q8_scales"], ref["q8_values"])
        np.testing.assert_array_equal(q8, ref["q8_blocks"])
        scales, values = unpack8(q8)
        np.testing.assert_array_equal(scales, ref["q8_decoded_scales"])
        np.testing.assert_array_equal(values, ref["q8_decoded_values"])


def native_kat_inputs() -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """The known-answer test of integrations/llama_cpp/tests/qpu_llama_q4_0_smoke.c:17-33.

    Scales 1.0 (fp16 0x3c00), activation value i - 16, weight codes (i + c) % 16
    (low nibble) and (3i + c) % 16 (high nibble); the expectation is the exact
    integer dot product.
    """
    columns = 32
    activation = np.zeros((1, 1, 34), dtype=np.uint8)
    activation[0, 0, :2] = np.array([0x00, 0x3C], dtype=np.uint8)
    values = (np.arange(32) - 16).astype(np.int8)
    activation[0, 0, 2:] = values.view(np.uint8)
    weights = np.zeros((columns, 1, 18), dtype=np.uint8)
    expected = np.zeros(columns, dtype=np.int64)
    for column in range(columns):
        weights[column, 0, 0:2] = (0x00, 0x3C)
        for index in range(16):
            low = (index + column) % 16
            high = (index * 3 + column) % 16
            weights[column, 0, 2 + index] = low | (high << 4)
            expected[column] += (low - 8) * int(values[index]) + (high - 8) * int(values[16 + index])
    return activation, weights, expected


def test_oracle_matches_native_known_answer_test() -> None:
    activation, weights, expected = native_kat_inputs()
    result = oracle.q4_0_q8_0_linear(activation, weights)
    np.testing.assert_array_equal(result[0], expected.astype(np.float32))


def test_q4_0_quantizer_round_trip_is_within_half_a_step() -> None:
    """ggml's quantize_row_q4_0_ref property: |dequant(w) - w| <= |d|/2 (rounding) except the clamped top code."""
    rng = np.random.default_rng(77)
    weight = rng.standard_normal((64, 256), dtype=np.float32) * np.float32(0.02)
    blocks = oracle.quantize_q4_0(weight)
    scales, values = oracle.unpack_q4_0_blocks(blocks)
    reconstructed = (values.astype(np.float32) * scales[..., None]).reshape(weight.shape)
    step = np.repeat(np.abs(scales), 32, axis=1).reshape(weight.shape)
    error = np.abs(reconstructed - weight)
    # One step of slack for the value mapped to +8 and clamped to code 15, plus the fp16
    # rounding of d (relative 2**-11, times at most 8 steps).
    assert np.all(error <= step * (1.0 + 8 * 2.0**-11) + 1e-7)
    assert np.mean(error <= step * 0.5 + 1e-6) > 0.99


def test_q8_0_quantizer_zero_block_and_saturation() -> None:
    values = np.zeros((2, 64), dtype=np.float32)
    values[1, 32:] = np.linspace(-3.0, 3.0, 32, dtype=np.float32)
    blocks = oracle.quantize_q8_0(values)
    scales, quantized = oracle.unpack_q8_0_blocks(blocks)
    assert np.all(scales[0] == 0) and np.all(quantized[0] == 0)
    assert quantized[1, 1].min() == -127 and quantized[1, 1].max() == 127


def test_int8_quantizer_scale_floor_and_zero_rows() -> None:
    """max(max|x| / 127, 1/127): tiny and all-zero rows use the 1/127 floor (quantization.py:165)."""
    values = np.array([[0.0, 0.0, 0.0, 0.0], [1e-4, -2e-4, 0.0, 0.0], [2.0, -4.0, 1.0, 0.5]], dtype=np.float32)
    quantized, scales = oracle.quantize_rows_int8(values)
    assert scales[0] == np.float32(1.0 / 127.0) and scales[1] == np.float32(1.0 / 127.0)
    np.testing.assert_array_equal(quantized[0], 0)
    assert scales[2] == np.float32(4.0) / np.float32(127.0)
    assert quantized[2].tolist() == [64, -127, 32, 16]


def test_conv2d_oracle_matches_the_reference_dynamic_group_reference(golden: dict) -> None:
    """oracle.conv2d_w8a8 against the reference test's own per-group dynamic reference
    (tests/test_qpu_xla_conv2d_w8a8.py:14-54) on its plan and hybrid-partition inputs, and
    oracle.im2col_nchw against _im2col_nchw (src/qpu_xla/ops/conv2d.py:47-79), bit for bit."""
    conv = golden["conv2d_w8a8"]
    lowered = oracle.im2col_nchw(conv["im2col_source"], (3, 2), stride=(2, 1), padding=(1, 2), dilation=(2, 1))
    np.testing.assert_array_equal(lowered, conv["im2col_expected"])
    for name in conv["case_names"]:
        stride, padding, groups = (int(v) for v in conv[f"{name}_params"])
        result = oracle.conv2d_w8a8(conv[f"{name}_source"], conv[f"{name}_weight"], stride=(stride, stride), padding=(padding, padding), groups=groups)
        np.testing.assert_array_equal(result, conv[f"{name}_expected"], err_msg=str(name))
