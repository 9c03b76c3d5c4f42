"""CPU oracle for the qpu_xla quantized-linear path -- TEST INFRASTRUCTURE ONLY.

This module restates, in NumPy, the reference's own CPU arithmetic for the two
halves of the hot path:

* dynamic W8A8 linear: per-row symmetric int8 activation quantization, exact
  int8 x int8 -> int32 accumulation, fp32 dequantization ``(acc*s_a)*s_w`` and an
  optional bias added afterwards;
* GGML Q4_0 x Q8_0 block-dot linear, with the native 18-byte / 34-byte block
  codecs and the two float -> block quantizers.

It is the *checker*. Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import it. The
product path (the CUDA library and the ``qpu_xla`` package) never calls into
this file; a product path that fell back to it would void every parity claim.

Parity pinning: the W8A8 functions and the Q4_0 block reference are pinned
against golden vectors produced by importing the reference itself
(``tests/golden/make_golden.py``) and against the reference's native
known-answer test. ``quantize_q4_0`` restates ggml's published
``quantize_row_q4_0_ref`` (llama.cpp ``ggml/src/ggml-quants.c`` at the
reference's pinned commit ``91d2fc387529940230555abd297a8b5e99737d3f``,
``scripts/bootstrap_llama_cpp.py:27``); no reference test pins its output, so
that one function is "parity unpinned" and is checked by round-trip bounds only.
"""

from __future__ import annotations

import numpy as np
import numpy.typing as npt

Q4_0_BLOCK_ELEMENTS = 32
Q4_0_BLOCK_BYTES = 18
Q8_0_BLOCK_BYTES = 34

# np.float32(1.0 / 127.0): the scale floor used by every per-row quantizer in
# src/qpu_xla/models/tinyllama/quantization.py (:165, :1068, :1089).
SCALE_FLOOR = np.float32(1.0 / 127.0)


# --------------------------------------------------------------------------
# W8A8 (src/qpu_xla/models/tinyllama/quantization.py)
# --------------------------------------------------------------------------


def quantize_rows_int8(values: npt.NDArray[np.float32]) -> tuple[npt.NDArray[np.int8], npt.NDArray[np.float32]]:
    """Per-row symmetric int8 quantization.

    Follows ``PreparedW8A8Linear._prepare_values`` (quantization.py:156-171),
    ``CalibratedW8A8Linear.execute.cpu_reference`` (:1065-1071) and
    ``quantize_per_output_channel_int8`` (:1085-1092), which are the same
    formula: ``s = max(max|x| / 127, 1/127)`` in fp32, then
    ``q = clip(rint(x / s), -127, 127)`` with an IEEE fp32 division and
    round-half-to-even.
    """
    values = np.asarray(values)
    if values.ndim != 2 or values.dtype != np.float32:
        raise ValueError("quantize_rows_int8 requires a rank-2 float32 matrix")
    scales = np.maximum(np.max(np.abs(values), axis=1) / np.float32(127.0), SCALE_FLOOR).astype(np.float32)
    quantized = np.rint(values / scales[:, None]).clip(-127, 127).astype(np.int8)
    return np.ascontiguousarray(quantized), np.ascontiguousarray(scales)


def quantize_per_output_channel_int8(weight: npt.NDArray[np.float32]) -> tuple[npt.NDArray[np.int8], npt.NDArray[np.float32]]:
    """Weight quantization, one scale per output row (quantization.py:1085-1092)."""
    return quantize_rows_int8(weight)


def int8_accumulate(left: npt.NDArray[np.int8], right_rows: npt.NDArray[np.int8]) -> npt.NDArray[np.int32]:
    """Exact ``left @ right_rows.T`` in int32 (quantization.py:1072).

    The product is formed in float64 through BLAS. That is exact here: every
    int8*int8 product and every partial sum is an integer of magnitude at most
    ``K * 127 * 127 < 2**53``, so no float64 addition rounds, in any order.
    """
    result = np.asarray(left, dtype=np.float64) @ np.asarray(right_rows, dtype=np.float64).T
    return result.astype(np.int32)


def int8_accumulate_int32(left: npt.NDArray[np.int8], right_rows: npt.NDArray[np.int8]) -> npt.NDArray[np.int32]:
    """The reference's literal int32 NumPy matmul (quantization.py:1070-1072); slow, used as the CPU baseline."""
    return left.astype(np.int32) @ right_rows.astype(np.int32).T


def w8a8_dequantize(
    accumulation: npt.NDArray[np.int32],
    row_scales: npt.NDArray[np.float32],
    column_scales: npt.NDArray[np.float32],
    bias: npt.NDArray[np.float32] | None = None,
) -> npt.NDArray[np.float32]:
    """``(float(acc) * s_a[m]) * s_w[n]`` left to right in fp32 (quantization.py:1073-1075).

    The bias, when present, is added after the dequantization, as in
    ``_StagedW8A8Linear._cpu`` (src/qpu_xla/models/smolvla/accelerated.py:260-261).
    """
    result = accumulation.astype(np.float32) * row_scales[:, None] * column_scales[None, :]
    if bias is not None:
        result = result + bias[None, :].astype(np.float32)
    return np.ascontiguousarray(result, dtype=np.float32)


def w8a8_linear(
    source: npt.NDArray[np.float32],
    weight_values: npt.NDArray[np.int8],
    weight_scales: npt.NDArray[np.float32],
    bias: npt.NDArray[np.float32] | None = None,
    *,
    literal_int32: bool = False,
) -> npt.NDArray[np.float32]:
    """Whole dynamic W8A8 linear, ``CalibratedW8A8Linear.execute.cpu_reference`` (quantization.py:1065-1082)."""
    quantized, scales = quantize_rows_int8(source)
    accumulate = int8_accumulate_int32 if literal_int32 else int8_accumulate
    return w8a8_dequantize(accumulate(quantized, weight_values), scales, weight_scales, bias)


# --------------------------------------------------------------------------
# W8A8 convolution (src/qpu_xla/ops/conv2d.py, src/qpu_xla/ops/conv2d_w8a8.py)
# --------------------------------------------------------------------------


def conv_output_hw(height: int, width: int, kernel: tuple[int, int], stride: tuple[int, int], padding: tuple[int, int], dilation: tuple[int, int]) -> tuple[int, int]:
    """Valid NCHW output size (conv2d.py:25-39)."""
    output_height = (height + 2 * padding[0] - dilation[0] * (kernel[0] - 1) - 1) // stride[0] + 1
    output_width = (width + 2 * padding[1] - dilation[1] * (kernel[1] - 1) - 1) // stride[1] + 1
    if output_height <= 0 or output_width <= 0:
        raise ValueError("convolution parameters produce an empty output")
    return output_height, output_width


def im2col_nchw(
    source: npt.NDArray[np.float32], kernel: tuple[int, int], *, stride: tuple[int, int], padding: tuple[int, int], dilation: tuple[int, int]
) -> npt.NDArray[np.float32]:
    """Rows (b, oh, ow), columns (c, i, j): the source value at (c, oh*s - p + i*d, ow*s - p + j*d),
    zero in the padding (``_im2col_nchw``, conv2d.py:47-79), written as explicit gathers."""
    batch, channels, height, width = source.shape
    output_height, output_width = conv_output_hw(height, width, kernel, stride, padding, dilation)
    padded = np.zeros((batch, channels, height + 2 * padding[0], width + 2 * padding[1]), dtype=source.dtype)
    padded[:, :, padding[0] : padding[0] + height, padding[1] : padding[1] + width] = source
    columns = np.empty((batch, output_height, output_width, channels, kernel[0], kernel[1]), dtype=source.dtype)
    rows_index = np.arange(output_height) * stride[0]
    cols_index = np.arange(output_width) * stride[1]
    for i in range(kernel[0]):
        for j in range(kernel[1]):
            window = padded[:, :, rows_index[:, None] + i * dilation[0], cols_index[None, :] + j * dilation[1]]
            columns[:, :, :, :, i, j] = window.transpose(0, 2, 3, 1)
    return np.ascontiguousarray(columns.reshape(batch * output_height * output_width, channels * kernel[0] * kernel[1]))


def conv2d_w8a8(
    source: npt.NDArray[np.float32],
    weight: npt.NDArray[np.float32],
    *,
    stride: tuple[int, int] = (1, 1),
    padding: tuple[int, int] = (0, 0),
    dilation: tuple[int, int] = (1, 1),
    groups: int = 1,
) -> npt.NDArray[np.float32]:
    """Per-group dynamic W8A8 convolution, NCHW in and out: each group's im2col rows through
    ``w8a8_linear`` with its output channels' weights quantized per channel, then the pixels x
    channels matrix back to NCHW (conv2d_w8a8.py:111-137, :171-305; the reference test's
    ``_dynamic_group_reference``, tests/test_qpu_xla_conv2d_w8a8.py:14-54)."""
    batch, channels, height, width = source.shape
    outputs, group_channels, kernel_height, kernel_width = weight.shape
    output_height, output_width = conv_output_hw(height, width, (kernel_height, kernel_width), stride, padding, dilation)
    rows = batch * output_height * output_width
    lowered = im2col_nchw(source, (kernel_height, kernel_width), stride=stride, padding=padding, dilation=dilation).reshape(rows, channels, kernel_height, kernel_width)
    output_group = outputs // groups
    results = []
    for group in range(groups):
        matrix = np.ascontiguousarray(lowered[:, group * group_channels : (group + 1) * group_channels].reshape(rows, -1))
        values, scales = quantize_per_output_channel_int8(np.ascontiguousarray(weight[group * output_group : (group + 1) * output_group].reshape(output_group, -1)))
        results.append(w8a8_linear(matrix, values, scales))
    return np.ascontiguousarray(np.concatenate(results, axis=1).reshape(batch, output_height, output_width, outputs).transpose(0, 3, 1, 2))


# --------------------------------------------------------------------------
# GGML Q4_0 / Q8_0 (src/qpu_xla/kernels/ggml_q4_0.py)
# --------------------------------------------------------------------------


def pack_q4_0_blocks(scales: npt.ArrayLike, codes: npt.ArrayLike) -> npt.NDArray[np.uint8]:
    """Native ``block_q4_0``: fp16 d (little-endian) then 16 bytes; byte j = code j | code j+16 << 4 (ggml_q4_0.py:28-40)."""
    scales = np.asarray(scales, dtype=np.float16)
    codes = np.asarray(codes)
    if codes.shape != (*scales.shape, Q4_0_BLOCK_ELEMENTS) or np.any((codes < 0) | (codes > 15)):
        raise ValueError("Q4_0 codes must have scales.shape + (32,) and values in 0..15")
    packed = np.empty((*scales.shape, Q4_0_BLOCK_BYTES), dtype=np.uint8)
    packed[..., :2] = scales.astype("<f2").view(np.uint8).reshape(*scales.shape, 2)
    packed[..., 2:] = codes[..., :16].astype(np.uint8) | (codes[..., 16:].astype(np.uint8) << 4)
    return np.ascontiguousarray(packed)


def pack_q8_0_blocks(scales: npt.ArrayLike, values: npt.ArrayLike) -> npt.NDArray[np.uint8]:
    """Native ``block_q8_0``: fp16 d then 32 signed bytes (ggml_q4_0.py:43-54)."""
    scales = np.asarray(scales, dtype=np.float16)
    values = np.asarray(values)
    if values.shape != (*scales.shape, Q4_0_BLOCK_ELEMENTS) or np.any((values < -128) | (values > 127)):
        raise ValueError("Q8_0 values must have scales.shape + (32,) and values in -128..127")
    packed = np.empty((*scales.shape, Q8_0_BLOCK_BYTES), dtype=np.uint8)
    packed[..., :2] = scales.astype("<f2").view(np.uint8).reshape(*scales.shape, 2)
    packed[..., 2:] = values.astype(np.int8).view(np.uint8)
    return np.ascontiguousarray(packed)


def unpack_q4_0_blocks(blocks: npt.NDArray[np.uint8]) -> tuple[npt.NDArray[np.float32], npt.NDArray[np.int8]]:
    """Decode native Q4_0 blocks to (fp32 scales, int8 values = code - 8) (ggml_q4_0.py:57-67)."""
    blocks = np.asarray(blocks)
    if blocks.dtype != np.uint8 or blocks.shape[-1] != Q4_0_BLOCK_BYTES:
        raise ValueError("Q4_0 blocks must be uint8 with a final extent of 18 bytes")
    scales = blocks[..., :2].copy().reshape(-1, 2).view("<f2").reshape(blocks.shape[:-1]).astype(np.float32)
    packed = blocks[..., 2:]
    values = np.empty((*blocks.shape[:-1], Q4_0_BLOCK_ELEMENTS), dtype=np.int8)
    values[..., :16] = (packed & 0x0F).astype(np.int8) - 8
    values[..., 16:] = (packed >> 4).astype(np.int8) - 8
    return scales, values


def unpack_q8_0_blocks(blocks: npt.NDArray[np.uint8]) -> tuple[npt.NDArray[np.float32], npt.NDArray[np.int8]]:
    """Decode native Q8_0 blocks to (fp32 scales, int8 values) (ggml_q4_0.py:70-78)."""
    blocks = np.asarray(blocks)
    if blocks.dtype != np.uint8 or blocks.shape[-1] != Q8_0_BLOCK_BYTES:
        raise ValueError("Q8_0 blocks must be uint8 with a final extent of 34 bytes")
    scales = blocks[..., :2].copy().reshape(-1, 2).view("<f2").reshape(blocks.shape[:-1]).astype(np.float32)
    return scales, blocks[..., 2:].view(np.int8)


def q4_0_q8_0_linear(activation_blocks: npt.NDArray[np.uint8], weight_blocks: npt.NDArray[np.uint8]) -> npt.NDArray[np.float32]:
    """``y[m,n] = sum_b ((float)dot_b * d_w[n,b]) * d_a[m,b]``, blocks summed in order (ggml_q4_0.py:81-100)."""
    if activation_blocks.ndim != 3 or weight_blocks.ndim != 3:
        raise ValueError("activation and weight blocks must both be rank three")
    rows, blocks, activation_bytes = activation_blocks.shape
    outputs, weight_block_count, weight_bytes = weight_blocks.shape
    if activation_bytes != Q8_0_BLOCK_BYTES or weight_bytes != Q4_0_BLOCK_BYTES or blocks != weight_block_count:
        raise ValueError("native Q8_0/Q4_0 block extents or reduction block counts do not match")
    activation_scales, activations = unpack_q8_0_blocks(activation_blocks)
    weight_scales, weights = unpack_q4_0_blocks(weight_blocks)
    result = np.zeros((rows, outputs), dtype=np.float32)
    for block in range(blocks):
        # Exact block dots: |dot| <= 32*128*8, computed in float64 BLAS without rounding.
        dots = (activations[:, block].astype(np.float64) @ weights[:, block].astype(np.float64).T).astype(np.int32)
        contribution = dots.astype(np.float32) * weight_scales[None, :, block]
        contribution *= activation_scales[:, block, None]
        result += contribution
    return result


def q4_0_q8_0_linear_mx(activation_blocks: npt.NDArray[np.uint8], weight_blocks: npt.NDArray[np.uint8]) -> npt.NDArray[np.float32]:
    """The reference's tiled (MX, rows > 4) program: per output one fp32 accumulator over the blocks
    in order, ``acc += ((float)dot_b * d_a[m, b]) * d_w[n, b]`` (activation scale first;
    src/qpu_xla/kernels/ggml_q4_0.py:506-513). Same exact block dots as ``q4_0_q8_0_linear``."""
    if activation_blocks.ndim != 3 or weight_blocks.ndim != 3:
        raise ValueError("activation and weight blocks must both be rank three")
    rows, blocks, _ = activation_blocks.shape
    if weight_blocks.shape[1] != blocks:
        raise ValueError("reduction block counts do not match")
    activation_scales, activations = unpack_q8_0_blocks(activation_blocks)
    weight_scales, weights = unpack_q4_0_blocks(weight_blocks)
    result = np.zeros((rows, weight_blocks.shape[0]), dtype=np.float32)
    for block in range(blocks):
        dots = (activations[:, block].astype(np.float64) @ weights[:, block].astype(np.float64).T).astype(np.int32)
        contribution = dots.astype(np.float32) * activation_scales[:, block, None]
        contribution *= weight_scales[None, :, block]
        result += contribution
    return result


def q4_0_q8_0_block_dots(activation_blocks: npt.NDArray[np.uint8], weight_blocks: npt.NDArray[np.uint8]) -> npt.NDArray[np.int32]:
    """Per-block exact integer dots ``[rows, outputs, blocks]`` (the int part of ggml_q4_0.py:96)."""
    _, activations = unpack_q8_0_blocks(activation_blocks)
    _, weights = unpack_q4_0_blocks(weight_blocks)
    return np.einsum("mbk,nbk->mnb", activations.astype(np.int32), weights.astype(np.int32))


def quantize_q8_0(values: npt.NDArray[np.float32]) -> npt.NDArray[np.uint8]:
    """fp32 rows -> native Q8_0 blocks.

    Follows the reference's in-repo restatement of llama.cpp ``quantize_row_q8_0``,
    ``quantize_q8_0_split`` (examples/benchmark_llama_cpp_qpu_persistent_q4.py:42-54):
    ``d = amax / 127`` (fp32), ``q = clip(rint(x * (1/d)), -127, 127)`` with 0 for an
    all-zero block, and the stored scale is ``fp16(d)``.
    """
    values = np.asarray(values)
    if values.ndim != 2 or values.dtype != np.float32 or values.shape[1] % Q4_0_BLOCK_ELEMENTS:
        raise ValueError("quantize_q8_0 requires float32 [rows, K] with K % 32 == 0")
    rows, columns = values.shape
    grouped = values.reshape(rows, columns // Q4_0_BLOCK_ELEMENTS, Q4_0_BLOCK_ELEMENTS)
    scales = np.max(np.abs(grouped), axis=2).astype(np.float32) / np.float32(127.0)
    inverse = np.zeros_like(scales)
    np.divide(np.float32(1.0), scales, out=inverse, where=scales != 0.0)
    quantized = np.clip(np.rint(grouped * inverse[..., None]), -127, 127).astype(np.int8)
    return pack_q8_0_blocks(scales.astype(np.float16), quantized)


def quantize_q4_0(values: npt.NDArray[np.float32]) -> npt.NDArray[np.uint8]:
    """fp32 rows -> native Q4_0 blocks, restating ggml's published ``quantize_row_q4_0_ref``.

    Per block of 32: ``max`` = the signed value of largest magnitude (first one on
    ties), ``d = max / -8``, ``id = 1/d`` (0 when d == 0), code =
    ``min(15, trunc(x*id + 8.5))``, stored scale ``fp16(d)``. Parity unpinned: no
    reference test fixes this function's output.
    """
    values = np.asarray(values)
    if values.ndim != 2 or values.dtype != np.float32 or values.shape[1] % Q4_0_BLOCK_ELEMENTS:
        raise ValueError("quantize_q4_0 requires float32 [rows, K] with K % 32 == 0")
    rows, columns = values.shape
    grouped = values.reshape(rows, columns // Q4_0_BLOCK_ELEMENTS, Q4_0_BLOCK_ELEMENTS)
    index = np.argmax(np.abs(grouped), axis=2)
    maximum = np.take_along_axis(grouped, index[..., None], axis=2)[..., 0]
    d = (maximum / np.float32(-8.0)).astype(np.float32)
    inverse = np.zeros_like(d)
    np.divide(np.float32(1.0), d, out=inverse, where=d != 0.0)
    scaled = (grouped * inverse[..., None]).astype(np.float32) + np.float32(8.5)
    codes = np.minimum(np.float32(15.0), np.trunc(scaled)).astype(np.int32)
    codes = np.clip(codes, 0, 15)
    return pack_q4_0_blocks(d.astype(np.float16), codes.astype(np.uint8))


def pack_q4_0x4(blocks: npt.NDArray[np.uint8]) -> npt.NDArray[np.uint8]:
    """Native ``block_q4_0`` rows ``[N, K/32, 18]`` (N % 4 == 0) into ggml-cpu's CPU_REPACK
    block_q4_0x4 bytes, the layout the reference's backend unpacks (ggml-qpu.cpp:250-283): per
    group of 4 rows and K block, the 4 fp16 scales (8 bytes), then 64 quant bytes in which the
    4-byte chunk c of row r sits at (c * 4 + r) * 4, every byte XOR 0x88."""
    n, nblocks, _ = blocks.shape
    if n % 4 != 0:
        raise ValueError("CPU_REPACK groups need N % 4 == 0")
    rows = blocks.reshape(n // 4, 4, nblocks, 18)
    packed = np.empty((n // 4, nblocks, 72), dtype=np.uint8)
    for r in range(4):
        packed[:, :, 2 * r : 2 * r + 2] = rows[:, r, :, 0:2]
        for c in range(4):
            at = 8 + (c * 4 + r) * 4
            packed[:, :, at : at + 4] = rows[:, r, :, 2 + c * 4 : 6 + c * 4] ^ np.uint8(0x88)
    return packed.reshape(-1)
