"""Q4_0 edge cases on the GPU through the C-ABI.

* The block quantizers (``quantize_q4_0_kernel``, ``quantize_q8_0_kernel``) against the
  blocks ggml-org's gguf-py 0.19.0 produces (``tests/golden/gguf_quants.npz``), byte for
  byte; at exact Q8_0 ties the kernel rounds half to even like the reference's platform
  (see tests/test_gguf_pin.py).
* The codec extremes of the reference's tests/test_qpu_xla_ggml_q4_0.py:25-44 (scales 0,
  -0.5 and 2**-14; codes 0, 15 and the full ramp; activation values -128 and 127 with
  scales 0 and 0.125) through the repack, the decode matvec (rows 1-4), the tiled MX
  path (rows > 4) and the native-block single-kernel entry point.
* The reference's 1- and 2-block K cases (tests/test_qpu_xla_ggml_q4_0.py:164-228: K = 32
  and 64, where the loaders zero-fill past the last block) on the same kernels.

Tolerance: with one or two blocks per output every order of the fp32 block sum rounds
alike ((0 + c0) + c1 = c0 + c1), so the decode matvec must equal the block reference
(ggml_q4_0_q8_0_reference, oracle.q4_0_q8_0_linear) bit for bit, and the MX path the
reference program's arithmetic (oracle.q4_0_q8_0_linear_mx) bit for bit.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np
import pytest

from oracle import qpu_oracle as oracle
from qpu_xla import _native

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def native():  # type: ignore[no-untyped-def]
    from gpu_helpers import Native

    context = Native()
    yield context
    context.close()


def test_block_quantizers_match_gguf(native, golden: dict) -> None:  # type: ignore[no-untyped-def]
    import torch

    ref = golden["gguf_quants"]
    q4 = native.quantize_blocks(torch.from_numpy(ref["q4_0_input"]).cuda(), "q4_0").cpu().numpy()
    np.testing.assert_array_equal(q4, ref["q4_0_blocks"])
    q8 = native.quantize_blocks(torch.from_numpy(ref["q8_0_input"]).cuda(), "q8_0").cpu().numpy()
    np.testing.assert_array_equal(q8, ref["q8_0_blocks"])
    ties = native.quantize_blocks(torch.from_numpy(ref["q8_0_tie_input"]).cuda(), "q8_0").cpu().numpy()
    np.testing.assert_array_equal(ties, oracle.quantize_q8_0(ref["q8_0_tie_input"]))


def extreme_operands(rows: int, blocks: int, outputs: int, seed: int) -> tuple[np.ndarray, np.ndarray]:
    """Q8_0 activations [rows, blocks, 34] and Q4_0 weights [outputs, blocks, 18] built from the
    reference's extreme blocks, mixed with random blocks so every output sees several kinds."""
    ext = np.load(Path(__file__).resolve().parent / "golden" / "codec_extremes.npz")
    rng = np.random.default_rng(seed)
    q4_pool = list(ext["q4_blocks"])
    q8_pool = list(ext["q8_blocks"])
    for _ in range(3):
        q4_pool.append(oracle.pack_q4_0_blocks(
            np.array([rng.uniform(-0.2, 0.2)], dtype=np.float16), rng.integers(0, 16, (1, 32), dtype=np.uint8))[0])
        q8_pool.append(oracle.pack_q8_0_blocks(
            np.array([rng.uniform(0.001, 0.2)], dtype=np.float16), rng.integers(-128, 128, (1, 32), dtype=np.int16))[0])
    weights = np.empty((outputs, blocks, 18), dtype=np.uint8)
    for n in range(outputs):
        for b in range(blocks):
            weights[n, b] = q4_pool[(n + 2 * b) % len(q4_pool)]
    activation = np.empty((rows, blocks, 34), dtype=np.uint8)
    for m in range(rows):
        for b in range(blocks):
            activation[m, b] = q8_pool[(m + 3 * b + 1) % len(q8_pool)]
    return activation, weights


def prepare(native, weights: np.ndarray, rows: int) -> int:  # type: ignore[no-untyped-def]
    weights = np.ascontiguousarray(weights)
    outputs, blocks, _ = weights.shape
    desc = _native.Q40LinearDesc(
        weights.ctypes.data, weights.nbytes, blocks * 32, outputs, rows, 0, outputs, 0, 0,
        native.lib.qpucuda_q4_0_kernel_source_hash(),
    )
    handle = ctypes.c_void_p()
    native.check("qpucuda_q4_0_linear_prepare", ctypes.byref(desc), ctypes.byref(handle))
    return int(handle.value)  # type: ignore[arg-type]


@pytest.mark.parametrize("blocks", (1, 2))
@pytest.mark.parametrize("rows", (1, 2, 3, 4, 5, 16))
def test_extreme_codes_and_short_reductions(native, rows: int, blocks: int) -> None:  # type: ignore[no-untyped-def]
    import torch

    outputs = 48
    activation, weights = extreme_operands(rows, blocks, outputs, seed=4480 + 10 * rows + blocks)
    expected = oracle.q4_0_q8_0_linear_mx(activation, weights) if rows > 4 else oracle.q4_0_q8_0_linear(activation, weights)
    handle = prepare(native, weights, rows)
    try:
        # prepared operator (repack at prepare), device entry point: all columns at an odd offset
        act = torch.from_numpy(activation).cuda()
        out = torch.full((rows, outputs + 4), float("nan"), dtype=torch.float32, device="cuda")
        native.context.set_stream(torch.cuda.current_stream().cuda_stream)
        native.context.check(
            native.lib.qpucuda_q4_0_linear_execute_device(handle, act.data_ptr(), rows, out.data_ptr(), outputs + 4, 0, outputs, 3),
            "execute_device",
        )
        # a column window starting at 16
        window = torch.full((rows, 32), float("nan"), dtype=torch.float32, device="cuda")
        native.context.check(
            native.lib.qpucuda_q4_0_linear_execute_device(handle, act.data_ptr(), rows, window.data_ptr(), 32, 16, 32, 0),
            "execute_device window",
        )
        native.sync()
        got = out.cpu().numpy()
        np.testing.assert_array_equal(got[:, 3 : 3 + outputs], expected)
        assert np.isnan(got[:, :3]).all() and np.isnan(got[:, 3 + outputs :]).all()
        np.testing.assert_array_equal(window.cpu().numpy(), expected[:, 16:48])
        # host entry point (staged copies, bounded wait)
        host = np.full((rows, outputs), np.nan, dtype=np.float32)
        execution = _native.Q40Execution(activation.ctypes.data, activation.nbytes, 0, host.ctypes.data, host.nbytes, 0, 0, outputs, rows, 0)
        timing = _native.Q40Timing()
        assert native.lib.qpucuda_q4_0_linear_execute(handle, ctypes.byref(execution), ctypes.byref(timing)) == _native.Status.OK
        np.testing.assert_array_equal(host, expected)
    finally:
        native.lib.qpucuda_q4_0_linear_destroy(handle)
    if rows <= 4:
        # the single-kernel entry point reads the native 18-byte blocks without a repack
        act = torch.from_numpy(activation).cuda()
        weight = torch.from_numpy(np.ascontiguousarray(weights[16:48])).cuda()
        out = torch.full((rows, 48), float("nan"), dtype=torch.float32, device="cuda")
        native.check("qpucuda_ggml_q4_0_q8_0_linear", act.data_ptr(), rows, blocks, weight.data_ptr(), 32, out.data_ptr(), 48, 0, 16, 32)
        native.sync()
        got = out.cpu().numpy()
        np.testing.assert_array_equal(got[:, 16:48], expected[:, 16:48])
        assert np.isnan(got[:, :16]).all()


def test_repack_keeps_extreme_blocks(native) -> None:  # type: ignore[no-untyped-def]
    """Extreme weight blocks survive the prepare-time repack: a one-hot activation per code
    position reads every weight value back, times the weight scale, exactly."""
    import torch

    _, weights = extreme_operands(1, 1, 16, seed=7)
    scales, values = oracle.unpack_q4_0_blocks(weights)
    handle = prepare(native, weights, 1)
    try:
        native.context.set_stream(torch.cuda.current_stream().cuda_stream)
        for position in range(32):
            q8 = np.zeros(32, dtype=np.int16)
            q8[position] = 1
            activation = oracle.pack_q8_0_blocks(np.array([1.0], dtype=np.float16), q8[None, :]).reshape(1, 1, 34)
            act = torch.from_numpy(activation).cuda()
            out = torch.empty((1, 16), dtype=torch.float32, device="cuda")
            native.context.check(
                native.lib.qpucuda_q4_0_linear_execute_device(handle, act.data_ptr(), 1, out.data_ptr(), 16, 0, 16, 0),
                "execute_device",
            )
            native.sync()
            expected = values[:, 0, position].astype(np.float32) * scales[:, 0]
            np.testing.assert_array_equal(out.cpu().numpy()[0], expected)
    finally:
        native.lib.qpucuda_q4_0_linear_destroy(handle)


def non_finite_operands(rows: int, blocks: int, outputs: int, seed: int) -> tuple[np.ndarray, np.ndarray]:
    """Random Q8_0/Q4_0 operands with fp16 scales of +inf, -inf, NaN and 65504 planted in both."""
    rng = np.random.default_rng(seed)
    a_scales = rng.uniform(0.001, 0.2, (rows, blocks)).astype(np.float16)
    a_values = rng.integers(-128, 128, (rows, blocks, 32), dtype=np.int16)
    w_scales = rng.uniform(-0.2, 0.2, (outputs, blocks)).astype(np.float16)
    w_codes = rng.integers(0, 16, (outputs, blocks, 32), dtype=np.uint8)
    special = (np.inf, -np.inf, np.nan, 65504.0)
    for i, value in enumerate(special):
        a_scales[i % rows, (3 * i + 1) % blocks] = value
        w_scales[(5 * i + 2) % outputs, (2 * i) % blocks] = value
    a_scales[rows - 1, blocks - 1] = np.inf
    a_values[rows - 1, blocks - 1] = 0  # +inf times a zero dot
    activation = oracle.pack_q8_0_blocks(a_scales.reshape(-1), a_values.reshape(-1, 32)).reshape(rows, blocks, 34)
    weights = oracle.pack_q4_0_blocks(w_scales.reshape(-1), w_codes.reshape(-1, 32)).reshape(outputs, blocks, 18)
    return activation, weights


@pytest.mark.parametrize("rows,outputs", [(1, 48), (4, 48), (5, 48), (16, 48), (130, 48), (16, 19200), (130, 9600)])
def test_non_finite_scales(native, rows: int, outputs: int) -> None:  # type: ignore[no-untyped-def]
    """Infinite and NaN block scales in either operand: the tiled MX path (rows > 4) equals the
    reference program's arithmetic bit for bit, infinities and NaN positions included; the decode
    matvec (rows 1-4) has the same non-finite positions and agrees elsewhere within its tolerance.
    The wide cases give the tcgen05 MX kernel a tile per SM; the narrow ones run the mma.sync kernel."""
    import torch

    blocks = 12
    activation, weights = non_finite_operands(rows, blocks, outputs, seed=9100 + rows)
    with np.errstate(all="ignore"):
        expected = oracle.q4_0_q8_0_linear_mx(activation, weights) if rows > 4 else oracle.q4_0_q8_0_linear(activation, weights)
    assert np.isnan(expected).any() and (rows == 1 or np.isinf(expected).any())
    handle = prepare(native, weights, rows)
    try:
        act = torch.from_numpy(activation).cuda()
        out = torch.full((rows, outputs), 7.0, dtype=torch.float32, device="cuda")
        native.context.set_stream(torch.cuda.current_stream().cuda_stream)
        native.context.check(
            native.lib.qpucuda_q4_0_linear_execute_device(handle, act.data_ptr(), rows, out.data_ptr(), outputs, 0, outputs, 0),
            "execute_device",
        )
        native.sync()
        got = out.cpu().numpy()
    finally:
        native.lib.qpucuda_q4_0_linear_destroy(handle)
    if rows > 4:
        np.testing.assert_array_equal(got, expected)
    else:
        np.testing.assert_array_equal(np.isnan(got), np.isnan(expected))
        np.testing.assert_array_equal(np.isposinf(got), np.isposinf(expected))
        np.testing.assert_array_equal(np.isneginf(got), np.isneginf(expected))
        finite = np.isfinite(expected)
        np.testing.assert_allclose(got[finite], expected[finite], rtol=2e-6, atol=2e-5)
