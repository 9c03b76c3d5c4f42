"""Fused GEMM + all-gather building blocks on one GPU, through the C-ABI.

``qpucuda_w8a8_linear_execute_device_fanout`` writes the same outputs to the local
destination and to every peer destination. With one GPU the "peers" are further
local buffers: the epilogue's fan-out stores (GEMM path) and the per-peer copies
(GEMV path) must reproduce the plain execute bit for bit and leave every column
outside the rank's slice untouched. Peer buffers are created and destroyed here;
mapping one needs a second process and runs in test_gpu_multi.py.
"""

from __future__ import annotations

import ctypes

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


def on_plan(native, name: str, handle: int, *args) -> int:  # type: ignore[no-untyped-def]
    """Call a plan-level function (its first argument is the plan, not the context) on torch's stream."""
    import torch

    native.context.set_stream(torch.cuda.current_stream().cuda_stream)
    return int(getattr(native.lib, name)(handle, *args))


def prepare(native, values: np.ndarray, scales: np.ndarray, bias: np.ndarray | None, *, max_batch: int, start: int, count: int) -> int:  # type: ignore[no-untyped-def]
    desc = _native.W8A8LinearDesc(
        values.ctypes.data, scales.ctypes.data, None if bias is None else bias.ctypes.data,
        values.shape[1], values.shape[0], max_batch, start, count, _native.MEMORY_HOST,
    )
    handle = ctypes.c_void_p()
    native.context.check(native.call("qpucuda_w8a8_linear_prepare", ctypes.byref(desc), ctypes.byref(handle)), "prepare")
    return int(handle.value)  # type: ignore[arg-type]


@pytest.mark.parametrize(
    "rows,k,total,start,count,with_bias",
    [
        (300, 1000, 1024, 256, 512, True),  # GEMM path, aligned 16-byte rows
        (130, 96, 601, 256, 345, False),  # GEMM path, odd row stride and a ragged last tile
        (5, 1000, 1024, 512, 512, True),  # GEMV path (<= 8 rows): local result copied to each peer
    ],
)
@pytest.mark.parametrize("peers", (1, 3, 7))
def test_fanout_matches_the_plain_execute(native, rows: int, k: int, total: int, start: int, count: int, with_bias: bool, peers: int) -> None:  # type: ignore[no-untyped-def]
    import torch

    rng = np.random.default_rng(rows + k + peers)
    weight = rng.standard_normal((total, k), dtype=np.float32) * 0.05
    values, scales = oracle.quantize_per_output_channel_int8(weight)
    bias = rng.standard_normal(total, dtype=np.float32) * 0.1 if with_bias else None
    source = torch.from_numpy(rng.standard_normal((rows, k), dtype=np.float32)).cuda()
    handle = prepare(native, values, scales, bias, max_batch=rows, start=start, count=count)
    try:
        expected = torch.empty((rows, count), dtype=torch.float32, device="cuda")
        assert on_plan(native, "qpucuda_w8a8_linear_execute_device", handle, source.data_ptr(), source.stride(0), rows, expected.data_ptr(), count) == 0
        buffers = [torch.full((rows, total), float("nan"), dtype=torch.float32, device="cuda") for _ in range(peers + 1)]
        addresses = [b.data_ptr() + 4 * start for b in buffers]
        peer_array = (ctypes.c_void_p * peers)(*[ctypes.c_void_p(a) for a in addresses[1:]])
        assert on_plan(native, "qpucuda_w8a8_linear_execute_device_fanout", handle, source.data_ptr(), source.stride(0), rows, addresses[0], peer_array, peers, total) == 0
        native.sync()
        want = expected.cpu().numpy()
        for buffer in buffers:
            got = buffer.cpu().numpy()
            np.testing.assert_array_equal(got[:, start : start + count], want)
            assert np.isnan(got[:, :start]).all() and np.isnan(got[:, start + count :]).all()
        # and the plain output is the reference's: ((float)acc * s_a) * s_w (+ bias)
        window = slice(start, start + count)
        reference = oracle.w8a8_linear(source.cpu().numpy(), values[window], scales[window], None if bias is None else bias[window])
        np.testing.assert_array_equal(want, reference)
    finally:
        native.lib.qpucuda_w8a8_linear_destroy(handle)


def test_fanout_argument_rules(native) -> None:  # type: ignore[no-untyped-def]
    import torch

    values = np.ones((256, 64), dtype=np.int8)
    scales = np.full(256, 0.5, dtype=np.float32)
    handle = prepare(native, values, scales, None, max_batch=16, start=0, count=256)
    try:
        source = torch.zeros((16, 64), dtype=torch.float32, device="cuda")
        out = torch.zeros((16, 256), dtype=torch.float32, device="cuda")
        eight = (ctypes.c_void_p * 8)(*[ctypes.c_void_p(out.data_ptr())] * 8)
        assert on_plan(native, "qpucuda_w8a8_linear_execute_device_fanout", handle, source.data_ptr(), 64, 16, out.data_ptr(), eight, 8, 256) == _native.Status.INVALID_ARGUMENT
        assert on_plan(native, "qpucuda_w8a8_linear_execute_device_fanout", handle, source.data_ptr(), 64, 16, out.data_ptr(), None, 1, 256) == _native.Status.INVALID_ARGUMENT
        null_peer = (ctypes.c_void_p * 1)(ctypes.c_void_p(0))
        assert on_plan(native, "qpucuda_w8a8_linear_execute_device_fanout", handle, source.data_ptr(), 64, 16, out.data_ptr(), null_peer, 1, 256) == _native.Status.INVALID_ARGUMENT
        assert on_plan(native, "qpucuda_w8a8_linear_execute_device_fanout", handle, source.data_ptr(), 64, 16, out.data_ptr(), None, 0, 255) == _native.Status.INVALID_ARGUMENT
        assert on_plan(native, "qpucuda_w8a8_linear_execute_device_fanout", handle, source.data_ptr(), 64, 16, out.data_ptr(), None, 0, 256) == _native.Status.OK
        native.sync()
        assert torch.all(out == 0.0)
    finally:
        native.lib.qpucuda_w8a8_linear_destroy(handle)


def test_peer_buffer_create_and_destroy(native) -> None:  # type: ignore[no-untyped-def]
    pointer = ctypes.c_void_p()
    handle = ctypes.create_string_buffer(64)
    assert native.call("qpucuda_peer_buffer_create", 1 << 20, ctypes.byref(pointer), handle) == _native.Status.OK
    assert pointer.value and any(handle.raw)
    assert native.call("qpucuda_peer_buffer_destroy", pointer) == _native.Status.OK
    native.context.set_failure_mask(int(_native.FailurePoint.ALLOCATION))
    try:
        assert native.call("qpucuda_peer_buffer_create", 1 << 20, ctypes.byref(pointer), handle) == _native.Status.ALLOCATION_FAILED
    finally:
        native.context.set_failure_mask(0)
    assert native.call("qpucuda_peer_buffer_create", 0, ctypes.byref(pointer), handle) == _native.Status.INVALID_ARGUMENT
