"""The GGML MUL_MAT offload's host logic (include/qpucuda_ggml.h) without a GPU: the support
predicate of the reference's backend (integrations/llama_cpp/backend/ggml-qpu.cpp:362-377 plus the
row window of :631-633) and the CPU_REPACK weight unpack (:250-283)."""

from __future__ import annotations

import numpy as np
import pytest

from oracle import qpu_oracle as oracle
from qpu_xla import _native
from qpu_xla.ggml import ggml_supports_mul_mat, ggml_tensor_view, ggml_unpack_q4_0x4


def _views(rows: int = 4, k: int = 64, n: int = 32):  # type: ignore[no-untyped-def]
    arrays = (
        np.zeros((n, k // 32, 18), dtype=np.uint8),
        np.zeros((rows, k), dtype=np.float32),
        np.zeros((rows, n), dtype=np.float32),
    )
    views = (
        ggml_tensor_view(arrays[0], _native.GGML_TYPE_Q4_0),
        ggml_tensor_view(arrays[1], _native.GGML_TYPE_F32),
        ggml_tensor_view(arrays[2], _native.GGML_TYPE_F32),
    )
    return arrays, views


def test_supported_node() -> None:
    _, (w, a, d) = _views()
    assert ggml_supports_mul_mat(w, a, d)
    assert ggml_supports_mul_mat(w, a, d, minimum_rows=4, maximum_rows=4)


@pytest.mark.parametrize(
    "mutate",
    [
        lambda w, a, d: setattr(w, "type", _native.GGML_TYPE_F32),  # weight not Q4_0
        lambda w, a, d: setattr(a, "type", _native.GGML_TYPE_Q4_0),  # activation not F32
        lambda w, a, d: (w.ne.__setitem__(0, 48), a.ne.__setitem__(0, 48)),  # K % 32 != 0
        lambda w, a, d: (w.ne.__setitem__(1, 24), d.ne.__setitem__(0, 24)),  # N % 16 != 0
        lambda w, a, d: a.ne.__setitem__(0, 32),  # activation K differs from the weight's
        lambda w, a, d: (a.ne.__setitem__(1, 4 * 65535 + 1), d.ne.__setitem__(1, 4 * 65535 + 1)),  # too many rows
        lambda w, a, d: w.ne.__setitem__(2, 2),  # batched weight
        lambda w, a, d: a.ne.__setitem__(3, 2),  # batched activation
        lambda w, a, d: a.nb.__setitem__(1, a.nb[1] + 16),  # activation rows not contiguous
        lambda w, a, d: w.nb.__setitem__(1, w.nb[1] + 18),  # weight rows not packed back to back
        lambda w, a, d: w.nb.__setitem__(0, 34),  # weight blocks are not Q4_0-sized
        lambda w, a, d: d.ne.__setitem__(0, 16),  # destination is not [N, M]
        lambda w, a, d: d.nb.__setitem__(0, 8),  # destination not contiguous
        lambda w, a, d: setattr(d, "data", None),  # no destination memory
    ],
)
def test_unsupported_nodes(mutate) -> None:  # type: ignore[no-untyped-def]
    _, (w, a, d) = _views()
    mutate(w, a, d)
    assert not ggml_supports_mul_mat(w, a, d)


def test_views_reject_arrays_they_cannot_describe() -> None:
    arrays, _ = _views()
    weight, activation, _ = arrays
    with pytest.raises(ValueError, match="C-contiguous"):
        ggml_tensor_view(activation[:, ::2], _native.GGML_TYPE_F32)
    with pytest.raises(ValueError, match="C-contiguous"):
        ggml_tensor_view(weight[::2], _native.GGML_TYPE_Q4_0)
    with pytest.raises(ValueError, match="float32"):
        ggml_tensor_view(activation.astype(np.float64), _native.GGML_TYPE_F32)
    with pytest.raises(ValueError, match="uint8"):
        ggml_tensor_view(weight.reshape(weight.shape[0], -1), _native.GGML_TYPE_Q4_0)


def test_row_window() -> None:
    _, (w, a, d) = _views(rows=3)
    assert not ggml_supports_mul_mat(w, a, d, minimum_rows=4)
    assert not ggml_supports_mul_mat(w, a, d, maximum_rows=2)
    assert ggml_supports_mul_mat(w, a, d, minimum_rows=1, maximum_rows=3)


def test_cpu_repack_unpack_round_trip() -> None:
    rng = np.random.default_rng(11)
    blocks = rng.integers(0, 256, size=(32, 8, 18), dtype=np.uint8)
    packed = oracle.pack_q4_0x4(blocks)
    assert packed.nbytes == blocks.nbytes
    np.testing.assert_array_equal(ggml_unpack_q4_0x4(packed, 8 * 32, 32), blocks)
    # a real quantized weight survives the round trip as well
    weight = oracle.quantize_q4_0(rng.standard_normal((16, 96)).astype(np.float32))
    np.testing.assert_array_equal(ggml_unpack_q4_0x4(oracle.pack_q4_0x4(weight), 96, 16), weight)


def test_unpack_rejects_bad_shapes() -> None:
    library = _native.load()
    packed = np.zeros(4 * 2 * 18, dtype=np.uint8)
    native = np.zeros_like(packed)
    bad = [
        (packed.nbytes, 64, 4, native.nbytes - 1),  # destination too small
        (packed.nbytes - 1, 64, 4, native.nbytes),  # source too small
        (packed.nbytes, 48, 4, native.nbytes),  # K % 32 != 0
        (packed.nbytes, 64, 6, native.nbytes),  # N % 4 != 0
    ]
    for packed_size, k, n, native_size in bad:
        status = library.qpucuda_ggml_unpack_q4_0x4(packed.ctypes.data, packed_size, k, n, native.ctypes.data, native_size)
        assert status == _native.Status.INVALID_ARGUMENT
