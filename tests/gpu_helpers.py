"""Helpers for the GPU tests: call libqpucuda's C-ABI on torch CUDA tensors."""

from __future__ import annotations

import ctypes
from typing import Any

import numpy as np
import torch

from qpu_xla import _native


def to_cuda(array: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(array)).cuda()


def padded_int8(values: np.ndarray, multiple: int = 16) -> torch.Tensor:
    """int8 rows zero-padded to a multiple of 16 bytes, on the GPU."""
    rows, cols = values.shape
    padded = np.zeros((rows, (cols + multiple - 1) // multiple * multiple), dtype=np.int8)
    padded[:, :cols] = values
    return to_cuda(padded)


class Native:
    """A libqpucuda context on GPU 0 issuing on torch's current stream."""

    def __init__(self, *, failure_mask: int = 0, timeout_ns: int = 0) -> None:
        self.context = _native.NativeContext(0, timeout_ns=timeout_ns, failure_mask=failure_mask)
        self.lib = self.context.library

    @property
    def handle(self) -> int:
        return self.context.handle

    def call(self, name: str, *args: Any) -> int:
        self.context.set_stream(torch.cuda.current_stream().cuda_stream)
        return int(getattr(self.lib, name)(self.handle, *args))

    def check(self, name: str, *args: Any) -> None:
        status = self.call(name, *args)
        self.context.check(status, name)

    def sync(self) -> None:
        self.context.set_stream(torch.cuda.current_stream().cuda_stream)
        self.context.synchronize()

    def close(self) -> None:
        self.context.close()

    # -- kernels ------------------------------------------------------------------

    def quantize_rows(self, x: torch.Tensor, padded_cols: int | None = None) -> tuple[torch.Tensor, torch.Tensor]:
        rows, cols = x.shape
        padded_cols = cols if padded_cols is None else padded_cols
        q = torch.full((rows, padded_cols), 99, dtype=torch.int8, device=x.device)
        scales = torch.empty(rows, dtype=torch.float32, device=x.device)
        self.check("qpucuda_quantize_rows_int8", x.data_ptr(), x.stride(0), rows, cols, padded_cols, q.data_ptr(), q.stride(0), scales.data_ptr())
        return q, scales

    def gemm_s32(self, a: torch.Tensor, w: torch.Tensor, k: int | None = None) -> torch.Tensor:
        m, n = a.shape[0], w.shape[0]
        k = a.shape[1] if k is None else k
        acc = torch.full((m, n), -7, dtype=torch.int32, device=a.device)
        self.check("qpucuda_w8a8_gemm_s32", a.data_ptr(), a.stride(0), w.data_ptr(), w.stride(0), m, n, k, acc.data_ptr(), n)
        return acc

    def gemm_dequantize(self, a, w, row_scales, col_scales, bias=None, k=None) -> torch.Tensor:  # type: ignore[no-untyped-def]
        m, n = a.shape[0], w.shape[0]
        k = a.shape[1] if k is None else k
        out = torch.full((m, n), float("nan"), dtype=torch.float32, device=a.device)
        self.check(
            "qpucuda_w8a8_gemm_dequantize", a.data_ptr(), a.stride(0), w.data_ptr(), w.stride(0), m, n, k,
            row_scales.data_ptr(), col_scales.data_ptr(), None if bias is None else bias.data_ptr(), out.data_ptr(), n,
        )
        return out

    def gemv(self, a, w, row_scales=None, col_scales=None, bias=None) -> torch.Tensor:  # type: ignore[no-untyped-def]
        m, k = a.shape
        n = w.shape[0]
        if row_scales is None:
            acc = torch.full((m, n), -7, dtype=torch.int32, device=a.device)
            self.check("qpucuda_w8a8_gemv", a.data_ptr(), a.stride(0), w.data_ptr(), w.stride(0), m, n, k, acc.data_ptr(), n, None, None, None, None, 0)
            return acc
        out = torch.full((m, n), float("nan"), dtype=torch.float32, device=a.device)
        self.check(
            "qpucuda_w8a8_gemv", a.data_ptr(), a.stride(0), w.data_ptr(), w.stride(0), m, n, k, None, 0,
            row_scales.data_ptr(), col_scales.data_ptr(), None if bias is None else bias.data_ptr(), out.data_ptr(), n,
        )
        return out

    def dequantize(self, acc, row_scales, col_scales, bias=None) -> torch.Tensor:  # type: ignore[no-untyped-def]
        m, n = acc.shape
        out = torch.empty((m, n), dtype=torch.float32, device=acc.device)
        self.check(
            "qpucuda_w8a8_dequantize", acc.data_ptr(), n, m, n, row_scales.data_ptr(), col_scales.data_ptr(),
            None if bias is None else bias.data_ptr(), out.data_ptr(), n,
        )
        return out

    def quantize_blocks(self, x: torch.Tensor, kind: str) -> torch.Tensor:
        rows, cols = x.shape
        block = 34 if kind == "q8_0" else 18
        out = torch.zeros((rows, cols // 32, block), dtype=torch.uint8, device=x.device)
        self.check(f"qpucuda_quantize_{kind}", x.data_ptr(), x.stride(0), rows, cols, out.data_ptr())
        return out

    # -- prepared W8A8 linear -------------------------------------------------------

    def w8a8_prepare(self, values: np.ndarray, scales: np.ndarray, bias: np.ndarray | None, max_batch: int, start: int = 0, count: int = 0) -> int:
        values = np.ascontiguousarray(values)
        scales = np.ascontiguousarray(scales)
        desc = _native.W8A8LinearDesc(
            values.ctypes.data, scales.ctypes.data, None if bias is None else np.ascontiguousarray(bias).ctypes.data,
            values.shape[1], values.shape[0], max_batch, start, count, _native.MEMORY_HOST,
        )
        handle = ctypes.c_void_p()
        self.check("qpucuda_w8a8_linear_prepare", ctypes.byref(desc), ctypes.byref(handle))
        return int(handle.value)  # type: ignore[arg-type]


def max_relative_error(actual: np.ndarray, expected: np.ndarray) -> float:
    scale = float(np.max(np.abs(expected))) or 1.0
    return float(np.max(np.abs(actual.astype(np.float64) - expected.astype(np.float64)))) / scale
