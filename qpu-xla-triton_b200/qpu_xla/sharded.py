"""Output-channel (N) split of one linear across the GPUs of a node.

The reference splits one operator between its CPU and QPU along output
columns, each side writing a disjoint column range and a host event joining
them (src/qpu_xla/models/tinyllama/quantization.py:350-514; Q4_0
``column_start/column_count``, integrations/llama_cpp/include/qpu_llama_q4_0.h:42-43).
Here the two sides become ``world_size`` GPUs, one process each: rank r holds
weight rows ``[start_r, start_r + count_r)`` (a multiple of the tile width
except for the last rank), every rank computes the same activations' product
with its slice, and one all-gather over NVLink (NCCL) joins the column blocks.
Ranks quantize identical activations with the same deterministic kernel, so
the joined output equals the single-GPU output bit for bit.
"""

from __future__ import annotations

import math
from typing import Any, Self

import numpy as np
import numpy.typing as npt

from qpu_xla.device import Device
from qpu_xla.quantization import PreparedW8A8Linear, QuantizedMatrixInt8

DEFAULT_ALIGNMENT = 256  # the tcgen05 GEMM's N tile


def shard_width(total: int, world_size: int, alignment: int) -> int:
    """Columns per rank: ceil(total / world_size) rounded up to ``alignment``."""
    if total <= 0 or world_size <= 0 or alignment <= 0:
        raise ValueError("shard_width needs positive sizes")
    return math.ceil(math.ceil(total / world_size) / alignment) * alignment


def shard_bounds(total: int, world_size: int, rank: int, alignment: int = DEFAULT_ALIGNMENT) -> tuple[int, int]:
    """``(start, count)`` of rank's disjoint column range; count may be 0 for trailing ranks."""
    if not 0 <= rank < world_size:
        raise ValueError("rank must lie in [0, world_size)")
    width = shard_width(total, world_size, alignment)
    start = min(rank * width, total)
    return start, min(start + width, total) - start


class ColumnGather:
    """All-gather of per-rank column blocks ``[rows, width]`` into ``[rows, total]``."""

    def __init__(self: Self, total: int, world_size: int, rank: int, *, group: Any = None, alignment: int = DEFAULT_ALIGNMENT) -> None:
        self.total = total
        self.world_size = world_size
        self.rank = rank
        self.group = group
        self.width = shard_width(total, world_size, alignment)
        self.start, self.count = shard_bounds(total, world_size, rank, alignment)

    def gather(self: Self, local: Any, out: Any = None) -> Any:
        """``local``: this rank's ``[rows, width]`` block (columns past ``count`` are ignored)."""
        import torch
        import torch.distributed as dist

        rows = local.shape[0]
        if tuple(local.shape) != (rows, self.width):
            raise ValueError("local block must be [rows, shard width]")
        gathered = torch.empty((self.world_size, rows, self.width), dtype=local.dtype, device=local.device)
        if dist.get_backend(self.group) == "nccl":
            dist.all_gather_into_tensor(gathered, local.contiguous(), group=self.group)
        else:
            dist.all_gather(list(gathered.unbind(0)), local.contiguous(), group=self.group)
        joined = gathered.permute(1, 0, 2).reshape(rows, self.world_size * self.width)[:, : self.total]
        if out is None:
            return joined if rows == 1 else joined.contiguous()
        out.copy_(joined)
        return out


class ShardedW8A8Linear:
    """One W8A8 linear split along N over the ranks of a process group (NCCL, one GPU per rank)."""

    def __init__(
        self: Self,
        device: Device,
        weight: QuantizedMatrixInt8,
        *,
        max_batch: int,
        bias: npt.NDArray[np.float32] | None = None,
        group: Any = None,
        alignment: int = DEFAULT_ALIGNMENT,
    ) -> None:
        import torch.distributed as dist

        self.world_size = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.gather = ColumnGather(weight.shape[0], self.world_size, self.rank, group=group, alignment=alignment)
        self.out_features = weight.shape[0]
        self.local = (
            PreparedW8A8Linear(device, weight, max_batch=max_batch, bias=bias, resident_outputs=(self.gather.start, self.gather.count))
            if self.gather.count > 0
            else None
        )
        self.device = device

    def forward_local(self: Self, source: Any) -> Any:
        """This rank's ``[rows, shard width]`` block (zero-padded past the rank's columns)."""
        import torch

        rows = source.shape[0]
        local = torch.zeros((rows, self.gather.width), dtype=torch.float32, device=source.device)
        if self.local is not None:
            self.local.forward(source, out=local[:, : self.gather.count])
        return local

    def forward(self: Self, source: Any, out: Any = None) -> Any:
        """Full ``[rows, N]`` output on every rank."""
        return self.gather.gather(self.forward_local(source), out)

    def close(self: Self) -> None:
        if self.local is not None:
            self.local.close()


class ShardedQ4_0Linear:
    """One Q4_0 x Q8_0 linear split along N over the ranks (M = 1..4 decode)."""

    def __init__(self: Self, device: Device, weight_blocks: npt.NDArray[np.uint8], *, rows: int, group: Any = None, alignment: int = 256) -> None:
        import torch.distributed as dist

        from qpu_xla.ggml import PreparedQ4_0Linear

        self.world_size = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        outputs = weight_blocks.shape[0]
        self.gather = ColumnGather(outputs, self.world_size, self.rank, group=group, alignment=alignment)
        self.local = (
            PreparedQ4_0Linear(device, weight_blocks, rows=rows, resident_column_start=self.gather.start, resident_column_count=self.gather.count)
            if self.gather.count > 0
            else None
        )

    def forward_local(self: Self, activation: Any, *, fp32_source: bool = False) -> Any:
        import torch

        rows = activation.shape[0]
        local = torch.zeros((rows, self.gather.width), dtype=torch.float32, device=activation.device)
        if self.local is not None:
            self.local.forward(activation, out=local[:, : self.gather.count], fp32_source=fp32_source)
        return local

    def forward(self: Self, activation: Any, out: Any = None, *, fp32_source: bool = False) -> Any:
        return self.gather.gather(self.forward_local(activation, fp32_source=fp32_source), out)

    def close(self: Self) -> None:
        if self.local is not None:
            self.local.close()


__all__ = ["ColumnGather", "ShardedQ4_0Linear", "ShardedW8A8Linear", "shard_bounds", "shard_width"]
