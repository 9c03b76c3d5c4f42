"""Output-channel (N) split of one linear across the GPUs of a node.

The reference splits one operator between its CPU and QPU along output
columns, each side writing a disjoint column range and a host event joining
them (src/qpu_xla/models/tinyllama/quantization.py:350-514; Q4_0
``column_start/column_count``, integrations/llama_cpp/include/qpu_llama_q4_0.h:42-43).
Here the two sides become ``world_size`` GPUs, one process each: rank r holds
weight rows ``[start_r, start_r + count_r)`` (a multiple of the tile width
except for the last rank), every rank computes the same activations' product
with its slice, and the column blocks are joined over NVLink: either by the GEMM
itself (``PeerOutput`` + ``ShardedW8A8Linear.forward_fused``: the epilogue stores
each finished tile into every rank's full output, mapped with CUDA IPC, followed
by one small NCCL all-reduce as the barrier) or by an NCCL all-gather after the
GEMM (``forward``). Ranks quantize identical activations with the same
deterministic kernel, so the joined output equals the single-GPU output bit for
bit.
"""

from __future__ import annotations

import ctypes
import math
from collections.abc import Sequence
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


class PeerOutput:
    """One full ``[rows, total]`` fp32 output per rank, in device memory that every other rank
    of the group maps (``qpucuda_peer_buffer_*``, CUDA IPC), for ``forward_fused``.

    Collective: every rank of ``group`` constructs and closes it together. ``tensor`` is this
    rank's buffer as a torch view (valid until ``close``). A buffer must not be written by a new
    fused call until every rank has finished reading the previous result from it.
    """

    def __init__(self: Self, device: Device, rows: int, total: int, *, group: Any = None) -> None:
        import torch
        import torch.distributed as dist

        self.world_size = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.rows = rows
        self.total = total
        self._group = group
        self._native = device.backend.native  # type: ignore[attr-defined]
        library, context = self._native.library, self._native.handle
        pointer = ctypes.c_void_p()
        handle = ctypes.create_string_buffer(64)
        self._native.check(library.qpucuda_peer_buffer_create(context, rows * total * 4, ctypes.byref(pointer), handle), "qpucuda_peer_buffer_create")
        self._own = int(pointer.value)  # type: ignore[arg-type]
        handles: list[Any] = [None] * self.world_size
        dist.all_gather_object(handles, handle.raw, group=group)
        self._bases: dict[int, int] = {self.rank: self._own}
        self._opened: list[int] = []
        try:
            for peer, peer_handle in enumerate(handles):
                if peer == self.rank:
                    continue
                mapped = ctypes.c_void_p()
                self._native.check(library.qpucuda_peer_buffer_open(context, peer_handle, ctypes.byref(mapped)), "qpucuda_peer_buffer_open")
                self._bases[peer] = int(mapped.value)  # type: ignore[arg-type]
                self._opened.append(self._bases[peer])
        except Exception:
            self._release()
            raise
        interface = {"shape": (rows, total), "typestr": "<f4", "data": (self._own, False), "version": 3, "strides": None}
        holder = type("PeerOutputView", (), {"__cuda_array_interface__": interface})()
        self.tensor = torch.as_tensor(holder, device=device.backend.torch_device)  # type: ignore[attr-defined]
        self._closed = False

    def slice_pointers(self: Self, column_start: int) -> tuple[int, list[int]]:
        """Device addresses of column ``column_start`` of row 0: this rank's buffer, then every
        other rank's mapped buffer in rank order."""
        offset = 4 * column_start
        return self._own + offset, [self._bases[r] + offset for r in range(self.world_size) if r != self.rank]

    def push_columns(self: Self, column_start: int, column_count: int, streams: Sequence[Any], rows: int | None = None) -> None:
        """Copy columns ``[column_start, column_start + column_count)`` of the first ``rows`` rows
        (default all) of this rank's buffer into the same place of every other rank's buffer with the copy engines
        (``qpucuda_peer_copy_rows``), peer i on ``streams[i % len(streams)]`` (torch CUDA streams
        of this device, already ordered after the kernel that wrote the columns). The SMs stay free
        for the next kernel while NVLink carries the block."""
        library, context = self._native.library, self._native.handle
        pitch = 4 * self.total
        source = self._own + 4 * column_start
        peers = [r for r in range(self.world_size) if r != self.rank]
        for i, peer in enumerate(peers):
            stream = streams[i % len(streams)]
            self._native.check(
                library.qpucuda_peer_copy_rows(context, self._bases[peer] + 4 * column_start, pitch, source, pitch,
                                               4 * column_count, self.rows if rows is None else rows, stream.cuda_stream),
                "qpucuda_peer_copy_rows",
            )

    def _release(self: Self) -> None:
        library, context = self._native.library, self._native.handle
        for mapped in self._opened:
            library.qpucuda_peer_buffer_close(context, mapped)
        self._opened = []
        if self._own:
            library.qpucuda_peer_buffer_destroy(context, self._own)
            self._own = 0

    def close(self: Self) -> None:
        """Collective: no rank writes into any buffer after the first barrier, and no buffer is
        freed before every rank has unmapped it."""
        import torch
        import torch.distributed as dist

        if self._closed:
            return
        self._closed = True
        torch.cuda.synchronize()
        dist.barrier(group=self._group)
        library, context = self._native.library, self._native.handle
        for mapped in self._opened:
            library.qpucuda_peer_buffer_close(context, mapped)
        self._opened = []
        dist.barrier(group=self._group)
        del self.tensor
        library.qpucuda_peer_buffer_destroy(context, self._own)
        self._own = 0


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

    def forward_fused(self: Self, source: Any, output: PeerOutput) -> Any:
        """Full ``[rows, N]`` output on every rank, joined by the GEMM epilogue itself: this
        rank's columns are stored into every rank's ``output`` buffer as each tile finishes,
        then a one-element NCCL all-reduce on the same stream orders every rank's stores before
        anything that follows. Returns ``output.tensor``."""
        import torch
        import torch.distributed as dist

        if output.total != self.out_features or source.shape[0] > output.rows:
            raise ValueError("peer output must be [rows >= batch, out_features]")
        if self.local is not None:
            destination, peers = output.slice_pointers(self.gather.start)
            self.local.forward_fanout(source, destination, peers, output.total)
        if getattr(self, "_barrier", None) is None:
            self._barrier = torch.zeros(1, dtype=torch.float32, device=source.device)
        dist.all_reduce(self._barrier, group=self.gather.group)
        return output.tensor[: source.shape[0]]

    def forward_copied(self: Self, source: Any, output: PeerOutput, streams: Sequence[Any]) -> Any:
        """``forward_fused`` with the exchange done by the copy engines: the GEMM writes this rank's
        columns into its own ``output`` buffer only, then ``output.push_columns`` copies them to every
        other rank on ``streams`` (ordered after the GEMM); the current stream waits for those copies
        before the one-element NCCL all-reduce. Returns ``output.tensor``."""
        import torch
        import torch.distributed as dist

        if output.total != self.out_features or source.shape[0] > output.rows:
            raise ValueError("peer output must be [rows >= batch, out_features]")
        current = torch.cuda.current_stream(source.device)
        if self.local is not None and self.gather.count > 0:
            destination, _ = output.slice_pointers(self.gather.start)
            self.local.forward_fanout(source, destination, [], output.total)
            written = torch.cuda.Event()
            written.record(current)
            for side in streams:
                side.wait_event(written)
            output.push_columns(self.gather.start, self.gather.count, streams, rows=source.shape[0])
            for side in streams:
                current.wait_stream(side)
        if getattr(self, "_barrier", None) is None:
            self._barrier = torch.zeros(1, dtype=torch.float32, device=source.device)
        dist.all_reduce(self._barrier, group=self.gather.group)
        return output.tensor[: source.shape[0]]

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


__all__ = ["ColumnGather", "PeerOutput", "ShardedQ4_0Linear", "ShardedW8A8Linear", "shard_bounds", "shard_width"]
