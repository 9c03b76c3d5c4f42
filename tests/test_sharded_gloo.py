"""Host logic of the output-channel split across ranks, on CPU with the gloo backend.

Two spawned ranks compute their column blocks with the oracle (standing in for
the per-GPU kernel) and join them with :class:`qpu_xla.sharded.ColumnGather`;
the joined output must equal the single-rank output bit for bit.
"""

from __future__ import annotations

import os
import socket
from pathlib import Path

import numpy as np
import pytest

from qpu_xla.sharded import shard_bounds, shard_width


def test_shard_bounds_cover_the_columns_disjointly() -> None:
    for total in (256, 2048, 5632, 8192, 11008, 28672, 300):
        for world in (1, 2, 4, 8):
            width = shard_width(total, world, 256)
            bounds = [shard_bounds(total, world, rank, 256) for rank in range(world)]
            covered = [column for start, count in bounds for column in range(start, start + count)]
            assert covered == list(range(total))
            assert all(start % 256 == 0 for start, count in bounds if count)
            assert all(count <= width for _, count in bounds)
    with pytest.raises(ValueError):
        shard_bounds(100, 2, 2)


def _free_port() -> int:
    with socket.socket() as sock:
        sock.bind(("127.0.0.1", 0))
        return int(sock.getsockname()[1])


def _rank_main(rank: int, world: int, port: int, out_dir: str) -> None:
    import sys

    repo = Path(__file__).resolve().parents[1]
    sys.path[:0] = [str(repo / "qpu-xla-triton_b200"), str(repo)]
    import torch
    import torch.distributed as dist

    from oracle import qpu_oracle as oracle
    from qpu_xla import workloads
    from qpu_xla.sharded import ColumnGather

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        case = workloads.linear_inputs(24, 96, 600, seed=11, weight_std=0.05, bias=True)
        values, scales = oracle.quantize_per_output_channel_int8(case.weight)
        gather = ColumnGather(600, world, rank, alignment=128)
        local = np.zeros((24, gather.width), dtype=np.float32)
        if gather.count:
            cols = slice(gather.start, gather.start + gather.count)
            local[:, : gather.count] = oracle.w8a8_linear(case.source, values[cols], scales[cols], case.bias[cols])
        joined = gather.gather(torch.from_numpy(local)).numpy()
        np.save(Path(out_dir) / f"rank{rank}.npy", joined)
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_join_column_blocks_bit_exactly(tmp_path: Path) -> None:
    import torch.multiprocessing as mp

    from oracle import qpu_oracle as oracle
    from qpu_xla import workloads

    world = 2
    mp.start_processes(_rank_main, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True, start_method="spawn")
    case = workloads.linear_inputs(24, 96, 600, seed=11, weight_std=0.05, bias=True)
    values, scales = oracle.quantize_per_output_channel_int8(case.weight)
    expected = oracle.w8a8_linear(case.source, values, scales, case.bias)
    for rank in range(world):
        np.testing.assert_array_equal(np.load(tmp_path / f"rank{rank}.npy"), expected)
