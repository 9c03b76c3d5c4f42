"""One rank of test_gpu_multi.py, launched by torch.distributed.run (one process per GPU).

Each rank builds the same seeded weights and activations, computes the full linear on its
own GPU with one plan (the 1-GPU result), then the N-split: the fused GEMM + all-gather
(``forward_fused`` into a ``PeerOutput``, twice into the same buffers), the same with the
copy engines doing the exchange (``forward_copied``, twice) and the NCCL all-gather path
(``forward``). All three must equal the 1-GPU result bit for bit on every rank;
a mismatch raises, the rank exits non-zero and the launcher stops the others.
"""

from __future__ import annotations

import os
import sys
from datetime import timedelta
from pathlib import Path

REPO = Path(__file__).resolve().parents[1]
for path in (str(REPO / "qpu-xla-triton_b200"), str(REPO)):
    if path not in sys.path:
        sys.path.insert(0, path)

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from oracle import qpu_oracle as oracle  # noqa: E402
from qpu_xla import Device  # noqa: E402
from qpu_xla.quantization import PreparedW8A8Linear, QuantizedMatrixInt8  # noqa: E402
from qpu_xla.sharded import PeerOutput, ShardedW8A8Linear  # noqa: E402

CASES = (
    # rows, K, N, bias: GEMM path with a ragged last shard (and empty trailing ranks at 8 GPUs),
    # a prefill-sized batch, and the GEMV path (<= 8 rows) whose peers get copies
    (300, 1000, 1000, True),
    (4096, 512, 2304, False),
    (5, 640, 1536, True),
)


def main() -> None:
    rank = int(os.environ["RANK"])
    local_rank = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local_rank)
    cuda = torch.device("cuda", local_rank)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=cuda)
    device = Device.open(device_ordinal=local_rank)
    try:
        for rows, k, n, with_bias in CASES:
            rng = np.random.default_rng(k * 7 + n)
            weight = rng.standard_normal((n, k), dtype=np.float32) * 0.05
            values, scales = oracle.quantize_per_output_channel_int8(weight)
            matrix = QuantizedMatrixInt8(values, scales)
            bias = rng.standard_normal(n, dtype=np.float32) * 0.1 if with_bias else None
            source = torch.from_numpy(rng.standard_normal((rows, k), dtype=np.float32)).to(cuda)
            full = PreparedW8A8Linear(device, matrix, max_batch=rows, bias=bias)
            expected = full.forward(source)
            # the 1-GPU result itself against the oracle (the reference's CPU arithmetic), on a row
            # sample: rows are quantized independently, so a row subset must match bit for bit
            sample = np.unique(np.linspace(0, rows - 1, num=min(rows, 64)).astype(np.int64))
            reference = oracle.w8a8_linear(source.cpu().numpy()[sample], values, scales, bias)
            if not np.array_equal(expected.cpu().numpy()[sample], reference):
                raise AssertionError(f"rank {rank}: the 1-GPU result differs from the oracle (case {rows}x{k}x{n})")
            sharded = ShardedW8A8Linear(device, matrix, max_batch=rows, bias=bias)
            output = PeerOutput(device, rows, n)
            for attempt in range(2):
                got = sharded.forward_fused(source, output)
                torch.cuda.synchronize()
                if not torch.equal(got, expected):
                    bad = int((got != expected).sum())
                    raise AssertionError(f"rank {rank}: fused all-gather differs in {bad} outputs (case {rows}x{k}x{n}, pass {attempt})")
                dist.barrier()  # every rank has read the buffers before they are written again
            streams = [torch.cuda.Stream(cuda) for _ in range(max(1, dist.get_world_size() - 1))]
            for attempt in range(2):
                got = sharded.forward_copied(source, output, streams)
                torch.cuda.synchronize()
                if not torch.equal(got, expected):
                    bad = int((got != expected).sum())
                    raise AssertionError(f"rank {rank}: copy-engine all-gather differs in {bad} outputs (case {rows}x{k}x{n}, pass {attempt})")
                dist.barrier()
            gathered = sharded.forward(source)
            torch.cuda.synchronize()
            if not torch.equal(gathered, expected):
                raise AssertionError(f"rank {rank}: NCCL all-gather differs (case {rows}x{k}x{n})")
            output.close()
            sharded.close()
            full.close()
        print(f"rank {rank}: ok", flush=True)
    finally:
        device.close()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
