#!/usr/bin/env python3
"""Headline benchmark: W8A8 GEMM TOPS (and Q4_0 GEMV GB/s) at 1/2/4/8 B200s.

Headline workload (benchmark configuration configs[4], the one the metric is quoted on
"at 1/2/4/8 GPUs"): the Llama-2-70B FFN at prefill, M = 4096 tokens, W8A8 dynamic
linear for gate (8192->28672), up (8192->28672) and down (28672->8192). Weights are
random-init ~N(0, 0.02), activations ~N(0, 1), drawn on the GPU from a fixed seed
(identical on every rank). Each projection's output channels (N) are split across the
ranks; N = 1 runs the identical inputs unsplit.

One step = for each projection: quantize the fp32 rows (int8 row-quantizer kernel) into
the plan's scratch, then the tcgen05 int8 GEMM with the fused dequant epilogue on the
rank's column shard, and (N > 1) the exchange that leaves the full [M, N] fp32 output on
every rank. From 3 GPUs on, the GEMM epilogue stores each tile into every rank's output
buffer (mapped with CUDA IPC) over NVLink as it finishes (the fused GEMM + all-gather); at
2 GPUs the GEMM writes the local buffer and the copy engines push each projection's column
block to the peer while the next projection computes (``--exchange`` overrides the
choice). One NCCL all-reduce of one element per step then orders all ranks' writes. If the
peer mapping is refused, the step falls back to an NCCL all-gather after each GEMM and the
line says so.
At N = 1 CUDA events recorded between the quantizer and the GEMM launches inside the
timed steps give the GEMM's own time, which the roofline uses.

L2 is flushed before every timed bracket, outside it: a 256 MiB write, then a 256 MiB
read of a second buffer, so the timed kernels start on a cache of clean lines; the
headline's inputs also exceed L2.

Further objects of the same JSON line time the other configurations at N = 1, each with
its own roofline (achieved / measured peak / ncu traffic per launch) and the reference's
CPU path timed on the host beside it:
  * ``q4_0_gemv`` / ``w8a8_gemv`` -- the decode of configs[4] on the same 70B shapes (Q4_0
    x Q8_0 at M = 1 and 4; W8A8 int8 GEMV at M = 1 and 8), per rank on its shard;
  * ``square`` -- configs[0-1], the reference's 64^3 and 512^3 (+bias) W8A8 cases;
  * ``tinyllama_w8a8`` -- configs[2], all seven projections of one TinyLlama layer at
    M = 1, 128 and 2048;
  * ``tinyllama_q4_0`` -- configs[3], Q4_0 x Q8_0 at M = 1 and 4 on the TinyLlama FFN
    shapes, each bracket streaming 16 distinct weight copies (the 6.5 MB weight would
    otherwise be served from L2);
  * ``llama7b_ffn`` -- the 7B FFN of configs[4] at M = 4096 (W8A8) and M = 1 (Q4_0).

``python bench.py [--gpus N --steps K --warmup W]``; for N > 1 run under
``torch.distributed.run`` (one rank per GPU). ``--impl reference`` times the reference's
own CPU implementation (the NumPy port of src/qpu_xla/models/tinyllama/quantization.py:
1065-1082) on a bounded sample.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path
from typing import Any, Callable

ROOT = Path(__file__).resolve().parent
sys.path[:0] = [str(ROOT / "qpu-xla-triton_b200"), str(ROOT)]

METRIC = "W8A8 GEMM TOPS & Q4_0 GEMV GB/s, % of B200 roofline, at 1/2/4/8 GPUs"
WORKLOAD = "llama2-70b-ffn prefill W8A8 M=4096 (gate 8192->28672, up 8192->28672, down 28672->8192) + Q4_0 decode M=1 on the same shapes"
TOKENS = 4096
SEED = 4
L2_FLUSH_BYTES = 256 << 20
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
OBJECTS = ("square", "tinyllama_w8a8", "tinyllama_q4_0", "llama7b_ffn", "q4_0_mx")
FP32_LANES = 148 * 128  # B200: SMs x fp32 lanes per SM
SM_MAX_MHZ = 1965.0
NVLINK_PEER_GBS = 770.0  # measured peer copy per direction per GPU on this pool's B200s
Q4_0_COPIES = 16  # distinct TinyLlama weight copies streamed per bracket (16 x 6.5 MB)


ONLY: set[str] = set()  # --only: restrict to some projections (profiling captures of a smaller case)


def shapes() -> list[tuple[str, int, int]]:
    from qpu_xla import workloads

    return [(s.name, s.in_features, s.out_features) for s in workloads.LLAMA2_70B_FFN if not ONLY or s.name in ONLY]


def measured_peaks() -> tuple[dict[str, float], str]:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return {k: float(data[k]) for k in ("hbm_gbs", "bf16_tflops", "bf16_tflops_sustained")}, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


def profile_traffic(name: str, key: str | None = None) -> float | None:
    """Per-launch DRAM bytes recorded by the committed ncu summary ``profiles/<name>.md``: the
    ``traffic_bytes_per_launch: <n>`` line, or with ``key`` the
    ``traffic_bytes_per_launch[<key>]: <n>`` line; None before a capture exists."""
    path = ROOT / "profiles" / f"{name}.md"
    if not path.exists():
        return None
    label = "traffic_bytes_per_launch" + (f"[{key}]" if key else "") + ":"
    for line in path.read_text().splitlines():
        if line.strip().startswith(label):
            try:
                return float(line.split(":", 1)[1].strip().split()[0])
            except ValueError:
                return None
    return None


def resolve_exchange(choice: str, world: int) -> str:
    """The N > 1 output exchange: ``auto`` takes the copy engines at 2 GPUs and the fused epilogue
    stores from 3 GPUs on (measured on B200, 70B FFN: 4507 against 4201 TOPS at 2 GPUs, 2423
    against 3614 at 4, 1578 against 3266 at 8); any other choice stands."""
    if choice != "auto":
        return choice
    return "copy" if world == 2 else "fused"


def roofline(*, kernel: str, seconds: float, ops: float, nbytes: float, int8_peak: float, hbm_peak: float,
             peak_note: str, traffic: float | None, traffic_launches: int = 1) -> dict[str, Any]:
    """Roofline of one timed launch sequence: the bound is whichever of ops / int8 peak and bytes
    / HBM peak takes longer; achieved is in that bound's unit; traffic is ncu's DRAM bytes for
    the same launches (per launch x launches), or None before a capture exists."""
    tensor_s = ops / (int8_peak * 1e12) if ops else 0.0
    hbm_s = nbytes / (hbm_peak * 1e9)
    if tensor_s >= hbm_s:
        achieved, peak, unit, bound = ops / seconds / 1e12, int8_peak, "TOPS", "tensor"
    else:
        achieved, peak, unit, bound = nbytes / seconds / 1e9, hbm_peak, "GB/s", "hbm"
    return {
        "kernel": kernel,
        "bound": bound,
        "achieved": round(achieved, 2),
        "peak": round(peak, 1),
        "unit": unit,
        "frac": round(achieved / peak, 4),
        "peak_source": peak_note,
        "algorithmic_ops": ops,
        "algorithmic_bytes": nbytes,
        "traffic": None if traffic is None else traffic * traffic_launches,
    }


# ---------------------------------------------------------------------------- clocks


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 100 ms while the timed work runs."""

    FIELDS = (
        "index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
        "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
        "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"
    )

    def __init__(self, gpu_index: int) -> None:
        self.gpu_index = gpu_index
        self.process: subprocess.Popen[str] | None = None
        self.lines: list[str] = []
        self._thread: threading.Thread | None = None

    def start(self) -> None:
        try:
            self.process = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100", "-i", str(self.gpu_index)],
                stdout=subprocess.PIPE,
                stderr=subprocess.DEVNULL,
                text=True,
            )
        except OSError:
            self.process = None
            return

        def pump() -> None:
            assert self.process is not None and self.process.stdout is not None
            for line in self.process.stdout:
                self.lines.append(line.strip())

        self._thread = threading.Thread(target=pump, daemon=True)
        self._thread.start()

    def stop(self) -> dict[str, object]:
        if self.process is not None:
            self.process.terminate()
            try:
                self.process.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.process.kill()
        if self._thread is not None:
            self._thread.join(timeout=5)
        sm: list[float] = []
        max_sm = 0.0
        power: list[float] = []
        reasons: set[str] = set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                max_sm = max(max_sm, float(parts[2]))
                power.append(float(parts[3]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower().startswith("active"):
                    reasons.add(name)
        return {
            "sm_mhz": statistics.median(sm) if sm else None,
            "sm_max_mhz": max_sm or None,
            "power_w_max": max(power) if power else None,
            "samples": len(sm),
            "reasons": sorted(reasons),
        }


# ---------------------------------------------------------------------------- ours


class Bench:
    """Device, stream, L2 flush and bracket timing shared by every object."""

    def __init__(self, device: Any, stream: Any, cuda: Any) -> None:
        import torch

        self.device = device
        self.stream = stream
        self.cuda = cuda
        self.native = device.backend.native
        self.flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=cuda)
        self.flush_clean = torch.ones(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=cuda)

    def launch(self, call: Callable[[Any, int], int]) -> None:
        """A C-ABI call on the bench stream: ``call(library, context handle) -> status``."""
        self.device.backend.launch(self.stream, lambda n: n.check(call(n.library, n.handle), "bench"))

    def prime(self, launches: int = 2) -> None:
        """Flush L2 (write one buffer larger than L2, then read another so the lines left are
        clean), then hold the stream long enough (~40 us per bracketed launch, at least 60 us)
        for the host to queue the bracketed launches before the start event executes, so no
        host launch latency falls inside a timed bracket."""
        import torch

        self.flush.zero_()
        self.flush_clean.sum()
        torch.cuda._sleep(max(120_000, 80_000 * launches))

    def brackets(self, fn: Callable[[], None], reps: int, warmup: int = 3, launches: int = 2) -> list[float]:
        """``reps`` CUDA-event brackets of ``fn`` (``launches`` kernel launches) on the bench
        stream, L2 flushed before each; ms."""
        import torch

        for _ in range(warmup):
            fn()
        events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
        for start, end in events:
            self.prime(launches)
            start.record(self.stream)
            fn()
            end.record(self.stream)
        torch.cuda.synchronize()
        return [start.elapsed_time(end) for start, end in events]

    def quantize_weight(self, weight: Any) -> Any:
        """fp32 [N, K] CUDA tensor -> QuantizedMatrixInt8 through the row-quantizer kernel."""
        import torch

        from qpu_xla.quantization import QuantizedMatrixInt8

        n, k = weight.shape
        values = torch.empty((n, k), dtype=torch.int8, device=self.cuda)
        scales = torch.empty((n,), dtype=torch.float32, device=self.cuda)
        self.launch(lambda lib, h: lib.qpucuda_quantize_rows_int8(h, weight.data_ptr(), k, n, k, k, values.data_ptr(), k, scales.data_ptr()))
        torch.cuda.synchronize()
        return QuantizedMatrixInt8(values.cpu().numpy(), scales.cpu().numpy())

    def q4_0_blocks(self, weight: Any) -> Any:
        """fp32 [N, K] CUDA tensor -> native Q4_0 blocks (host uint8 [N, K/32, 18])."""
        import torch

        n, k = weight.shape
        blocks = torch.empty((n, k // 32, 18), dtype=torch.uint8, device=self.cuda)
        self.launch(lambda lib, h: lib.qpucuda_quantize_q4_0(h, weight.data_ptr(), k, n, k, blocks.data_ptr()))
        torch.cuda.synchronize()
        return blocks.cpu().numpy()

    def q8_0(self, source: Any) -> Any:
        """fp32 [M, K] CUDA rows -> Q8_0 blocks on the device."""
        import torch

        m, k = source.shape
        act = torch.empty((m, k // 32, 34), dtype=torch.uint8, device=self.cuda)
        self.launch(lambda lib, h: lib.qpucuda_quantize_q8_0(h, source.data_ptr(), source.stride(0), m, k, act.data_ptr()))
        return act


class PrefillProjection:
    """One W8A8 projection of a prefill step: the plan, its source and output, and the two launches
    of a step (row quantizer into the plan's scratch, then the GEMM from that scratch)."""

    def __init__(self, bench: Bench, name: str, plan: Any, source: Any, out: Any, k: int, count: int) -> None:
        self.bench = bench
        self.name = name
        self.plan = plan
        self.source = source
        self.out = out
        self.k = k
        self.count = count
        self.quantized, self.row_scales = plan.scratch()
        self.handle = plan._handle

    def quantize(self) -> None:
        src, q, s, k = self.source, self.quantized, self.row_scales, self.k
        self.bench.launch(lambda lib, h: lib.qpucuda_quantize_rows_int8(
            h, src.data_ptr(), src.stride(0), src.shape[0], k, q.shape[1], q.data_ptr(), q.stride(0), s.data_ptr()))

    def gemm(self) -> None:
        handle, q, s, out, rows = self.handle, self.quantized, self.row_scales, self.out, self.source.shape[0]
        self.bench.launch(lambda lib, h: lib.qpucuda_w8a8_linear_execute_prepared_device(
            handle, q.data_ptr(), q.stride(0), s.data_ptr(), rows, out.data_ptr(), out.stride(0)))


def timed_prefill(bench: Bench, projections: list[PrefillProjection], steps: int, warmup: int,
                  extra: Callable[[], None] | None = None) -> tuple[float, list[float], list[float]]:
    """``steps`` prefill steps (each projection: quantize, GEMM), L2 flushed before each, CUDA
    events around every step and around every launch inside it. Returns (ms per step, ms per
    quantizer launch per projection, ms per GEMM launch per projection)."""
    import torch

    def step(marks: list[Any] | None) -> None:
        for i, p in enumerate(projections):
            if marks is not None:
                marks[2 * i].record(bench.stream)
            p.quantize()
            if marks is not None:
                marks[2 * i + 1].record(bench.stream)
            p.gemm()
        if marks is not None:
            marks[-1].record(bench.stream)
        if extra is not None:
            extra()

    for _ in range(warmup):
        bench.prime()
        step(None)
    torch.cuda.synchronize()
    records = []
    for _ in range(steps):
        marks = [torch.cuda.Event(enable_timing=True) for _ in range(2 * len(projections) + 1)]
        bench.prime()
        step(marks)
        records.append(marks)
    torch.cuda.synchronize()
    step_ms = statistics.mean(r[0].elapsed_time(r[-1]) for r in records)
    quant_ms, gemm_ms = [], []
    for i in range(len(projections)):
        quant_ms.append(statistics.mean(r[2 * i].elapsed_time(r[2 * i + 1]) for r in records))
        end = (lambda r, i=i: r[2 * i + 2])
        gemm_ms.append(statistics.mean(r[2 * i + 1].elapsed_time(end(r)) for r in records))
    return step_ms, quant_ms, gemm_ms


def run_ours(args: argparse.Namespace) -> None:
    import torch
    import torch.distributed as dist

    from qpu_xla import Device
    from qpu_xla.ggml import PreparedQ4_0Linear
    from qpu_xla.quantization import PreparedW8A8Linear
    from qpu_xla.sharded import ColumnGather

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}; launch N > 1 with torch.distributed.run")
    torch.cuda.set_device(local_rank)
    cuda = torch.device("cuda", local_rank)
    if world > 1:
        from datetime import timedelta

        # NCCL's communicator set-up lines (rank count, transports) go to stderr, so a scaling
        # record shows the ranks the run really had
        os.environ.setdefault("NCCL_DEBUG", "INFO")
        os.environ.setdefault("NCCL_DEBUG_SUBSYS", "INIT")
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=cuda)
    device = Device.open(device_ordinal=local_rank)
    stream = torch.cuda.current_stream(cuda)
    bench = Bench(device, stream, cuda)
    peaks, peak_kind = measured_peaks()

    # ---- inputs and plans (identical on every rank: seeded GPU generator) ----
    generator = torch.Generator(device=cuda)
    generator.manual_seed(SEED)
    projections: list[dict[str, Any]] = []
    sources: dict[int, torch.Tensor] = {}
    for name, k, n in shapes():
        if k not in sources:
            sources[k] = torch.randn((TOKENS, k), generator=generator, device=cuda, dtype=torch.float32)
        weight = torch.randn((n, k), generator=generator, device=cuda, dtype=torch.float32) * 0.02
        quantized = bench.quantize_weight(weight)
        q4_blocks = bench.q4_0_blocks(weight)
        gather = ColumnGather(n, world, rank)
        plan = PreparedW8A8Linear(device, quantized, max_batch=TOKENS, resident_outputs=(gather.start, gather.count))
        q4 = PreparedQ4_0Linear(device, q4_blocks, rows=4, resident_column_start=gather.start, resident_column_count=gather.count)
        local = torch.zeros((TOKENS, gather.width), dtype=torch.float32, device=cuda)
        full = torch.empty((TOKENS, n), dtype=torch.float32, device=cuda) if world > 1 else local
        projections.append({
            "name": name, "k": k, "n": n, "gather": gather, "plan": plan, "q4": q4, "local": local, "full": full,
            "source": sources[k], "step": PrefillProjection(bench, name, plan, sources[k], local[:, : gather.count], k, gather.count),
        })
        del weight, quantized, q4_blocks
    exchange = "none"
    copy_streams: list[Any] = []
    args.exchange = resolve_exchange(args.exchange, world)
    if world > 1 and args.exchange == "nccl":
        exchange = "NCCL all-gather after the GEMM (selected with --exchange nccl)"
        barrier_flag = None
    elif world > 1:
        from qpu_xla.sharded import PeerOutput

        exchange = "fused GEMM epilogue stores into every rank's output (CUDA IPC over NVLink) + one NCCL all-reduce per step"
        if args.exchange == "copy":
            exchange = ("GEMM into the local output, then copy-engine pushes of each projection's column block to every "
                        "peer (one stream per peer, overlapping the next projection) + one NCCL all-reduce per step")
            copy_streams = [torch.cuda.Stream(cuda) for _ in range(world - 1)]
        try:
            for p in projections:
                p["peer"] = PeerOutput(device, TOKENS, p["n"])
                p["written"] = torch.cuda.Event()
        except Exception as error:  # noqa: BLE001 - the mapping refusal is reported, not hidden
            for p in projections:
                if "peer" in p:
                    p.pop("peer").close()
            exchange = f"NCCL all-gather after the GEMM (peer mapping refused: {str(error)[:120]})"
            copy_streams.clear()
        barrier_flag = torch.zeros(1, dtype=torch.float32, device=cuda)
    torch.cuda.empty_cache()

    def step() -> None:
        fused = False
        for p in projections:
            g = p["gather"]
            if "peer" in p:
                destination, peers = p["peer"].slice_pointers(g.start)
                if copy_streams:
                    p["plan"].forward_fanout(p["source"], destination, [], p["n"])
                    p["written"].record(stream)
                    for side in copy_streams:
                        side.wait_event(p["written"])
                    p["peer"].push_columns(g.start, g.count, copy_streams)
                else:
                    p["plan"].forward_fanout(p["source"], destination, peers, p["n"])
                fused = True
                continue
            p["step"].quantize()
            p["step"].gemm()
            if world > 1:
                g.gather(p["local"], out=p["full"])
        if fused:
            for side in copy_streams:
                stream.wait_stream(side)
            dist.all_reduce(barrier_flag)  # every rank's peer stores of this step are done

    def barrier() -> None:
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(value: float) -> float:
        if world == 1:
            return value
        t = torch.tensor([value], dtype=torch.float64, device=cuda)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def sum_over_ranks(value: float) -> float:
        if world == 1:
            return value
        t = torch.tensor([value], dtype=torch.float64, device=cuda)
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        return float(t.item())

    sampler = ClockSampler(local_rank)
    if rank == 0:
        sampler.start()

    # ---- headline: K whole steps, per-step CUDA events, L2 flushed in between ----
    for _ in range(args.warmup):
        bench.prime()
        step()
    barrier()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    wall0 = time.perf_counter()
    for i in range(args.steps):
        bench.prime()
        starts[i].record(stream)
        step()
        ends[i].record(stream)
    barrier()
    wall = time.perf_counter() - wall0
    step_ms = max_over_ranks(sum(s.elapsed_time(e) for s, e in zip(starts, ends)) / args.steps)
    total_ops = sum(2.0 * TOKENS * p["n"] * p["k"] for p in projections)  # whole job, all ranks
    value_tops = total_ops / (step_ms * 1e-3) / 1e12

    # ---- the rank's own kernels: the same step on its shard with an event between every launch
    # (at N = 1 this is the headline step again; at N > 1 it leaves out the exchange) ----
    local_ms, quant_ms, gemm_ms = timed_prefill(bench, [p["step"] for p in projections], args.steps, args.warmup)
    local_ms = max_over_ranks(local_ms)
    multi_gpu = None
    if world > 1:
        received = sum(TOKENS * (p["n"] - p["gather"].count) * 4 for p in projections)
        multi_gpu = {
            "kernel_ms_per_step": round(local_ms, 4),
            "exchange_ms_per_step": round(step_ms - local_ms, 4),
            "end_to_end_ms_per_step": round(step_ms, 4),
            "exchange": exchange,
            "received_bytes_per_rank_step": received,
            "received_gbs_per_rank": round(received / (step_ms * 1e-3) / 1e9, 1),
            "note": "kernel = quantize + GEMM on the rank's column shard alone; exchange = the step's extra time "
            "over that (the fused epilogue overlaps the peer stores with the GEMM, so this is the exposed part)",
        }
    # Roofline of the fused GEMM + all-gather: the step cannot beat the slower of the rank's GEMM
    # work at the int8 peak and the fp32 outputs every rank must receive over NVLink (peer-copy
    # bandwidth measured on this pool, per direction per GPU); filled in below once the peak is known.
    rank_gemm_ops = sum(2.0 * TOKENS * p["gather"].count * p["k"] for p in projections)
    gemm_seconds = sum(gemm_ms) * 1e-3
    achieved_tops = rank_gemm_ops / gemm_seconds / 1e12 if gemm_seconds > 0 else 0.0
    achieved_tops = -max_over_ranks(-achieved_tops)  # the slowest rank's rate

    # ---- the library's int8 rate on this GPU, as the roofline's denominator ----
    # cuBLASLt's int8 GEMM (torch._int_mm, int32 output: the same output bytes as the fp32
    # dequantized output) on each of the rank's projection shapes, random int8 operands, same L2
    # protocol. B200's int8 rate is nominally twice bf16; measured here it runs above twice the
    # measured bf16 burst, so the larger of the two is the peak the GEMM is judged against.
    library_ms = []
    for p in projections:
        a8 = torch.randint(-127, 128, (TOKENS, p["k"]), dtype=torch.int8, device=cuda)
        w8 = torch.randint(-127, 128, (p["gather"].count, p["k"]), dtype=torch.int8, device=cuda)
        library_ms.append(statistics.mean(bench.brackets(lambda a8=a8, w8=w8: torch._int_mm(a8, w8.t()), 10)))
        del a8, w8
    torch.cuda.empty_cache()
    library_tops = max_over_ranks(rank_gemm_ops / (sum(library_ms) * 1e-3) / 1e12)
    bf16_doubled = 2.0 * peaks["bf16_tflops"]
    int8_peak = max(bf16_doubled, library_tops)
    if multi_gpu is not None:
        compute_ms = rank_gemm_ops / (int8_peak * 1e12) * 1e3
        link_ms = multi_gpu["received_bytes_per_rank_step"] / (NVLINK_PEER_GBS * 1e9) * 1e3
        target_ms = max(compute_ms, link_ms)
        multi_gpu["roofline"] = {
            "bound": "nvlink" if link_ms >= compute_ms else "tensor",
            "target_ms_per_step": round(target_ms, 4),
            "compute_ms_at_peak": round(compute_ms, 4),
            "receive_ms_at_link": round(link_ms, 4),
            "link_gbs": NVLINK_PEER_GBS,
            "link_source": "peer copy per direction per GPU measured on this pool (nominal NVLink 5: 900 GB/s)",
            "frac": round(target_ms / step_ms, 4),
        }
    int8_note = (f"the larger of cuBLASLt int8 (torch._int_mm) measured live on the 70B FFN shapes ({library_tops:.1f} TOPS) "
                 f"and 2 x {peak_kind} cuBLAS bf16 burst ({bf16_doubled:.1f} TOPS)")
    hbm_note = f"{peak_kind} STREAM-style copy"

    # ---- Q4_0 x Q8_0 decode (M = 1 and 4) on the 70B shapes, Q8_0 activations on the device ----
    # One decode step of the FFN = gate, up and down back to back on the stream. The three weight
    # matrices (3 x 132 MB at full width) exceed L2, and L2 is flushed before every bracket.
    reps = 20
    q4_rows: dict[str, dict[str, float]] = {}
    q4_alone: list[float] = []
    for rows in (1, 4):
        q4_inputs = []
        q4_bytes_rank = 0.0
        for p in projections:
            g = p["gather"]
            act = bench.q8_0(p["source"][:rows])
            out = torch.empty((rows, g.width), dtype=torch.float32, device=cuda)
            q4_inputs.append((p["q4"], act, out[:, : g.count]))
            q4_bytes_rank += 18.0 * g.count * p["k"] / 32 + 34.0 * rows * p["k"] / 32 + 4.0 * rows * g.count

        def decode_ffn(q4_inputs: list[Any] = q4_inputs) -> None:
            for q4, act, out in q4_inputs:
                q4.forward(act, out=out)

        q4_ms = statistics.mean(bench.brackets(decode_ffn, reps, launches=len(q4_inputs)))
        q4_seconds = max_over_ranks(q4_ms * 1e-3)
        q4_rows[str(rows)] = {
            "value": round(sum_over_ranks(q4_bytes_rank) / q4_seconds / 1e9, 1),
            "rank_gbs": round(q4_bytes_rank / (q4_ms * 1e-3) / 1e9, 1),
            "us_per_decode_ffn": round(q4_ms * 1e3, 2),
            "frac": round(q4_bytes_rank / (q4_ms * 1e-3) / 1e9 / peaks["hbm_gbs"], 4),
        }
        if rows == 1:
            # each projection alone in its own bracket (includes one bracket's fixed event overhead)
            for q4, act, out in q4_inputs:
                q4_alone.append(statistics.mean(bench.brackets(lambda q4=q4, act=act, out=out: q4.forward(act, out=out), reps)))

    # ---- W8A8 decode (rows <= 8 take the int8 GEMV): the prefill plans at M = 1 and M = 8,
    # fp32 rows on the device (row quantizer + GEMV per projection), L2 flushed per bracket.
    # Algorithmic bytes per projection: N*K weights + M*K activations + 4(N + M + M*N). ----
    w8a8_gemv: dict[str, dict[str, float]] = {}
    for gemv_rows in (1, 8):

        def decode_w8a8(rows: int = gemv_rows) -> None:
            for p in projections:
                p["plan"].forward(p["source"][:rows], out=p["local"][:rows, : p["gather"].count])

        gemv_bytes_rank = sum(
            float(p["gather"].count) * p["k"] + gemv_rows * p["k"] + 4.0 * (p["gather"].count + gemv_rows + gemv_rows * p["gather"].count)
            for p in projections
        )
        gemv_step_ms = max_over_ranks(statistics.mean(bench.brackets(decode_w8a8, reps, launches=2 * len(projections))))
        w8a8_gemv[str(gemv_rows)] = {
            "value": round(sum_over_ranks(gemv_bytes_rank) / (gemv_step_ms * 1e-3) / 1e9, 1),
            "rank_gbs": round(gemv_bytes_rank / (gemv_step_ms * 1e-3) / 1e9, 1),
            "us_per_decode_ffn": round(gemv_step_ms * 1e3, 2),
            "frac": round(gemv_bytes_rank / (gemv_step_ms * 1e-3) / 1e9 / peaks["hbm_gbs"], 4),
        }

    # ---- the other configurations (N = 1 only; they are single-GPU configurations) ----
    objects: dict[str, Any] = {}
    wanted = [o for o in OBJECTS if not args.objects or o in args.objects]
    if world == 1:
        for name in wanted:
            objects[name] = OBJECT_RUNNERS[name](bench, int8_peak, peaks["hbm_gbs"], int8_note, hbm_note)
            torch.cuda.empty_cache()

    clocks = sampler.stop() if rank == 0 else {}

    # ---- end to end through the C-ABI with host (pinned) buffers ----
    e2e = None
    if not args.no_e2e:
        host_sources = {k: torch.empty((TOKENS, k), dtype=torch.float32, pin_memory=True) for k in sources}
        for k, t in sources.items():
            host_sources[k].copy_(t)
        host_out = [torch.empty((TOKENS, p["gather"].count), dtype=torch.float32, pin_memory=True) for p in projections]
        torch.cuda.synchronize()

        def e2e_step() -> None:
            # all three projections queued before the first wait: each plan's device-to-host copies
            # overlap the next projection's host-to-device copies and kernels
            submissions = [p["plan"].submit_direct(host_sources[p["k"]].numpy(), out.numpy()) for p, out in zip(projections, host_out)]
            for submission in submissions:
                submission.wait()

        e2e_step()
        barrier()
        e2e_steps = max(1, min(args.steps, 5))
        t0 = time.perf_counter()
        for _ in range(e2e_steps):
            e2e_step()
        e2e_seconds = max_over_ranks((time.perf_counter() - t0) / e2e_steps)
        h2d = sum(TOKENS * p["k"] * 4 for p in projections)
        d2h = sum(TOKENS * p["gather"].count * 4 for p in projections)
        e2e = {
            "value": total_ops / e2e_seconds / 1e12,
            "unit": "TOPS",
            "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h,
            "ms_per_step": e2e_seconds * 1e3,
            "path": "qpucuda_w8a8_linear_submit_direct for gate, up and down, then their waits (page-locked host "
            "source and destination, copies by DMA on each plan's copy streams overlapping the kernels and the other "
            "projections' copies) per rank on its column shard; host wall clock, max over ranks",
        }

    cpu_baseline = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu_baseline = cpu_reference_sample(target_seconds=args.cpu_seconds)
        cpu_baseline["torch_int32"] = cpu_torch_int32_sample(workload_shapes=shapes(), tokens=TOKENS, target_seconds=args.cpu_seconds / 4)
        for name, entry in objects.items():
            entry["cpu"] = OBJECT_CPU[name](args.cpu_seconds / 5)

    traffic = profile_traffic("w8a8_gemm_sm100_70b_ffn")
    line = {
        "metric": METRIC,
        "value": round(value_tops, 3),
        "unit": "TOPS",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(step_ms, 4),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "int8",
        "data": "synthetic: seeded N(0,1) activations, N(0,0.02) random-init weights (torch CUDA generator, seed 4)",
        "config": {
            "workload": WORKLOAD,
            "tokens": TOKENS,
            "projections": [f"{name} {k}->{n}" for name, k, n in shapes()],
            "parallelism": f"output-channel split x{world}" + (f" + {exchange}" if world > 1 else ""),
            "l2": "flushed before every timed step or bracket (256 MiB write, then 256 MiB read of a second buffer; outside the CUDA-event brackets); the headline's inputs exceed L2",
            "timing": "per-step CUDA events on the launching stream, summed over K steps, max over ranks",
            "wall_s_timed_loop": round(wall, 4),
        },
        "gpu_launches": 2 * len(projections) * args.steps,
        "roofline": {
            "kernel": "w8a8_gemm_sm100 (tcgen05 kind::i8, fused dequant)",
            "bound": "tensor",
            "achieved": round(achieved_tops, 2),
            "peak": round(int8_peak, 1),
            "unit": "TOPS",
            "frac": round(achieved_tops / int8_peak, 4),
            "peak_source": int8_note,
            "library_int8_tops": round(library_tops, 1),
            "library_int8_ms_per_projection": [round(x, 4) for x in library_ms],
            "peak_2x_bf16": round(bf16_doubled, 1),
            "traffic": traffic,
            "algorithmic_ops_per_rank_step": rank_gemm_ops,
            "gemm_ms_per_projection": [round(x, 4) for x in gemm_ms],
            "gemm_timing": "CUDA events recorded between the row-quantizer and GEMM launches inside the timed steps (L2 flushed before each step)",
            "row_quantizer_ms_per_projection": [round(x, 4) for x in quant_ms],
            "row_quantizer_gbs": [round((4.0 + 1.0) * TOKENS * p["k"] / (ms * 1e-3) / 1e9, 1) for p, ms in zip(projections, quant_ms)],
            "row_quantizer_traffic": [profile_traffic("quantize_rows_int8_70b_ffn", f"k{p['k']}") for p in projections],
        },
        "q4_0_gemv": {
            "metric": "Q4_0 x Q8_0 GEMV GB/s (whole job), one decode FFN step (gate, up, down) per bracket, at M = 1 and 4",
            "value": q4_rows["1"]["value"],
            "unit": "GB/s",
            "rows": q4_rows,
            "roofline": {
                "kernel": "q4_0_direct_kernel (dp4a, prepared nibble layout, two columns per warp)",
                "bound": "hbm",
                "achieved": q4_rows["1"]["rank_gbs"],
                "peak": peaks["hbm_gbs"],
                "unit": "GB/s",
                "frac": q4_rows["1"]["frac"],
                "peak_source": hbm_note,
                "traffic": profile_traffic("q4_0_gemv_70b_decode"),
            },
            "us_per_decode_ffn": q4_rows["1"]["us_per_decode_ffn"],
            "us_per_projection_alone": [round(x * 1e3, 2) for x in q4_alone],
        },
        "w8a8_gemv": {
            "metric": "W8A8 decode GB/s (whole job), one FFN step (gate, up, down: row quantization + int8 GEMV; at M = 1 the GEMV quantizes rows of up to 8192 columns itself) per bracket, at M = 1 and M = 8",
            "value": w8a8_gemv["1"]["value"],
            "unit": "GB/s",
            "rows": w8a8_gemv,
            "roofline": {
                "kernel": "w8a8_gemv_kernel (dp4a, persistent balanced grid, split-K across a CTA's warps; at M = 1 and K <= 8192 it quantizes the row itself)",
                "bound": "hbm",
                "achieved": w8a8_gemv["1"]["rank_gbs"],
                "peak": peaks["hbm_gbs"],
                "unit": "GB/s",
                "frac": w8a8_gemv["1"]["frac"],
                "peak_source": hbm_note,
                "traffic": profile_traffic("objects_traffic", "w8a8_gemv_70b_decode"),
            },
        },
        "clocks": clocks,
    }
    line.update(objects)
    if multi_gpu is not None:
        line["multi_gpu"] = multi_gpu
    if e2e is not None:
        line["e2e"] = e2e
    if cpu_baseline is not None:
        line["cpu_baseline"] = cpu_baseline
    if rank == 0:
        print(json.dumps(line), flush=True)
    for p in projections:
        if "peer" in p:
            p["peer"].close()
        p["plan"].close()
        p["q4"].close()
    device.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


# ---------------------------------------------------------------------------- objects (N = 1)


def object_square(bench: Bench, int8_peak: float, hbm_peak: float, int8_note: str, hbm_note: str) -> dict[str, Any]:
    """configs[0-1]: the reference's square W8A8 cases (64^3; 512^3 with bias) through the
    prepared plan, one call (row quantizer + GEMM) per bracket."""
    import torch

    from qpu_xla import workloads
    from qpu_xla.quantization import PreparedW8A8Linear, quantize_per_output_channel_int8

    result: dict[str, Any] = {"metric": "W8A8 linear (quantize + GEMM + dequant) per call, M = K = N", "unit": "TOPS"}
    for size in (64, 512):
        case = workloads.square_case(size)
        weight = quantize_per_output_channel_int8(case.weight, device=bench.device)
        src = torch.from_numpy(case.source).to(bench.cuda)
        dst = torch.empty((size, size), dtype=torch.float32, device=bench.cuda)
        with PreparedW8A8Linear(bench.device, weight, max_batch=size, bias=case.bias) as plan:
            ms = statistics.median(bench.brackets(lambda plan=plan: plan.forward(src, out=dst), 50))
        ops = 2.0 * size**3
        nbytes = 4.0 * size * size * 2 + size * size + 4.0 * (2 * size + (size if case.bias is not None else 0))
        result[str(size)] = {
            "value": round(ops / (ms * 1e-3) / 1e12, 4),
            "us_per_call": round(ms * 1e3, 2),
            "bias": case.bias is not None,
            "roofline": roofline(kernel="row quantizer + w8a8_gemm_sm100 (one tile)", seconds=ms * 1e-3, ops=ops, nbytes=nbytes,
                                 int8_peak=int8_peak, hbm_peak=hbm_peak, peak_note=int8_note,
                                 traffic=profile_traffic("objects_traffic", f"square_{size}")),
            "note": "two launches of a few microseconds each: launch latency bounds this size, not the tensor pipe or HBM",
        }
    result["value"] = result["512"]["value"]
    return result


def object_tinyllama_w8a8(bench: Bench, int8_peak: float, hbm_peak: float, int8_note: str, hbm_note: str) -> dict[str, Any]:
    """the seven projections of one TinyLlama layer (q, k, v, o, gate, up, down) back to
    back per bracket, at M = 1, 128 and 2048; random-init weights ~N(0, 0.02)."""
    import torch

    from qpu_xla import workloads
    from qpu_xla.quantization import PreparedW8A8Linear, quantize_per_output_channel_int8

    shapes7 = workloads.TINYLLAMA_LAYER
    plans = []
    for shape in shapes7:
        case = workloads.tinyllama_case(shape, workloads.TINYLLAMA_TOKENS[-1])
        plans.append(PreparedW8A8Linear(bench.device, quantize_per_output_channel_int8(case.weight, device=bench.device),
                                        max_batch=max(workloads.TINYLLAMA_TOKENS)))
    result: dict[str, Any] = {"metric": "TinyLlama layer, 7 W8A8 projections per bracket", "unit": "TOPS", "tokens": {}}
    try:
        for tokens in workloads.TINYLLAMA_TOKENS:
            sources = [torch.from_numpy(workloads.tinyllama_case(shape, tokens).source).to(bench.cuda) for shape in shapes7]
            outs = [torch.empty((tokens, shape.out_features), dtype=torch.float32, device=bench.cuda) for shape in shapes7]

            def layer(sources: list[Any] = sources, outs: list[Any] = outs) -> None:
                for plan, src, out in zip(plans, sources, outs):
                    plan.forward(src, out=out)

            ms = statistics.median(bench.brackets(layer, 20, launches=2 * len(plans)))
            ops = sum(2.0 * tokens * s.in_features * s.out_features for s in shapes7)
            k16 = [((s.in_features + 15) // 16) * 16 for s in shapes7]
            nbytes = sum(s.out_features * k + tokens * s.in_features * 4.0 + tokens * k + 4.0 * (s.out_features + tokens + tokens * s.out_features)
                         for s, k in zip(shapes7, k16))
            path = "row quantizer + w8a8_gemv_kernel" if tokens <= 8 else "row quantizer + w8a8_gemm_sm100"
            result["tokens"][str(tokens)] = {
                "tops": round(ops / (ms * 1e-3) / 1e12, 2),
                "gbs": round(nbytes / (ms * 1e-3) / 1e9, 1),
                "us_per_layer": round(ms * 1e3, 2),
                "roofline": roofline(kernel=path, seconds=ms * 1e-3, ops=ops, nbytes=nbytes, int8_peak=int8_peak, hbm_peak=hbm_peak,
                                     peak_note=int8_note if ops / (int8_peak * 1e12) >= nbytes / (hbm_peak * 1e9) else hbm_note,
                                     traffic=profile_traffic("objects_traffic", f"tinyllama_w8a8_m{tokens}")),
            }
            del sources, outs
    finally:
        for plan in plans:
            plan.close()
    result["value"] = result["tokens"]["2048"]["tops"]
    result["merged"] = tinyllama_merged(bench, int8_peak, hbm_peak, int8_note, hbm_note)
    return result


def tinyllama_merged(bench: Bench, int8_peak: float, hbm_peak: float, int8_note: str, hbm_note: str) -> dict[str, Any]:
    """The same seven projections as four plans: q/k/v and gate/up read one input each in a layer,
    so each trio or pair runs as one MergedW8A8Linear (one row quantization, one GEMM or GEMV over
    the stacked output channels); o and down stay single. Same weights and outputs column for column."""
    import torch

    from qpu_xla import workloads
    from qpu_xla.quantization import MergedW8A8Linear, quantize_per_output_channel_int8

    shapes7 = workloads.TINYLLAMA_LAYER
    groups = ((0, 1, 2), (3,), (4, 5), (6,))
    weights = [quantize_per_output_channel_int8(workloads.tinyllama_case(s, workloads.TINYLLAMA_TOKENS[-1]).weight, device=bench.device)
               for s in shapes7]
    plans = [MergedW8A8Linear(bench.device, [weights[i] for i in g], max_batch=max(workloads.TINYLLAMA_TOKENS)) for g in groups]
    result: dict[str, Any] = {
        "groups": ["q+k+v", "o", "gate+up", "down"],
        "note": "q/k/v share the layer input and gate/up the FFN input, so each group is one row quantization and one "
                "GEMM/GEMV over the stacked output channels (8 launches per layer instead of 14); outputs equal the "
                "seven separate plans bit for bit",
        "tokens": {},
    }
    try:
        for tokens in workloads.TINYLLAMA_TOKENS:
            sources = [torch.from_numpy(workloads.tinyllama_case(shapes7[g[0]], tokens).source).to(bench.cuda) for g in groups]
            outs = [torch.empty((tokens, plan.output_count), dtype=torch.float32, device=bench.cuda) for plan in plans]

            def layer(sources: list[Any] = sources, outs: list[Any] = outs) -> None:
                for plan, src, out in zip(plans, sources, outs):
                    plan.plan.forward(src, out=out)

            ms = statistics.median(bench.brackets(layer, 20, launches=2 * len(plans)))
            ops = sum(2.0 * tokens * s.in_features * s.out_features for s in shapes7)
            nbytes = 0.0
            for g in groups:
                k = shapes7[g[0]].in_features
                n = sum(shapes7[i].out_features for i in g)
                k16 = (k + 15) // 16 * 16
                nbytes += n * k16 + tokens * k * 4.0 + tokens * k16 + 4.0 * (n + tokens + tokens * n)
            path = "row quantizer + w8a8_gemv (merged sections)" if tokens <= 8 else "row quantizer + w8a8_gemm_sm100 (merged sections)"
            result["tokens"][str(tokens)] = {
                "tops": round(ops / (ms * 1e-3) / 1e12, 2),
                "gbs": round(nbytes / (ms * 1e-3) / 1e9, 1),
                "us_per_layer": round(ms * 1e3, 2),
                "roofline": roofline(kernel=path, seconds=ms * 1e-3, ops=ops, nbytes=nbytes, int8_peak=int8_peak, hbm_peak=hbm_peak,
                                     peak_note=int8_note if ops / (int8_peak * 1e12) >= nbytes / (hbm_peak * 1e9) else hbm_note,
                                     traffic=None),
            }
            del sources, outs
    finally:
        for plan in plans:
            plan.close()
    return result


def object_tinyllama_q4_0(bench: Bench, int8_peak: float, hbm_peak: float, int8_note: str, hbm_note: str) -> dict[str, Any]:
    """Q4_0 x Q8_0 at M = 1 and 4 on the TinyLlama FFN shapes. Each weight is 6.5 MB,
    so a bracket streams Q4_0_COPIES distinct prepared copies of it (one launch each, L2 flushed
    before the bracket): every copy comes from DRAM."""
    import torch

    from qpu_xla import workloads
    from qpu_xla.ggml import PreparedQ4_0Linear

    result: dict[str, Any] = {"metric": f"Q4_0 x Q8_0 GB/s, {Q4_0_COPIES} weight copies per bracket", "unit": "GB/s", "shapes": {}}
    for shape in workloads.TINYLLAMA_Q4_0_SHAPES:
        _, weight = workloads.q4_0_case(shape, 1)
        blocks = bench.q4_0_blocks(torch.from_numpy(weight).to(bench.cuda))
        copies = [PreparedQ4_0Linear(bench.device, blocks, rows=4) for _ in range(Q4_0_COPIES)]
        entry: dict[str, Any] = {}
        try:
            for rows in (1, 4):
                source, _ = workloads.q4_0_case(shape, rows)
                act = bench.q8_0(torch.from_numpy(source).to(bench.cuda))
                out = torch.empty((rows, shape.out_features), dtype=torch.float32, device=bench.cuda)

                def run(act: Any = act, out: Any = out) -> None:
                    for plan in copies:
                        plan.forward(act, out=out)

                ms = statistics.median(bench.brackets(run, 20, launches=len(copies)))
                per_launch = 18.0 * shape.out_features * shape.in_features / 32 + 34.0 * rows * shape.in_features / 32 + 4.0 * rows * shape.out_features
                seconds = ms * 1e-3 / Q4_0_COPIES
                entry[str(rows)] = {
                    "gbs": round(per_launch / seconds / 1e9, 1),
                    "us_per_launch": round(seconds * 1e6, 2),
                    "roofline": roofline(kernel="q4_0_direct_kernel", seconds=seconds, ops=0.0, nbytes=per_launch, int8_peak=int8_peak,
                                         hbm_peak=hbm_peak, peak_note=hbm_note,
                                         traffic=profile_traffic("objects_traffic", f"tinyllama_q4_0_{shape.name}_m{rows}")),
                }
        finally:
            for plan in copies:
                plan.close()
        result["shapes"][f"{shape.name} {shape.in_features}->{shape.out_features}"] = entry
    first = next(iter(result["shapes"].values()))
    result["value"] = first["1"]["gbs"]
    return result


def object_llama7b_ffn(bench: Bench, int8_peak: float, hbm_peak: float, int8_note: str, hbm_note: str) -> dict[str, Any]:
    """configs[4]'s 7B FFN (4096 -> 11008 -> 4096): W8A8 prefill at M = 4096 (the headline's step,
    events between launches) and the Q4_0 decode FFN at M = 1 (76 MB of weights per bracket)."""
    import torch

    from qpu_xla import workloads
    from qpu_xla.ggml import PreparedQ4_0Linear
    from qpu_xla.quantization import PreparedW8A8Linear

    generator = torch.Generator(device=bench.cuda)
    generator.manual_seed(SEED + 3)
    prefill, q4_plans, keep = [], [], []
    srcs: dict[int, Any] = {}
    for shape in workloads.LLAMA2_7B_FFN:
        k, n = shape.in_features, shape.out_features
        if k not in srcs:
            srcs[k] = torch.randn((TOKENS, k), generator=generator, device=bench.cuda, dtype=torch.float32)
        weight = torch.randn((n, k), generator=generator, device=bench.cuda, dtype=torch.float32) * 0.02
        plan = PreparedW8A8Linear(bench.device, bench.quantize_weight(weight), max_batch=TOKENS)
        out = torch.empty((TOKENS, n), dtype=torch.float32, device=bench.cuda)
        prefill.append(PrefillProjection(bench, shape.name, plan, srcs[k], out, k, n))
        q4_plans.append(PreparedQ4_0Linear(bench.device, bench.q4_0_blocks(weight), rows=1))
        keep.append(out)
        del weight
    try:
        step_ms, quant_ms, gemm_ms = timed_prefill(bench, prefill, 10, 3)
        ops = [2.0 * TOKENS * p.count * p.k for p in prefill]
        decode = []
        q4_bytes = 0.0
        for shape, q4 in zip(workloads.LLAMA2_7B_FFN, q4_plans):
            act = bench.q8_0(srcs[shape.in_features][:1])
            decode.append((q4, act, torch.empty((1, shape.out_features), dtype=torch.float32, device=bench.cuda)))
            q4_bytes += 18.0 * shape.out_features * shape.in_features / 32 + 34.0 * shape.in_features / 32 + 4.0 * shape.out_features

        def decode_ffn() -> None:
            for q4, act, out in decode:
                q4.forward(act, out=out)

        q4_ms = statistics.median(bench.brackets(decode_ffn, 20, launches=len(decode)))
    finally:
        for p in prefill:
            p.plan.close()
        for q4 in q4_plans:
            q4.close()
    return {
        "metric": "Llama-2-7B FFN: W8A8 prefill TOPS at M = 4096, Q4_0 decode GB/s at M = 1",
        "value": round(sum(ops) / (step_ms * 1e-3) / 1e12, 2),
        "unit": "TOPS",
        "ms_per_step": round(step_ms, 4),
        "gemm_ms_per_projection": [round(x, 4) for x in gemm_ms],
        "row_quantizer_ms_per_projection": [round(x, 4) for x in quant_ms],
        "roofline": roofline(kernel="w8a8_gemm_sm100 (in-step events)", seconds=sum(gemm_ms) * 1e-3, ops=sum(ops), nbytes=0.0,
                             int8_peak=int8_peak, hbm_peak=hbm_peak, peak_note=int8_note,
                             traffic=profile_traffic("objects_traffic", "llama7b_gemm_step")),
        "q4_0_decode": {
            "gbs": round(q4_bytes / (q4_ms * 1e-3) / 1e9, 1),
            "us_per_decode_ffn": round(q4_ms * 1e3, 2),
            "roofline": roofline(kernel="q4_0_direct_kernel (gate, up, down)", seconds=q4_ms * 1e-3, ops=0.0, nbytes=q4_bytes,
                                 int8_peak=int8_peak, hbm_peak=hbm_peak, peak_note=hbm_note,
                                 traffic=profile_traffic("objects_traffic", "llama7b_q4_0_decode_ffn")),
        },
    }


def object_q4_0_mx(bench: Bench, int8_peak: float, hbm_peak: float, int8_note: str, hbm_note: str) -> dict[str, Any]:
    """The reference's MX path (Q4_0 x Q8_0 with rows > 4, exact per-block scaling) at prefill size:
    M = 4096 rows on the 70B gate (8192 -> 28672) and down (28672 -> 8192) shapes, Q8_0 activations
    on the device; one projection per bracket (split activation + tcgen05 MX kernel)."""
    import torch

    from qpu_xla.ggml import PreparedQ4_0Linear

    rows = TOKENS
    generator = torch.Generator(device=bench.cuda)
    generator.manual_seed(SEED + 5)
    result: dict[str, Any] = {"metric": "Q4_0 x Q8_0 MX path TOPS (2MNK / time), M = 4096", "unit": "TOPS", "shapes": {}}
    for name, k, n in (("gate_proj", 8192, 28672), ("down_proj", 28672, 8192)):
        weight = torch.randn((n, k), generator=generator, device=bench.cuda, dtype=torch.float32) * 0.02
        plan = PreparedQ4_0Linear(bench.device, bench.q4_0_blocks(weight), rows=rows)
        del weight
        source = torch.randn((rows, k), generator=generator, device=bench.cuda, dtype=torch.float32)
        act = bench.q8_0(source)
        del source
        out = torch.empty((rows, n), dtype=torch.float32, device=bench.cuda)
        try:
            ms = statistics.median(bench.brackets(lambda plan=plan, act=act, out=out: plan.forward(act, out=out), 5))
        finally:
            plan.close()
        ops = 2.0 * rows * n * k
        # The fp32 side: 4 roundings per (row, column, block) on 148 SMs x 128 fp32 lanes at the
        # maximum SM clock, expressed in the metric's int ops (2 x 32 per (row, column, block)).
        fp32_bound_tops = FP32_LANES * SM_MAX_MHZ * 1e6 / 4.0 * 64.0 / 1e12
        result["shapes"][f"{name} {k}->{n}"] = {
            "tops": round(ops / (ms * 1e-3) / 1e12, 1),
            "ms_per_call": round(ms, 4),
            "roofline": roofline(kernel="activation split + q4_0_mx_sm100_kernel (tcgen05 kind::i8, one MMA per block)",
                                 seconds=ms * 1e-3, ops=ops, nbytes=0.0, int8_peak=int8_peak, hbm_peak=hbm_peak,
                                 peak_note=int8_note,
                                 traffic=profile_traffic("q4_0_mx_sm100_70b_gate_m4096") if name == "gate_proj" else None),
            "fp32_scaling_bound": {
                "tops": round(fp32_bound_tops, 1),
                "frac": round(ops / (ms * 1e-3) / 1e12 / fp32_bound_tops, 4),
                "source": "nominal: 148 SMs x 128 fp32 lanes x the maximum SM clock, 4 fp32 roundings per (row, column, block)",
            },
        }
        del act, out
    result["value"] = next(iter(result["shapes"].values()))["tops"]
    result["note"] = ("the exact per-block fp32 scaling (((float)dot * d_a) * d_w, then a sequential fp32 add per "
                      "output and block) runs on the CUDA cores and bounds this path, not the tensor pipe")
    return result


OBJECT_RUNNERS: dict[str, Callable[..., dict[str, Any]]] = {
    "square": object_square,
    "tinyllama_w8a8": object_tinyllama_w8a8,
    "tinyllama_q4_0": object_tinyllama_q4_0,
    "llama7b_ffn": object_llama7b_ffn,
    "q4_0_mx": object_q4_0_mx,
}


# ---------------------------------------------------------------------------- reference (CPU)


_CPU_SAMPLES: dict[tuple[tuple[str, int, int], ...], list[tuple[object, object, object]]] = {}
CPU_COLUMNS = 1024


def host_cores() -> int:
    return len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)


def cpu_reference_sample(*, target_seconds: float, rows: int | None = None,
                         workload_shapes: list[tuple[str, int, int]] | None = None, tokens: int = TOKENS,
                         label: str = "70B FFN") -> dict[str, object]:
    """The reference's CPU path (NumPy port of quantization.py:1065-1082: per-row quantization,
    int32 matmul, fp32 dequant) on a bounded sample of a prefill workload: ``rows`` token rows
    (sized to ``target_seconds``, at most ``tokens``) x at most 1024 output columns of each
    projection at its full K, the matmul split over all host threads."""
    import numpy as np

    from oracle import qpu_oracle as oracle

    cores = host_cores()
    workload_shapes = shapes() if workload_shapes is None else workload_shapes
    key = tuple(workload_shapes)
    if key not in _CPU_SAMPLES:
        rng = np.random.default_rng(SEED)
        samples = []
        for _, k, n in workload_shapes:
            x = rng.standard_normal((tokens, k), dtype=np.float32)
            w = (rng.standard_normal((min(CPU_COLUMNS, n), k), dtype=np.float32) * np.float32(0.02)).astype(np.float32)
            values, scales = oracle.quantize_per_output_channel_int8(w)
            samples.append((x, values.astype(np.int32), scales))
        _CPU_SAMPLES[key] = samples
    pool = ThreadPoolExecutor(max_workers=cores)

    def run(sample_rows: int) -> tuple[float, float]:
        ops = full_ops = 0.0
        for (x, w32, scales), (_, k, n) in zip(_CPU_SAMPLES[key], workload_shapes):
            xs = x[:sample_rows]  # type: ignore[index]
            q, s = oracle.quantize_rows_int8(xs)
            q32 = q.astype(np.int32)
            chunks = np.array_split(np.arange(w32.shape[0]), cores)  # type: ignore[union-attr]
            parts = list(pool.map(lambda idx: q32 @ w32[idx].T, [c for c in chunks if len(c)]))  # type: ignore[index]
            acc = np.concatenate(parts, axis=1)
            oracle.w8a8_dequantize(acc, s, scales)  # type: ignore[arg-type]
            ops += 2.0 * xs.shape[0] * w32.shape[0] * xs.shape[1]  # type: ignore[union-attr]
        return ops, full_ops

    if rows is None:
        probe_rows = min(8, tokens)
        t0 = time.perf_counter()
        probe_ops, _ = run(probe_rows)
        rate = probe_ops / max(time.perf_counter() - t0, 1e-6)
        rows = int(max(probe_rows, min(tokens, target_seconds * rate / (probe_ops / probe_rows))))
    t0 = time.perf_counter()
    ops, _ = run(rows)
    seconds = time.perf_counter() - t0
    pool.shutdown()
    return {
        "value": ops / seconds / 1e12,
        "unit": "TOPS",
        "cores": cores,
        "kind": "port",
        "seconds": round(seconds, 3),
        "sample": f"{rows} token rows x {CPU_COLUMNS} output columns of each {label} projection at full K "
        "(NumPy int32 matmul split over output columns across host threads)",
    }


def cpu_torch_int32_sample(*, workload_shapes: list[tuple[str, int, int]], tokens: int, target_seconds: float) -> dict[str, object]:
    """The reference benchmark's second CPU baseline, its torch int32 path
    (examples/benchmark_qpu_xla_w8a8.py:227-238: amax/127 floored at 1/127, round, clamp, int32
    matmul, fp32 dequant), on ``rows`` token rows x at most 1024 output columns per projection,
    torch using every host thread."""
    import torch

    cores = host_cores()
    torch.set_num_threads(cores)
    generator = torch.Generator().manual_seed(SEED)
    samples = []
    for _, k, n in workload_shapes:
        x = torch.randn((tokens, k), generator=generator, dtype=torch.float32)
        w = torch.randint(-127, 128, (min(CPU_COLUMNS, n), k), generator=generator, dtype=torch.int32)
        ws = torch.rand((min(CPU_COLUMNS, n),), generator=generator, dtype=torch.float32) * 0.001 + 1e-4
        samples.append((x, w, ws))

    def run(rows: int) -> float:
        ops = 0.0
        for x, w, ws in samples:
            xs = x[:rows]
            scales = torch.maximum(torch.amax(torch.abs(xs), dim=1) / 127, torch.tensor(1.0 / 127.0))
            q = torch.round(xs / scales[:, None]).clamp(-127, 127).to(torch.int32)
            acc = q @ w.T
            _ = acc.to(torch.float32) * scales[:, None] * ws[None, :]
            ops += 2.0 * rows * w.shape[0] * w.shape[1]
        return ops

    probe_rows = min(32, tokens)
    t0 = time.perf_counter()
    probe = run(probe_rows)
    rate = probe / max(time.perf_counter() - t0, 1e-6)
    rows = int(max(probe_rows, min(tokens, target_seconds * rate / (probe / probe_rows))))
    t0 = time.perf_counter()
    ops = run(rows)
    seconds = time.perf_counter() - t0
    return {
        "value": ops / seconds / 1e12,
        "unit": "TOPS",
        "cores": cores,
        "kind": "port",
        "seconds": round(seconds, 3),
        "sample": f"{rows} token rows x {CPU_COLUMNS} output columns per projection at full K (torch int32 matmul)",
    }


def cpu_square(target_seconds: float) -> dict[str, object]:
    """The reference's CPU path on the square cases, whole workload (NumPy int32 and torch int32)."""
    import numpy as np

    from oracle import qpu_oracle as oracle
    from qpu_xla import workloads

    result: dict[str, object] = {"kind": "port", "cores": host_cores()}
    for size in (64, 512):
        case = workloads.square_case(size)
        values, scales = oracle.quantize_per_output_channel_int8(case.weight)
        w32 = values.astype(np.int32)
        reps = 0
        t0 = time.perf_counter()
        while reps < 3 or time.perf_counter() - t0 < min(1.0, target_seconds / 2):
            q, s = oracle.quantize_rows_int8(case.source)
            y = oracle.w8a8_dequantize(q.astype(np.int32) @ w32.T, s, scales)
            if case.bias is not None:
                y = y + case.bias
            reps += 1
        seconds = (time.perf_counter() - t0) / reps
        result[str(size)] = {"numpy_int32_tops": 2.0 * size**3 / seconds / 1e12, "us_per_call": round(seconds * 1e6, 1)}
    result["sample"] = "the whole square workload per call (NumPy int32 path of quantization.py:1065-1082)"
    return result


def cpu_tinyllama_w8a8(target_seconds: float) -> dict[str, object]:
    from qpu_xla import workloads

    layer = [(s.name, s.in_features, s.out_features) for s in workloads.TINYLLAMA_LAYER]
    result: dict[str, object] = {"kind": "port", "cores": host_cores()}
    for tokens in workloads.TINYLLAMA_TOKENS:
        sample = cpu_reference_sample(target_seconds=target_seconds / 3, workload_shapes=layer, tokens=tokens, label="TinyLlama")
        result[str(tokens)] = {"numpy_int32_tops": sample["value"], "sample": sample["sample"]}
    result["torch_int32"] = cpu_torch_int32_sample(workload_shapes=layer, tokens=2048, target_seconds=target_seconds / 3)
    return result


def cpu_q4_0(target_seconds: float) -> dict[str, object]:
    """ggml_q4_0_q8_0_reference (NumPy port, ggml_q4_0.py:81-100) on the TinyLlama Q4_0 shapes."""
    import numpy as np

    from oracle import qpu_oracle as oracle
    from qpu_xla import workloads

    result: dict[str, object] = {"kind": "port", "cores": 1}
    for shape in workloads.TINYLLAMA_Q4_0_SHAPES:
        for rows in (1, 4):
            source, weight = workloads.q4_0_case(shape, rows)
            blocks = oracle.quantize_q4_0(weight)
            act = oracle.quantize_q8_0(source)
            reps = 0
            t0 = time.perf_counter()
            while reps < 2 or time.perf_counter() - t0 < target_seconds / 4:
                oracle.q4_0_q8_0_linear(act, blocks)
                reps += 1
            seconds = (time.perf_counter() - t0) / reps
            nbytes = 18.0 * shape.out_features * shape.in_features / 32 + 34.0 * rows * shape.in_features / 32 + 4.0 * rows * shape.out_features
            result[f"{shape.name}_m{rows}"] = {"gbs": round(nbytes / seconds / 1e9, 3), "ms_per_call": round(seconds * 1e3, 2)}
    result["sample"] = "the whole matvec per call (NumPy block loop of ggml_q4_0_q8_0_reference)"
    return result


def cpu_llama7b(target_seconds: float) -> dict[str, object]:
    from qpu_xla import workloads

    ffn = [(s.name, s.in_features, s.out_features) for s in workloads.LLAMA2_7B_FFN]
    return cpu_reference_sample(target_seconds=target_seconds, workload_shapes=ffn, tokens=TOKENS, label="7B FFN")


def cpu_q4_0_mx(target_seconds: float) -> dict[str, object]:
    """The reference program's MX arithmetic (NumPy port, per-block exact scaling) on a row sample of
    the 70B gate shape: 16 rows x 1024 output columns at full K, scaled to TOPS."""
    import numpy as np

    from oracle import qpu_oracle as oracle

    rng = np.random.default_rng(SEED)
    k, columns, rows = 8192, 1024, 16
    blocks = oracle.quantize_q4_0((rng.standard_normal((columns, k), dtype=np.float32) * np.float32(0.02)).astype(np.float32))
    act = oracle.quantize_q8_0(rng.standard_normal((rows, k), dtype=np.float32))
    reps, t0 = 0, time.perf_counter()
    while reps < 1 or time.perf_counter() - t0 < target_seconds / 4:
        oracle.q4_0_q8_0_linear_mx(act, blocks)
        reps += 1
    seconds = (time.perf_counter() - t0) / reps
    return {"value": 2.0 * rows * columns * k / seconds / 1e12, "unit": "TOPS", "cores": 1, "kind": "port",
            "sample": f"{rows} rows x {columns} output columns of the 70B gate shape at full K (NumPy port of the MX program)"}


OBJECT_CPU: dict[str, Callable[[float], dict[str, object]]] = {
    "square": cpu_square,
    "tinyllama_w8a8": cpu_tinyllama_w8a8,
    "tinyllama_q4_0": cpu_q4_0,
    "llama7b_ffn": cpu_llama7b,
    "q4_0_mx": cpu_q4_0_mx,
}


def run_reference(args: argparse.Namespace) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    per_step = max(0.05, min(20.0, 120.0 / max(1, args.steps + args.warmup)))
    first = cpu_reference_sample(target_seconds=per_step)
    rows = int(str(first["sample"]).split()[0])
    for _ in range(max(0, args.warmup - 1)):
        cpu_reference_sample(target_seconds=per_step, rows=rows)
    values = []
    t_total = 0.0
    for _ in range(args.steps):
        result = cpu_reference_sample(target_seconds=per_step, rows=rows)
        values.append(float(result["value"]))
        t_total += float(result["seconds"])
    value = statistics.median(values)
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": value,
        "unit": "TOPS",
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": t_total / max(1, args.steps) * 1e3,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "int8",
        "data": "synthetic: seeded N(0,1) activations, N(0,0.02) random-init weights (torch CUDA generator, seed 4)",
        "config": {
            "workload": WORKLOAD,
            "tokens": TOKENS,
            "projections": [f"{name} {k}->{n}" for name, k, n in shapes()],
            "parallelism": "host CPU (the reference's CPU path, NumPy port)",
        },
        "cpu_baseline": {"value": value, "unit": "TOPS", "cores": first["cores"], "kind": "port", "sample": first["sample"]},
        "e2e": {"value": value, "unit": "TOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=20)
    parser.add_argument("--warmup", type=int, default=5)
    parser.add_argument("--impl", choices=("ours", "reference"), default="ours")
    parser.add_argument("--no-e2e", action="store_true")
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--cpu-seconds", type=float, default=15.0)
    parser.add_argument("--only", default="", help="comma-separated projections (profiling captures only)")
    parser.add_argument("--objects", default=None,
                        help=f"comma-separated subset of {','.join(OBJECTS)} to time at N = 1 (default all; empty string: none)")
    parser.add_argument(
        "--exchange",
        choices=("auto", "fused", "copy", "nccl"),
        default="auto",
        help="N > 1: fused GEMM + all-gather over NVLink, copy-engine pushes after each GEMM, or NCCL all-gather after "
        "the GEMM; auto (default) takes the copy engines at 2 GPUs and the fused exchange from 3 on (measured on B200, "
        "70B FFN: 4507 against 4201 TOPS at 2 GPUs, 2423 against 3614 at 4, 1578 against 3266 at 8)",
    )
    args = parser.parse_args()
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    ONLY.update(name for name in args.only.split(",") if name)
    if args.objects is None:
        args.objects = list(OBJECTS)
    else:
        args.objects = [o for o in args.objects.split(",") if o]
        unknown = set(args.objects) - set(OBJECTS)
        if unknown:
            raise SystemExit(f"unknown --objects {sorted(unknown)}; choose from {OBJECTS}")
        if not args.objects:
            args.objects = ["__none__"]
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
