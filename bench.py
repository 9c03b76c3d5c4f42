#!/usr/bin/env python3
"""Headline benchmark: W8A8 GEMM TOPS (and Q4_0 GEMV GB/s) at 1/2/4/8 B200s.

Workload (the configuration the metric is quoted on
"at 1/2/4/8 GPUs"): the Llama-2-70B FFN at prefill, M = 4096 tokens, W8A8
dynamic linear for gate (8192->28672), up (8192->28672) and down (28672->8192);
plus, as objects of the same line, the Q4_0 x Q8_0 decode matvec (M = 1) and the
W8A8 decode (the same plans at M = 1 and 8, int8 GEMV) on the same three shapes. Weights are
random-init ~N(0, 0.02), activations ~N(0, 1), drawn on the GPU from a fixed
seed (identical on every rank). Each projection's output channels (N) are split
across the ranks; N = 1 runs the identical inputs unsplit.

One step = for each projection: quantize the fp32 rows (int8 kernel), tcgen05
int8 GEMM with the fused dequant epilogue on the rank's column shard, and (N > 1)
the exchange that leaves the full [M, N] fp32 output on every rank: the GEMM
epilogue stores each tile into every rank's output buffer (mapped with CUDA IPC)
over NVLink as it finishes, then a one-element NCCL all-reduce orders all ranks'
stores (the fused GEMM + all-gather). If the peer mapping is refused, the step
falls back to an NCCL all-gather after the GEMM and the line says so. L2 is
flushed between timed steps, outside the
per-step CUDA-event brackets: a 256 MiB write, then a 256 MiB read of a second
buffer, so the timed kernels start on a cache of clean lines (as after the
previous layer's weight stream) rather than paying the write-back of the flush's
own dirty lines; inputs also exceed L2.

``python bench.py [--gpus N --steps K --warmup W]``; for N > 1 run under
``torch.distributed.run`` (one rank per GPU). ``--impl reference`` times the
reference's own CPU implementation (the oracle port of
src/qpu_xla/models/tinyllama/quantization.py:1065-1082) on a bounded sample.
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

ROOT = Path(__file__).resolve().parent
sys.path[:0] = [str(ROOT / "qpu-xla-triton_b200"), str(ROOT)]

METRIC = "W8A8 GEMM TOPS & Q4_0 GEMV GB/s, % of B200 roofline, at 1/2/4/8 GPUs"
WORKLOAD = "llama2-70b-ffn prefill W8A8 M=4096 (gate 8192->28672, up 8192->28672, down 28672->8192) + Q4_0 decode M=1 on the same shapes"
TOKENS = 4096
SEED = 4
L2_FLUSH_BYTES = 256 << 20
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


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


def profile_traffic(name: str) -> float | None:
    """Per-launch DRAM bytes recorded by the committed ncu summary ``profiles/<name>.md`` (a
    ``traffic_bytes_per_launch: <n>`` line), or None before a capture exists."""
    path = ROOT / "profiles" / f"{name}.md"
    if not path.exists():
        return None
    for line in path.read_text().splitlines():
        if line.strip().startswith("traffic_bytes_per_launch:"):
            try:
                return float(line.split(":", 1)[1].strip().split()[0])
            except ValueError:
                return None
    return None


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


def run_ours(args: argparse.Namespace) -> None:
    import torch
    import torch.distributed as dist

    from qpu_xla import Device
    from qpu_xla.ggml import PreparedQ4_0Linear
    from qpu_xla.quantization import PreparedW8A8Linear, QuantizedMatrixInt8
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

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=cuda)
    device = Device.open(device_ordinal=local_rank)
    native = device.backend.native  # type: ignore[attr-defined]
    stream = torch.cuda.current_stream(cuda)

    def launch(call):  # type: ignore[no-untyped-def]
        device.backend.launch(stream, lambda n: n.check(call(n.library, n.handle), "bench"))  # type: ignore[attr-defined]

    # ---- inputs and plans (identical on every rank: seeded GPU generator) ----
    generator = torch.Generator(device=cuda)
    generator.manual_seed(SEED)
    projections = []
    sources: dict[int, torch.Tensor] = {}
    for index, (name, k, n) in enumerate(shapes()):
        if k not in sources:
            sources[k] = torch.randn((TOKENS, k), generator=generator, device=cuda, dtype=torch.float32)
        weight = torch.randn((n, k), generator=generator, device=cuda, dtype=torch.float32) * 0.02
        values = torch.empty((n, k), dtype=torch.int8, device=cuda)
        scales = torch.empty((n,), dtype=torch.float32, device=cuda)
        launch(lambda lib, h: lib.qpucuda_quantize_rows_int8(h, weight.data_ptr(), k, n, k, k, values.data_ptr(), k, scales.data_ptr()))
        q4_blocks = torch.empty((n, k // 32, 18), dtype=torch.uint8, device=cuda)
        launch(lambda lib, h: lib.qpucuda_quantize_q4_0(h, weight.data_ptr(), k, n, k, q4_blocks.data_ptr()))
        torch.cuda.synchronize()
        gather = ColumnGather(n, world, rank)
        quantized = QuantizedMatrixInt8(values.cpu().numpy(), scales.cpu().numpy())
        plan = PreparedW8A8Linear(device, quantized, max_batch=TOKENS, resident_outputs=(gather.start, gather.count))
        q4 = PreparedQ4_0Linear(device, q4_blocks.cpu().numpy(), rows=1, resident_column_start=gather.start, resident_column_count=gather.count)
        local = torch.zeros((TOKENS, gather.width), dtype=torch.float32, device=cuda)
        full = torch.empty((TOKENS, n), dtype=torch.float32, device=cuda) if world > 1 else local
        projections.append({"name": name, "k": k, "n": n, "gather": gather, "plan": plan, "q4": q4, "local": local, "full": full, "source": sources[k]})
        del weight, values, scales, q4_blocks
    exchange = "none"
    if world > 1 and args.exchange == "nccl":
        exchange = "NCCL all-gather after the GEMM (selected with --exchange nccl)"
        barrier_flag = None
    elif world > 1:
        from qpu_xla.sharded import PeerOutput

        exchange = "fused GEMM epilogue stores into every rank's output (CUDA IPC over NVLink) + NCCL all-reduce barrier"
        try:
            for p in projections:
                p["peer"] = PeerOutput(device, TOKENS, p["n"])
        except Exception as error:  # noqa: BLE001 - the mapping refusal is reported, not hidden
            for p in projections:
                if "peer" in p:
                    p.pop("peer").close()
            exchange = f"NCCL all-gather after the GEMM (peer mapping refused: {str(error)[:120]})"
        barrier_flag = torch.zeros(1, dtype=torch.float32, device=cuda)
    torch.cuda.empty_cache()
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=cuda)
    flush_clean = torch.ones(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=cuda)

    def prime() -> None:
        """Flush L2 (write one buffer larger than L2, then read another so the lines left are
        clean), then hold the stream ~60 us so the host has queued the bracketed launches
        before the start event executes (no host launch latency inside a timed bracket)."""
        flush.zero_()
        flush_clean.sum()
        torch.cuda._sleep(120_000)

    def step() -> None:
        for p in projections:
            g = p["gather"]
            if "peer" in p:
                destination, peers = p["peer"].slice_pointers(g.start)
                p["plan"].forward_fanout(p["source"], destination, peers, p["n"])
                dist.all_reduce(barrier_flag)
                continue
            p["plan"].forward(p["source"], out=p["local"][:, : g.count])
            if world > 1:
                g.gather(p["local"], out=p["full"])

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
        prime()
        step()
    barrier()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    wall0 = time.perf_counter()
    for i in range(args.steps):
        prime()
        starts[i].record(stream)
        step()
        ends[i].record(stream)
    barrier()
    wall = time.perf_counter() - wall0
    step_ms = max_over_ranks(sum(s.elapsed_time(e) for s, e in zip(starts, ends)) / args.steps)
    total_ops = sum(2.0 * TOKENS * p["n"] * p["k"] for p in projections)  # whole job, all ranks
    value_tops = total_ops / (step_ms * 1e-3) / 1e12

    # ---- N > 1: the same step without the exchange (quantize + GEMM on the rank's shard) ----
    multi_gpu = None
    if world > 1:

        def local_step() -> None:
            for p in projections:
                p["plan"].forward(p["source"], out=p["local"][:, : p["gather"].count])

        for _ in range(args.warmup):
            prime()
            local_step()
        barrier()
        local_starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        local_ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        for i in range(args.steps):
            prime()
            local_starts[i].record(stream)
            local_step()
            local_ends[i].record(stream)
        barrier()
        local_ms = max_over_ranks(sum(s.elapsed_time(e) for s, e in zip(local_starts, local_ends)) / args.steps)
        # fp32 output columns every rank receives from the others per step
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

    # ---- dominant kernel: the tcgen05 GEMM alone (activations already quantized) ----
    gemm_ms = []
    for p in projections:
        plan = p["plan"]
        quantized, row_scales = plan.scratch()
        plan.forward(p["source"], out=p["local"][:, : p["gather"].count])  # fills the scratch for this projection
        handle = plan._handle
        out = p["local"]

        def gemm(handle=handle, quantized=quantized, row_scales=row_scales, out=out, count=p["gather"].count):  # type: ignore[no-untyped-def]
            launch(lambda lib, h: lib.qpucuda_w8a8_linear_execute_prepared_device(
                handle, quantized.data_ptr(), quantized.stride(0), row_scales.data_ptr(), TOKENS, out.data_ptr(), out.stride(0)))

        for _ in range(3):
            gemm()
        reps = 10
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
        for s, e in evs:
            prime()
            s.record(stream)
            gemm()
            e.record(stream)
        torch.cuda.synchronize()
        gemm_ms.append(statistics.mean(s.elapsed_time(e) for s, e in evs))
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
        for _ in range(3):
            torch._int_mm(a8, w8.t())
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(10)]
        for s_ev, e_ev in evs:
            prime()
            s_ev.record(stream)
            torch._int_mm(a8, w8.t())
            e_ev.record(stream)
        torch.cuda.synchronize()
        library_ms.append(statistics.mean(s_ev.elapsed_time(e_ev) for s_ev, e_ev in evs))
        del a8, w8
    torch.cuda.empty_cache()
    library_tops = rank_gemm_ops / (sum(library_ms) * 1e-3) / 1e12
    library_tops = max_over_ranks(library_tops)

    # ---- Q4_0 x Q8_0 decode matvec (M = 1), Q8_0 activations already on the device ----
    # One decode step of the FFN = gate, up and down back to back on the stream. The three
    # weight matrices (3 x 132 MB at full width) exceed L2, so each launch streams its weight
    # from DRAM; L2 is flushed before every bracketed step as for the prefill steps.
    q4_inputs = []
    q4_bytes_rank = 0.0
    for p in projections:
        g = p["gather"]
        act = torch.empty((1, p["k"] // 32, 34), dtype=torch.uint8, device=cuda)
        src = p["source"][:1]
        launch(lambda lib, h: lib.qpucuda_quantize_q8_0(h, src.data_ptr(), src.stride(0), 1, p["k"], act.data_ptr()))
        out = torch.empty((1, g.width), dtype=torch.float32, device=cuda)
        q4_inputs.append((p["q4"], act, out[:, : g.count]))
        q4_bytes_rank += 18.0 * g.count * p["k"] / 32 + 34.0 * p["k"] / 32 + 4.0 * g.count

    def decode_ffn() -> None:
        for q4, act, out in q4_inputs:
            q4.forward(act, out=out)

    for _ in range(3):
        decode_ffn()
    reps = 20
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
    for s, e in evs:
        prime()
        s.record(stream)
        decode_ffn()
        e.record(stream)
    torch.cuda.synchronize()
    q4_step_ms = statistics.mean(s.elapsed_time(e) for s, e in evs)
    # each projection alone in its own bracket (includes one bracket's fixed event overhead)
    q4_ms = []
    for q4, act, out in q4_inputs:
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
        for s, e in evs:
            prime()
            s.record(stream)
            q4.forward(act, out=out)
            e.record(stream)
        torch.cuda.synchronize()
        q4_ms.append(statistics.mean(s.elapsed_time(e) for s, e in evs))
    q4_seconds = max_over_ranks(q4_step_ms * 1e-3)
    q4_total_bytes = sum_over_ranks(q4_bytes_rank)
    q4_gbs = q4_total_bytes / q4_seconds / 1e9
    q4_rank_gbs = q4_bytes_rank / (q4_step_ms * 1e-3) / 1e9

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
        for _ in range(3):
            decode_w8a8()
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
        for s, e in evs:
            prime()
            s.record(stream)
            decode_w8a8()
            e.record(stream)
        torch.cuda.synchronize()
        gemv_step_ms = max_over_ranks(statistics.mean(s.elapsed_time(e) for s, e in evs))
        w8a8_gemv[str(gemv_rows)] = {
            "value": round(sum_over_ranks(gemv_bytes_rank) / (gemv_step_ms * 1e-3) / 1e9, 1),
            "rank_gbs": round(gemv_bytes_rank / (gemv_step_ms * 1e-3) / 1e9, 1),
            "us_per_decode_ffn": round(gemv_step_ms * 1e3, 2),
        }

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
            for p, out in zip(projections, host_out):
                p["plan"].execute_host(host_sources[p["k"]].numpy(), out.numpy())

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
            "path": "qpucuda_w8a8_linear_execute (host pinned buffers) per rank on its column shard",
        }

    cpu_baseline = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu_baseline = cpu_reference_sample(target_seconds=args.cpu_seconds)

    peaks, peak_kind = measured_peaks()
    bf16_doubled = 2.0 * peaks["bf16_tflops"]
    int8_peak = max(bf16_doubled, library_tops)
    traffic = profile_traffic("w8a8_gemm_sm100_70b_ffn")
    q4_traffic = profile_traffic("q4_0_gemv_70b_decode")
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
            "l2": "flushed between timed steps (256 MiB write, then 256 MiB read of a second buffer; outside the CUDA-event brackets); inputs exceed L2",
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
            "peak_source": (
                f"the larger of cuBLASLt int8 (torch._int_mm) measured live on the same shapes ({library_tops:.1f} TOPS) "
                f"and 2 x {peak_kind} cuBLAS bf16 burst ({bf16_doubled:.1f} TOPS)"
            ),
            "library_int8_tops": round(library_tops, 1),
            "library_int8_ms_per_projection": [round(x, 4) for x in library_ms],
            "peak_2x_bf16": round(bf16_doubled, 1),
            "traffic": traffic,
            "algorithmic_ops_per_rank_step": rank_gemm_ops,
            "gemm_ms_per_projection": [round(x, 4) for x in gemm_ms],
        },
        "q4_0_gemv": {
            "metric": "Q4_0 x Q8_0 M=1 GEMV GB/s (whole job), one decode FFN step (gate, up, down) per bracket",
            "value": round(q4_gbs, 1),
            "unit": "GB/s",
            "roofline": {
                "kernel": "q4_0_direct_kernel (dp4a, prepared nibble layout, two columns per warp)",
                "bound": "hbm",
                "achieved": round(q4_rank_gbs, 1),
                "peak": peaks["hbm_gbs"],
                "unit": "GB/s",
                "frac": round(q4_rank_gbs / peaks["hbm_gbs"], 4),
                "peak_source": f"{peak_kind} STREAM-style copy",
                "traffic": q4_traffic,
            },
            "us_per_decode_ffn": round(q4_step_ms * 1e3, 2),
            "us_per_projection_alone": [round(x * 1e3, 2) for x in q4_ms],
        },
        "w8a8_gemv": {
            "metric": "W8A8 decode GB/s (whole job), one FFN step (gate, up, down: row quantizer + int8 GEMV) per bracket, at M = 1 and M = 8",
            "value": w8a8_gemv["1"]["value"],
            "unit": "GB/s",
            "rows": w8a8_gemv,
            "roofline": {
                "kernel": "w8a8_gemv_kernel (dp4a, persistent balanced grid, split-K across a CTA's warps, next column's first loads issued before the reduction at M <= 2)",
                "bound": "hbm",
                "achieved": w8a8_gemv["1"]["rank_gbs"],
                "peak": peaks["hbm_gbs"],
                "unit": "GB/s",
                "frac": round(w8a8_gemv["1"]["rank_gbs"] / peaks["hbm_gbs"], 4),
                "peak_source": f"{peak_kind} STREAM-style copy",
                "traffic": None,
            },
        },
        "clocks": clocks,
    }
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


# ---------------------------------------------------------------------------- reference (CPU)


_CPU_SAMPLES: list[tuple[object, object, object]] = []
CPU_COLUMNS = 1024


def cpu_reference_sample(*, target_seconds: float, rows: int | None = None) -> dict[str, object]:
    """The reference's CPU path (oracle port of quantization.py:1065-1082: NumPy per-row
    quantization, int32 matmul, fp32 dequant) on a bounded sample of the workload: ``rows``
    token rows (sized to ``target_seconds``, at most the full 4096) x 1024 output columns of
    each projection at its full K, split over all host threads."""
    import numpy as np

    from oracle import qpu_oracle as oracle

    cores = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    columns = CPU_COLUMNS
    if not _CPU_SAMPLES:
        rng = np.random.default_rng(SEED)
        for _, k, _n in shapes():
            x = rng.standard_normal((TOKENS, k), dtype=np.float32)
            w = (rng.standard_normal((columns, k), dtype=np.float32) * np.float32(0.02)).astype(np.float32)
            values, scales = oracle.quantize_per_output_channel_int8(w)
            _CPU_SAMPLES.append((x, values.astype(np.int32), scales))
    pool = ThreadPoolExecutor(max_workers=cores)

    def run(sample_rows: int) -> float:
        ops = 0.0
        for x, w32, scales in _CPU_SAMPLES:
            xs = x[:sample_rows]  # type: ignore[index]
            q, s = oracle.quantize_rows_int8(xs)
            q32 = q.astype(np.int32)
            chunks = np.array_split(np.arange(w32.shape[0]), cores)  # type: ignore[union-attr]
            parts = list(pool.map(lambda idx: q32 @ w32[idx].T, [c for c in chunks if len(c)]))  # type: ignore[index]
            acc = np.concatenate(parts, axis=1)
            oracle.w8a8_dequantize(acc, s, scales)  # type: ignore[arg-type]
            ops += 2.0 * xs.shape[0] * w32.shape[0] * xs.shape[1]  # type: ignore[union-attr]
        return ops

    if rows is None:
        t0 = time.perf_counter()
        probe_ops = run(8)
        rate = probe_ops / max(time.perf_counter() - t0, 1e-6)
        rows = int(max(8, min(TOKENS, target_seconds * rate / (probe_ops / 8))))
    t0 = time.perf_counter()
    ops = run(rows)
    seconds = time.perf_counter() - t0
    pool.shutdown()
    return {
        "value": ops / seconds / 1e12,
        "unit": "TOPS",
        "cores": cores,
        "kind": "port",
        "seconds": round(seconds, 3),
        "sample": f"{rows} token rows x {columns} output columns of each 70B FFN projection at full K "
        "(NumPy int32 matmul split over output columns across host threads)",
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
        "data": "synthetic: seeded N(0,1) activations, N(0,0.02) weights",
        "config": {"workload": WORKLOAD, "tokens": TOKENS, "parallelism": "host CPU (reference CPU path)"},
        "cpu_baseline": {"value": value, "unit": "TOPS", "cores": first["cores"], "kind": "port", "sample": first["sample"]},
        "e2e": {"value": value, "unit": "TOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=300)
    parser.add_argument("--warmup", type=int, default=5)
    parser.add_argument("--impl", choices=("ours", "reference"), default="ours")
    parser.add_argument("--no-e2e", action="store_true")
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--cpu-seconds", type=float, default=15.0)
    parser.add_argument("--only", default="", help="comma-separated projections (profiling captures only)")
    parser.add_argument(
        "--exchange",
        choices=("fused", "nccl"),
        default="fused",
        help="N > 1: fused GEMM + all-gather over NVLink (default) or NCCL all-gather after the GEMM",
    )
    args = parser.parse_args()
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    ONLY.update(name for name in args.only.split(",") if name)
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
