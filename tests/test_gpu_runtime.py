"""The drop-in Python surface on the GPU: Device/Tensor on CUDA memory, Queue/Event on
CUDA streams and events, the W8A8 and Q4_0 plans, kernel handles and the N-split."""

from __future__ import annotations

import os

import numpy as np
import pytest

from oracle import qpu_oracle as oracle
from qpu_xla import AccessMode, DependencyError, Device, EventStatus, Placement, workloads
from qpu_xla.candidates import CandidateRegistry
from qpu_xla.ggml import PreparedQ4_0Linear, quantize_q8_0
from qpu_xla.kernels import (
    CUDA_QUANTIZE_ROWS_INT8_KERNEL,
    CUDA_W8A8_DEQUANTIZE_KERNEL,
    CUDA_W8A8_GEMM_DEQUANTIZE_KERNEL,
    CUDA_W8A8_GEMM_KERNEL,
    CUDA_GGML_Q4_0_Q8_0_LINEAR_KERNEL,
)
from qpu_xla.quantization import CalibratedW8A8Linear, PreparedW8A8Linear, QuantizedMatrixInt8, quantize_per_output_channel_int8

pytestmark = pytest.mark.gpu


def test_cuda_tensors_write_read_and_slice(cuda_device: Device) -> None:
    tensor = cuda_device.tensor((8, 16), np.float32)
    values = np.arange(128, dtype=np.float32).reshape(8, 16)
    tensor.write(values)
    np.testing.assert_array_equal(tensor.numpy(), values)
    view = tensor.slice((slice(2, 5), slice(4, 12)))
    np.testing.assert_array_equal(view.numpy(), values[2:5, 4:12])
    assert view.torch().data_ptr() == view.address
    assert tensor.address % 256 == 0


def test_quantize_per_output_channel_on_gpu_matches_reference_weights(cuda_device: Device, golden: dict) -> None:
    case = workloads.square_case(512)
    quantized = quantize_per_output_channel_int8(case.weight, device=cuda_device)
    np.testing.assert_array_equal(quantized.values, golden["w8a8_square_512"]["weight_values"])
    np.testing.assert_array_equal(quantized.scales, golden["w8a8_square_512"]["weight_scales"])


def test_prepared_linear_on_a_queue_matches_the_reference(cuda_device: Device, golden: dict) -> None:
    ref = golden["w8a8_square_512"]
    case = workloads.square_case(512)
    weight = QuantizedMatrixInt8(ref["weight_values"], ref["weight_scales"])
    with cuda_device.queue() as queue, PreparedW8A8Linear(cuda_device, weight, max_batch=512, bias=ref["bias"]) as plan:
        source = cuda_device.tensor((512, 512), np.float32)
        destination = cuda_device.tensor((512, 512), np.float32)
        source.write(case.source)
        event = plan.execute(destination, source, queue=queue)
        event.wait()
        assert event.name == "cuda.w8a8_gemm_dequantize" and event.status is EventStatus.SUCCEEDED
        assert event.device_milliseconds is not None and event.device_milliseconds > 0
        np.testing.assert_array_equal(destination.numpy(), ref["output"])
        # the decode row goes through the GEMV kernel
        one = cuda_device.tensor((1, 512), np.float32)
        one_out = cuda_device.tensor((1, 512), np.float32)
        one.write(case.source[:1])
        event = plan.execute(one_out, one, queue=queue)
        event.wait()
        assert event.name == "cuda.w8a8_gemv"
        np.testing.assert_array_equal(one_out.numpy(), ref["output"][:1])
        # host-buffer C-ABI path of the same plan
        np.testing.assert_array_equal(plan.execute_host(case.source), ref["output"])


def test_execute_hybrid_computes_both_parts_on_the_gpu(cuda_device: Device, golden: dict) -> None:
    """quantization.py:350-514: the aligned prefix and the tail both run on the GPU here, so the
    output is the reference's whole result (its two parts share one exact arithmetic)."""
    ref = golden["w8a8_square_512"]
    case = workloads.square_case(512)
    weight = QuantizedMatrixInt8(ref["weight_values"], ref["weight_scales"])
    with cuda_device.queue() as gpu_queue, cuda_device.queue() as cpu_queue, PreparedW8A8Linear(
        cuda_device, weight, max_batch=512, bias=ref["bias"]
    ) as plan:
        source = cuda_device.tensor((512, 512), np.float32)
        destination = cuda_device.tensor((512, 512), np.float32)
        source.write(case.source)
        with pytest.raises(DependencyError):
            plan.execute_hybrid(destination, source, qpu_queue=gpu_queue, cpu_queue=gpu_queue, qpu_outputs=256)
        with pytest.raises(ValueError):
            plan.execute_hybrid(destination, source, qpu_queue=gpu_queue, cpu_queue=cpu_queue, qpu_outputs=100)
        plan.execute_hybrid(destination, source, qpu_queue=gpu_queue, cpu_queue=cpu_queue, qpu_outputs=256).wait()
        np.testing.assert_array_equal(destination.numpy(), ref["output"])


def test_host_execute_of_a_large_batch_is_sliced_and_exact(cuda_device: Device) -> None:
    """Batches above 1024 rows go through the pipelined host path (copy in, GEMM, copy out in
    row slices on three streams); a ragged last slice and a reused plan stay bit-exact."""
    rng = np.random.default_rng(71)
    rows, k, n = 2500, 320, 384
    weight = rng.standard_normal((n, k)).astype(np.float32)
    bias = rng.standard_normal(n).astype(np.float32)
    values, scales = oracle.quantize_per_output_channel_int8(weight)
    with PreparedW8A8Linear(cuda_device, QuantizedMatrixInt8(values, scales), max_batch=rows, bias=bias) as plan:
        for batch in (rows, 1025, 2048):
            source = (rng.standard_normal((batch, k)) * rng.uniform(0.1, 8.0, (batch, 1))).astype(np.float32)
            expected = oracle.w8a8_linear(source, values, scales, bias)
            np.testing.assert_array_equal(plan.execute_host(source), expected)


def test_direct_host_execute_writes_a_page_locked_destination_in_place(cuda_device: Device) -> None:
    """qpucuda_w8a8_linear_execute_direct: the same results as the staged host call, written by
    DMA into a page-locked destination (sliced and single-slice batches, GEMM and GEMV rows);
    a pageable destination is refused before anything runs."""
    import torch

    rng = np.random.default_rng(72)
    rows, k, n = 2300, 256, 512
    weight = rng.standard_normal((n, k)).astype(np.float32)
    values, scales = oracle.quantize_per_output_channel_int8(weight)
    with PreparedW8A8Linear(cuda_device, QuantizedMatrixInt8(values, scales), max_batch=rows) as plan:
        for batch in (rows, 700, 3):
            source = torch.from_numpy(rng.standard_normal((batch, k)).astype(np.float32)).pin_memory()
            pinned = torch.full((batch, n), float("nan"), dtype=torch.float32).pin_memory()
            plan.execute_host(source.numpy(), pinned.numpy(), direct=True)
            np.testing.assert_array_equal(pinned.numpy(), oracle.w8a8_linear(source.numpy(), values, scales))
        pageable = np.full((3, n), np.nan, dtype=np.float32)
        with pytest.raises(ValueError, match="page-locked"):
            plan.execute_host(rng.standard_normal((3, k)).astype(np.float32), pageable, direct=True)
        assert np.isnan(pageable).all()


def test_submissions_on_three_plans_overlap_and_match(cuda_device: Device) -> None:
    """qpucuda_w8a8_linear_submit_direct on three plans of one context, queued back to back before any
    wait (sliced and single-slice batches, the GEMV rows, one plan with bias): every destination
    equals the oracle bit for bit after its wait; a second submission on a plan still in flight is
    refused; waiting twice returns the same result."""
    import torch

    from qpu_xla.quantization import PreparedW8A8Linear as Plan

    rng = np.random.default_rng(91)
    shapes = ((2300, 256, 512, False), (1500, 384, 1024, True), (5, 512, 256, False))
    plans, jobs = [], []
    try:
        for rows, k, n, with_bias in shapes:
            values, scales = oracle.quantize_per_output_channel_int8(rng.standard_normal((n, k)).astype(np.float32))
            bias = rng.standard_normal(n).astype(np.float32) if with_bias else None
            plan = Plan(cuda_device, QuantizedMatrixInt8(values, scales), max_batch=rows, bias=bias)
            plans.append(plan)
            source = torch.from_numpy(rng.standard_normal((rows, k)).astype(np.float32)).pin_memory()
            pinned = torch.full((rows, n), float("nan"), dtype=torch.float32).pin_memory()
            jobs.append((plan.submit_direct(source.numpy(), pinned.numpy()), source, pinned, values, scales, bias))
        with pytest.raises(RuntimeError):
            plans[0].submit_direct(jobs[0][1].numpy(), jobs[0][2].numpy())
        for submission, source, pinned, values, scales, bias in jobs:
            result = submission.wait()
            np.testing.assert_array_equal(result, oracle.w8a8_linear(source.numpy(), values, scales, bias))
            assert submission.wait() is result
    finally:
        for plan in plans:
            plan.close()


def test_two_contexts_driven_from_two_threads_at_once() -> None:
    """Two contexts on one device, each called from its own host thread at the same time (the C
    calls release the GIL): every kernel's one-time set-up is per device and thread-safe, and each
    context keeps its own stream and staging. Rows of 16384 columns take the bulk-staged row
    quantizer, batches above 1024 rows the sliced host pipeline, M > 128 the CTA-pair GEMM."""
    import threading

    rng = np.random.default_rng(83)
    rows, k, n = 1100, 16384, 384
    weight = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    bias = rng.standard_normal(n).astype(np.float32)
    values, scales = oracle.quantize_per_output_channel_int8(weight)
    sources = [(rng.standard_normal((rows, k)) * rng.uniform(0.1, 8.0, (rows, 1))).astype(np.float32) for _ in range(2)]
    devices = [Device.open(device_ordinal=0) for _ in range(2)]
    plans: list[PreparedW8A8Linear] = []
    try:
        plans = [PreparedW8A8Linear(d, QuantizedMatrixInt8(values, scales), max_batch=rows, bias=bias) for d in devices]
        results: list[np.ndarray | None] = [None, None]
        errors: list[BaseException] = []
        start = threading.Barrier(2)

        def run(index: int) -> None:
            try:
                start.wait(timeout=60)
                for _ in range(3):
                    results[index] = plans[index].execute_host(sources[index])
            except BaseException as error:  # noqa: BLE001 - reported below
                errors.append(error)

        threads = [threading.Thread(target=run, args=(index,)) for index in range(2)]
        for thread in threads:
            thread.start()
        for thread in threads:
            thread.join(timeout=300)
        assert not any(thread.is_alive() for thread in threads) and not errors, errors
        for index in range(2):
            result = results[index]
            assert result is not None
            for part in (slice(0, 64), slice(rows - 64, rows)):
                expected = oracle.w8a8_linear(sources[index][part], values, scales, bias)
                np.testing.assert_array_equal(result[part], expected)
            np.testing.assert_array_equal(result, plans[index].execute_host(sources[index]))
    finally:
        for plan in plans:
            plan.close()
        for device in devices:
            device.close()


def test_plan_binding_and_in_flight_rules(cuda_device: Device) -> None:
    from qpu_xla import DependencyError

    values = np.ones((32, 32), dtype=np.int8)
    scales = np.full(32, 0.5, dtype=np.float32)
    with cuda_device.queue() as first, cuda_device.queue() as second:
        plan = PreparedW8A8Linear(cuda_device, QuantizedMatrixInt8(values, scales), max_batch=16)
        source = cuda_device.tensor((16, 32), np.float32)
        source.write(np.ones((16, 32), dtype=np.float32))
        destination = cuda_device.tensor((16, 32), np.float32)
        plan.execute(destination, source, queue=first).wait()
        with pytest.raises(DependencyError):
            plan.execute(destination, source, queue=second)
        with pytest.raises(ValueError):
            plan.execute(cuda_device.tensor((16, 31), np.float32), source, queue=first)
        plan.close()
        with pytest.raises(RuntimeError):
            plan.execute(destination, source, queue=first)


def test_kernel_handles_compose_on_queues_with_cross_queue_events(cuda_device: Device) -> None:
    """quantize on one queue, GEMM s32 + standalone dequant on another, fused GEMM on a third."""
    rng = np.random.default_rng(8)
    m, k, n = 200, 256, 384
    x = rng.standard_normal((m, k), dtype=np.float32)
    weight_values, weight_scales = oracle.quantize_per_output_channel_int8(rng.standard_normal((n, k), dtype=np.float32))
    bias = rng.standard_normal(n).astype(np.float32)
    expected = oracle.w8a8_linear(x, weight_values, weight_scales, bias)
    with cuda_device.queue() as q1, cuda_device.queue() as q2:
        source = cuda_device.tensor((m, k), np.float32)
        source.write(x)
        quantized = cuda_device.tensor((m, k), np.int8)
        row_scales = cuda_device.tensor((m,), np.float32)
        weight = cuda_device.tensor((n, k), np.int8)
        weight.write(weight_values)
        col_scales = cuda_device.tensor((n,), np.float32)
        col_scales.write(weight_scales)
        bias_t = cuda_device.tensor((n,), np.float32)
        bias_t.write(bias)
        acc = cuda_device.tensor((m, n), np.int32)
        out = cuda_device.tensor((m, n), np.float32)
        fused = cuda_device.tensor((m, n), np.float32)
        e_quant = q1.submit(CUDA_QUANTIZE_ROWS_INT8_KERNEL, (source, quantized, row_scales), buffers=(quantized.access(AccessMode.WRITE),))
        e_gemm = q2.submit(CUDA_W8A8_GEMM_KERNEL, (quantized, weight, acc), wait_for=(e_quant,))
        e_deq = q2.submit(CUDA_W8A8_DEQUANTIZE_KERNEL, (acc, row_scales, col_scales, out, bias_t), wait_for=(e_gemm,))
        e_fused = q1.submit(CUDA_W8A8_GEMM_DEQUANTIZE_KERNEL, (quantized, weight, row_scales, col_scales, fused, bias_t), wait_for=(e_quant,))
        e_deq.wait()
        e_fused.wait()
        np.testing.assert_array_equal(acc.numpy(), oracle.int8_accumulate(oracle.quantize_rows_int8(x)[0], weight_values))
        np.testing.assert_array_equal(out.numpy(), expected)
        np.testing.assert_array_equal(fused.numpy(), expected)
        trace = q2.chrome_trace()["traceEvents"]
        assert {"cuda.w8a8_gemm", "cuda.w8a8_dequantize", "dependency"} <= {event["name"] for event in trace}
        assert q2.consume_completed_event_counts() == {"cuda": 2}


def test_calibrated_linear_auto_runs_on_cuda(cuda_device: Device, golden: dict) -> None:
    ref = golden["w8a8_square_64"]
    case = workloads.square_case(64)
    weight = QuantizedMatrixInt8(ref["weight_values"], ref["weight_scales"])
    with cuda_device.queue() as queue, CalibratedW8A8Linear(cuda_device, weight, max_batch=64, candidates=CandidateRegistry()) as plan:
        source = cuda_device.tensor((64, 64), np.float32)
        destination = cuda_device.tensor((64, 64), np.float32)
        source.write(case.source)
        plan.execute(destination, source, queue=queue, placement=Placement.CUDA).wait()
        np.testing.assert_array_equal(destination.numpy(), ref["output"])
        with pytest.raises(ValueError):
            plan.execute(destination, source, queue=queue, placement=Placement.QPU)


def test_q4_0_plan_and_kernel_handle(cuda_device: Device, golden: dict) -> None:
    import torch

    ref = golden["q4_0_reference"]
    source, weight = workloads.q4_0_case(workloads.TINYLLAMA_Q4_0_SHAPES[1], 4)
    weight_blocks = oracle.quantize_q4_0(weight)
    with cuda_device.queue() as queue, PreparedQ4_0Linear(cuda_device, weight_blocks, rows=4) as plan:
        activation = cuda_device.tensor((4, 176, 34), np.uint8)
        activation.write(ref["ffn_down_m4_activation"])
        destination = cuda_device.tensor((4, 2048), np.float32)
        plan.execute(destination, activation, queue=queue).wait()
        expected = ref["ffn_down_m4_expected"]
        scale = float(np.abs(expected).max())
        assert float(np.abs(destination.numpy() - expected).max()) <= 1e-4 * scale
        # weight/output column split: weight columns [512, 1024) -> destination columns [0, 512)
        split = cuda_device.tensor((4, 512), np.float32)
        plan.execute(split, activation, queue=queue, column_start=512, column_count=512, output_column_start=0).wait()
        np.testing.assert_array_equal(split.numpy(), destination.numpy()[:, 512:1024])
        # fused fp32 path from the queue and the torch path
        fp32 = cuda_device.tensor((4, 5632), np.float32)
        fp32.write(source)
        fused = cuda_device.tensor((4, 2048), np.float32)
        plan.execute_f32(fused, fp32, queue=queue).wait()
        np.testing.assert_array_equal(fused.numpy(), destination.numpy())
        torch_out = plan.forward(quantize_q8_0(cuda_device, fp32.torch()))
        torch.cuda.synchronize()
        np.testing.assert_array_equal(torch_out.cpu().numpy(), destination.numpy())
        # the single-kernel handle over native blocks
        weight_t = cuda_device.tensor(weight_blocks.shape, np.uint8)
        weight_t.write(weight_blocks)
        native_out = cuda_device.tensor((4, 2048), np.float32)
        queue.submit(CUDA_GGML_Q4_0_Q8_0_LINEAR_KERNEL, (activation, weight_t, native_out, 0, 0, 2048)).wait()
        np.testing.assert_array_equal(native_out.numpy(), destination.numpy())


def test_sharded_linear_on_one_rank_equals_the_unsharded_plan(cuda_device: Device) -> None:
    """The N-split code path with a one-rank NCCL group (the multi-rank run is bench.py --gpus N)."""
    import torch
    import torch.distributed as dist

    from qpu_xla.sharded import ShardedQ4_0Linear, ShardedW8A8Linear

    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", "29517")
    owned = not dist.is_initialized()
    if owned:
        dist.init_process_group("nccl", rank=0, world_size=1, device_id=torch.device("cuda", 0))
    try:
        case = workloads.linear_inputs(96, 512, 1000, seed=31, weight_std=0.02, bias=True)
        values, scales = oracle.quantize_per_output_channel_int8(case.weight)
        weight = QuantizedMatrixInt8(values, scales)
        sharded = ShardedW8A8Linear(cuda_device, weight, max_batch=96, bias=case.bias)
        out = sharded.forward(torch.from_numpy(case.source).cuda())
        torch.cuda.synchronize()
        np.testing.assert_array_equal(out.cpu().numpy(), oracle.w8a8_linear(case.source, values, scales, case.bias))
        sharded.close()
        source, w = workloads.q4_0_case(workloads.TINYLLAMA_Q4_0_SHAPES[0], 1)
        blocks = oracle.quantize_q4_0(w)
        q4 = ShardedQ4_0Linear(cuda_device, blocks, rows=1)
        y = q4.forward(torch.from_numpy(source).cuda(), fp32_source=True)
        torch.cuda.synchronize()
        expected = oracle.q4_0_q8_0_linear(oracle.quantize_q8_0(source), blocks)
        assert float(np.abs(y.cpu().numpy() - expected).max()) <= 1e-4 * float(np.abs(expected).max())
        q4.close()
    finally:
        if owned:
            dist.destroy_process_group()


@pytest.mark.parametrize("with_bias", (False, True), ids=("no-bias", "bias"))
def test_merged_linear_sections_equal_their_own_linears(cuda_device: Device, with_bias: bool) -> None:
    """q/k/v-shaped weights (wide, narrow, narrow) merged into one plan: at GEMV, split-K,
    single-tile and CTA-pair batch sizes each section of the merged output equals the oracle of
    its own linear bit for bit, and the merged output equals three separate plans."""
    import torch

    from qpu_xla.quantization import MergedW8A8Linear

    rng = np.random.default_rng(57)
    k, sections = 1040, (512, 64, 64)
    weights, biases = [], []
    for n in sections:
        values, scales = oracle.quantize_per_output_channel_int8((rng.standard_normal((n, k)) * 0.02).astype(np.float32))
        weights.append(QuantizedMatrixInt8(values, scales))
        biases.append(rng.standard_normal(n).astype(np.float32))
    merged = MergedW8A8Linear(cuda_device, weights, max_batch=600, biases=biases if with_bias else None)
    separate = [PreparedW8A8Linear(cuda_device, w, max_batch=600, bias=b if with_bias else None) for w, b in zip(weights, biases)]
    try:
        assert merged.output_count == sum(sections)
        for rows in (1, 6, 64, 600):
            source_np = rng.standard_normal((rows, k)).astype(np.float32)
            source = torch.from_numpy(source_np).cuda()
            parts = merged.forward(source)
            alone = [plan.forward(source) for plan in separate]
            torch.cuda.synchronize()
            for part, single, w, b in zip(parts, alone, weights, biases):
                expected = oracle.w8a8_linear(source_np, w.values, w.scales, b if with_bias else None)
                np.testing.assert_array_equal(part.cpu().numpy(), expected)
                assert torch.equal(part, single)
    finally:
        merged.close()
        for plan in separate:
            plan.close()


@pytest.mark.parametrize("k", (16, 1036, 2048, 8192, 8196, 1038), ids=lambda k: f"k{k}")
def test_single_row_plan_call_quantizes_inside_the_gemv(cuda_device: Device, k: int) -> None:
    """One fp32 row through the plan: up to 8192 columns (a multiple of 4) the GEMV quantizes the
    row itself, otherwise the row quantizer runs first. Either way the output equals the oracle
    bit for bit, and the plan scratch holds the oracle's int8 row, zero padded over stale bytes,
    and its scale (execute_prepared reads them back). Rows of normal values, with a huge value,
    and all zeros (the 1/127 scale floor)."""
    import torch

    rng = np.random.default_rng(k)
    n = 700
    values, scales = oracle.quantize_per_output_channel_int8((rng.standard_normal((n, k)) * 0.02).astype(np.float32))
    bias = rng.standard_normal(n).astype(np.float32)
    with PreparedW8A8Linear(cuda_device, QuantizedMatrixInt8(values, scales), max_batch=4, bias=bias) as plan:
        quantized, row_scales = plan.scratch()
        for case in range(3):
            row = rng.standard_normal((1, k)).astype(np.float32)
            if case == 1:
                row[0, k // 3] = np.float32(3.0e38)
                row[0, 0] = np.float32(0.0)
            if case == 2:
                row[:] = np.float32(0.0)
            quantized.fill_(0x5A)
            row_scales.fill_(-1.0)
            out = plan.forward(torch.from_numpy(row).cuda())
            torch.cuda.synchronize()
            np.testing.assert_array_equal(out.cpu().numpy(), oracle.w8a8_linear(row, values, scales, bias))
            q_expected, s_expected = oracle.quantize_rows_int8(row)
            q_row = quantized[0].cpu().numpy()
            np.testing.assert_array_equal(q_row[:k], q_expected[0])
            assert not q_row[k:].any()
            assert row_scales[0].item() == float(s_expected[0])
