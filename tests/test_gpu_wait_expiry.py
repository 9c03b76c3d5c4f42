"""A kernel's bounded barrier wait runs out on the device, and the host sees it.

Every tcgen05 and bulk-copy mbarrier wait in this library is bounded by %globaltimer; on
expiry the kernel records an error word and returns. ``qpucuda_context_probe_wait_expiry``
runs that same bounded wait on an mbarrier nothing arrives at (bound 1 ms), so the wait
expires without any fault, trap or unbounded spin. The context must then behave as the
reference's does after a failed wait (qpu_llama_runtime.c:616-619, checked by host
injection in integrations/llama_cpp/tests/qpu_llama_native_safety_smoke.c:655-669): the
call returns TIMEOUT, the context is poisoned and rejects new work with IO_FAILED, and a
fresh context on the same device computes the 64^3 W8A8 case bit for bit.
"""

from __future__ import annotations

import time

import numpy as np
import pytest

from qpu_xla import _native, workloads

pytestmark = pytest.mark.gpu


def test_expired_kernel_wait_returns_timeout_and_poisons_the_context(golden: dict) -> None:
    import torch

    from gpu_helpers import Native

    native = Native()
    try:
        assert native.call("qpucuda_context_probe_wait_expiry", 0) == _native.Status.INVALID_ARGUMENT
        assert native.call("qpucuda_context_probe_wait_expiry", 2_000_000_000) == _native.Status.INVALID_ARGUMENT
        assert not native.context.poisoned
        start = time.perf_counter()
        status = native.call("qpucuda_context_probe_wait_expiry", 1_000_000)
        elapsed = time.perf_counter() - start
        assert status == _native.Status.TIMEOUT
        assert "exceeded its bound" in native.context.last_error()
        assert native.context.poisoned
        assert elapsed < 5.0  # the kernel's 1 ms bound ended it, not the host's 10 s timeout
        x = torch.randn((4, 64), dtype=torch.float32, device="cuda")
        q = torch.empty((4, 64), dtype=torch.int8, device="cuda")
        s = torch.empty(4, dtype=torch.float32, device="cuda")
        status = native.call("qpucuda_quantize_rows_int8", x.data_ptr(), 64, 4, 64, 64, q.data_ptr(), 64, s.data_ptr())
        assert status == _native.Status.IO_FAILED
    finally:
        native.close()
    torch.cuda.synchronize()  # the CUDA context itself stayed usable

    fresh = Native()
    try:
        ref = golden["w8a8_square_64"]
        case = workloads.square_case(64)
        plan = fresh.w8a8_prepare(ref["weight_values"], ref["weight_scales"], None, max_batch=64)
        try:
            source = torch.from_numpy(case.source).cuda()
            out = torch.full((64, 64), float("nan"), dtype=torch.float32, device="cuda")
            fresh.context.set_stream(torch.cuda.current_stream().cuda_stream)
            fresh.context.check(
                fresh.lib.qpucuda_w8a8_linear_execute_device(plan, source.data_ptr(), 64, 64, out.data_ptr(), 64),
                "execute_device",
            )
            fresh.sync()
            np.testing.assert_array_equal(out.cpu().numpy(), ref["output"])
        finally:
            fresh.lib.qpucuda_w8a8_linear_destroy(plan)
    finally:
        fresh.close()
