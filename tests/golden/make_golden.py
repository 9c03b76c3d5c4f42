"""Generate the golden fixtures under tests/golden/ by running the reference's own CPU code.

Run in a container where the reference checkout is available (read-only):

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py --reference <checkout>

It imports ``qpu_xla`` from ``<checkout>/src`` (with a stub for the
setuptools-scm version module that the checkout lacks, and a stub ``ioctl_opt``
so the example module that holds the Q8_0 quantizer imports without the V3D
driver) and records, on the seeded inputs of ``qpu_xla.workloads``:

* ``w8a8_square_64.npz`` / ``w8a8_square_512.npz`` -- the reference's
  ``quantize_per_output_channel_int8`` weights, the per-row activation
  quantization (the same reference function applied to the activations), the
  exact int32 accumulators, and the fp32 output of
  ``CalibratedW8A8Linear(...).execute`` on ``Device.fake()``
  (quantization.py:1065-1082) -- with the bias added by the reference's
  ``_StagedW8A8Linear._cpu`` (smolvla/accelerated.py:248-262) for 512^3;
* ``w8a8_tinyllama.npz`` -- SHA-256 digests of the reference's fp32 outputs for
  the seven TinyLlama projections at M = 1 and M = 128;
* ``q4_0_reference.npz`` -- ``ggml_q4_0_q8_0_reference`` (ggml_q4_0.py:81-100)
  on the inputs of the reference's own hardware test (seed 4404, 5 blocks, 32
  outputs) and on TinyLlama FFN shapes at M = 1 and 4, with the Q8_0
  activations from the reference's ``quantize_q8_0_split``
  (examples/benchmark_llama_cpp_qpu_persistent_q4.py:42-54);
* ``codec_extremes.npz`` -- the reference's pack/unpack on the extreme codes of
  tests/test_qpu_xla_ggml_q4_0.py:25-44.

The GPU box never runs this script; the tests read only the .npz files.
"""

from __future__ import annotations

import argparse
import hashlib
import sys
import types
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO / "qpu-xla-triton_b200"))
sys.path.insert(0, str(REPO))

from oracle import qpu_oracle  # noqa: E402  (used only to build Q4_0 weights; see quantize_q4_0)
from qpu_xla import workloads  # noqa: E402


def import_reference(checkout: Path) -> dict[str, object]:
    version = types.ModuleType("_videocore7._version")
    version.__version__ = "0"  # type: ignore[attr-defined]
    sys.modules["_videocore7._version"] = version
    ioctl_stub = types.ModuleType("ioctl_opt")
    for name in ("IO", "IOR", "IOW", "IOWR"):
        setattr(ioctl_stub, name, lambda *args, **kwargs: 0)
    sys.modules["ioctl_opt"] = ioctl_stub
    saved = list(sys.path)
    sys.path[:0] = [str(checkout / "src"), str(checkout / "examples"), str(checkout)]
    # The reference package is also called qpu_xla: drop ours for the import.
    for name in [n for n in sys.modules if n == "qpu_xla" or n.startswith("qpu_xla.")]:
        del sys.modules[name]
    sys.path = [p for p in sys.path if not p.endswith("qpu-xla-triton_b200")]
    import qpu_xla as reference_qpu_xla
    from qpu_xla.benchmark import CandidateRegistry
    from qpu_xla.kernels import ggml_q4_0
    from qpu_xla.models.smolvla.accelerated import _StagedW8A8Linear
    from qpu_xla.models.tinyllama.quantization import CalibratedW8A8Linear, quantize_per_output_channel_int8

    import benchmark_llama_cpp_qpu_persistent_q4 as persistent_example
    from qpu_xla.ops.conv2d import _im2col_nchw

    sys.path.insert(0, str(checkout / "tests"))
    import test_qpu_xla_conv2d_w8a8 as conv_tests

    assert Path(reference_qpu_xla.__file__).is_relative_to(checkout), "imported the wrong qpu_xla"
    sys.path = saved
    return {
        "Device": reference_qpu_xla.Device,
        "CandidateRegistry": CandidateRegistry,
        "CalibratedW8A8Linear": CalibratedW8A8Linear,
        "quantize_per_output_channel_int8": quantize_per_output_channel_int8,
        "staged_cpu": _StagedW8A8Linear._cpu,
        "ggml": ggml_q4_0,
        "quantize_q8_0_split": persistent_example.quantize_q8_0_split,
        "im2col_nchw": _im2col_nchw,
        "conv_dynamic_group_reference": conv_tests._dynamic_group_reference,
    }


def reference_linear(ref: dict[str, object], source: np.ndarray, weight: np.ndarray, bias: np.ndarray | None) -> dict[str, np.ndarray]:
    quantize = ref["quantize_per_output_channel_int8"]
    quantized = quantize(weight)  # type: ignore[operator]
    activations = quantize(source)  # same formula as the activation quantizer (quantization.py:1066-1071)
    accumulation = (activations.values.astype(np.int64) @ quantized.values.astype(np.int64).T).astype(np.int32)
    Device = ref["Device"]
    with Device.fake() as device, device.queue() as queue:  # type: ignore[attr-defined]
        src = device.tensor(source.shape, np.float32)
        dst = device.tensor((source.shape[0], weight.shape[0]), np.float32)
        src.numpy()[:] = source
        with ref["CalibratedW8A8Linear"](device, quantized, max_batch=source.shape[0], candidates=ref["CandidateRegistry"]()) as plan:  # type: ignore[operator]
            event = plan.execute(dst, src, queue=queue)
            event.wait()
            assert event.name == "w8a8_linear.cpu_reference"
            output = np.array(dst.numpy(), copy=True)
    if bias is not None:
        weight_record = types.SimpleNamespace(values=quantized.values, scales=quantized.scales)
        output = ref["staged_cpu"](source, weight_record, bias)  # type: ignore[operator]
    return {
        "weight_values": quantized.values,
        "weight_scales": quantized.scales,
        "activation_values": activations.values,
        "activation_scales": activations.scales,
        "accumulation": accumulation,
        "output": np.ascontiguousarray(output, dtype=np.float32),
    }


def sha256(array: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(array).tobytes()).hexdigest()


def main() -> int:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--reference", type=Path, required=True)
    args = parser.parse_args()
    ref = import_reference(args.reference.resolve())

    for size in (64, 512):
        case = workloads.square_case(size)
        result = reference_linear(ref, case.source, case.weight, case.bias)
        extra = {"bias": case.bias} if case.bias is not None else {}
        np.savez_compressed(HERE / f"w8a8_square_{size}.npz", source_sha256=sha256(case.source), **result, **extra)
        print(f"w8a8_square_{size}: output {result['output'].shape}")

    digests: dict[str, str] = {}
    for shape in workloads.TINYLLAMA_LAYER:
        for tokens in (1, 128):
            case = workloads.tinyllama_case(shape, tokens)
            result = reference_linear(ref, case.source, case.weight, None)
            key = f"{shape.name}_m{tokens}"
            digests[f"{key}_output"] = sha256(result["output"])
            digests[f"{key}_weight_values"] = sha256(result["weight_values"])
            digests[f"{key}_source"] = sha256(case.source)
            print(f"tinyllama {key}")
    np.savez_compressed(HERE / "w8a8_tinyllama.npz", **{k: np.array(v) for k, v in digests.items()})

    ggml = ref["ggml"]
    q4: dict[str, np.ndarray] = {}
    # The reference's own hardware test inputs (tests/test_qpu_xla_ggml_q4_0.py:47-80).
    rng = np.random.default_rng(4400 + 4)
    rows, blocks, outputs = 4, 5, 32
    activation_scales = rng.uniform(0.0001, 0.2, size=(rows, blocks)).astype(np.float32)
    activation_values = rng.integers(-128, 128, size=(rows, blocks, 32), dtype=np.int16)
    weight_scales = rng.uniform(-0.2, 0.2, size=(outputs, blocks)).astype(np.float16)
    weight_codes = rng.integers(0, 16, size=(outputs, blocks, 32), dtype=np.uint8)
    activation_blocks = ggml.pack_ggml_q8_0_blocks(activation_scales, activation_values)  # type: ignore[attr-defined]
    weight_blocks = ggml.pack_ggml_q4_0_blocks(weight_scales, weight_codes)  # type: ignore[attr-defined]
    q4["hw_activation"] = activation_blocks
    q4["hw_weight"] = weight_blocks
    q4["hw_expected"] = ggml.ggml_q4_0_q8_0_reference(activation_blocks, weight_blocks)  # type: ignore[attr-defined]
    for shape in workloads.TINYLLAMA_Q4_0_SHAPES:
        for rows in (1, 4):
            source, weight = workloads.q4_0_case(shape, rows)
            scale_words, values = ref["quantize_q8_0_split"](source)  # type: ignore[operator]
            act = np.empty((rows, shape.in_features // 32, 34), dtype=np.uint8)
            act[..., :2] = scale_words.reshape(rows, -1).view(np.uint8).reshape(rows, -1, 2)
            act[..., 2:] = values.reshape(rows, -1, 32)
            w_blocks = qpu_oracle.quantize_q4_0(weight)
            key = f"{shape.name}_m{rows}"
            q4[f"{key}_activation"] = act
            q4[f"{key}_weight_sha256"] = np.array(sha256(w_blocks))
            q4[f"{key}_expected"] = ggml.ggml_q4_0_q8_0_reference(act, w_blocks)  # type: ignore[attr-defined]
            print(f"q4_0 {key}")
    np.savez_compressed(HERE / "q4_0_reference.npz", **q4)

    q4_scales = np.array([0.0, -0.5, np.float16(2**-14)], dtype=np.float16)
    q4_codes = np.stack((np.zeros(32, dtype=np.uint8), np.full(32, 15, dtype=np.uint8), np.arange(32, dtype=np.uint8) % 16))
    q8_scales = np.array([0.0, 0.125], dtype=np.float16)
    q8_values = np.stack((np.full(32, -128, np.int16), np.full(32, 127, np.int16)))
    q4_blocks = ggml.pack_ggml_q4_0_blocks(q4_scales, q4_codes)  # type: ignore[attr-defined]
    q8_blocks = ggml.pack_ggml_q8_0_blocks(q8_scales, q8_values)  # type: ignore[attr-defined]
    q4_decoded = ggml.unpack_ggml_q4_0_blocks(q4_blocks)  # type: ignore[attr-defined]
    q8_decoded = ggml.unpack_ggml_q8_0_blocks(q8_blocks)  # type: ignore[attr-defined]
    np.savez_compressed(
        HERE / "codec_extremes.npz",
        q4_scales=q4_scales,
        q4_codes=q4_codes,
        q4_blocks=q4_blocks,
        q4_decoded_scales=q4_decoded[0],
        q4_decoded_values=q4_decoded[1],
        q8_scales=q8_scales,
        q8_values=q8_values,
        q8_blocks=q8_blocks,
        q8_decoded_scales=q8_decoded[0],
        q8_decoded_values=np.array(q8_decoded[1]),
    )
    print("codec extremes")

    # W8A8 convolution: the reference test's own per-group dynamic reference
    # (tests/test_qpu_xla_conv2d_w8a8.py:14-54) on the inputs of its plan test (:55-89) and of
    # its hybrid-partition test (:92-130), plus _im2col_nchw (src/qpu_xla/ops/conv2d.py:47-79)
    # on a strided, dilated case.
    conv: dict[str, np.ndarray] = {}
    cases = [(f"plan_g{groups}", 1200 + groups, (1, 4, 4, 4), (4, 4 // groups, 3, 3), 1, 1, groups) for groups in (1, 2, 4)]
    for channels, outputs, kernel, stride, groups, size in ((16, 1, 1, 1, 1, 5), (4, 32, 1, 1, 1, 5), (4, 32, 3, 2, 1, 12), (4, 64, 3, 1, 2, 5), (16, 16, 3, 1, 16, 5)):
        seed = 3100 + channels + outputs + kernel + stride + groups + size
        cases.append((f"hybrid_c{channels}_o{outputs}_k{kernel}_s{stride}_g{groups}_n{size}", seed, (1, channels, size, size), (outputs, channels // groups, kernel, kernel), stride, kernel // 2, groups))
    for name, seed, source_shape, weight_shape, stride, padding, groups in cases:
        rng = np.random.default_rng(seed)
        source = rng.standard_normal(source_shape, dtype=np.float32)
        weight = np.ascontiguousarray(rng.standard_normal(weight_shape, dtype=np.float32))
        expected = ref["conv_dynamic_group_reference"](source, weight, groups=groups, stride=stride, padding=padding)  # type: ignore[operator]
        conv[f"{name}_source"] = source
        conv[f"{name}_weight"] = weight
        conv[f"{name}_params"] = np.array([stride, padding, groups], dtype=np.int64)
        conv[f"{name}_expected"] = np.ascontiguousarray(expected, dtype=np.float32)
    rng = np.random.default_rng(77)
    im2col_source = rng.standard_normal((2, 3, 9, 7), dtype=np.float32)
    conv["im2col_source"] = im2col_source
    conv["im2col_expected"] = ref["im2col_nchw"](im2col_source, 3, 2, stride=(2, 1), padding=(1, 2), dilation=(2, 1))  # type: ignore[operator]
    conv["case_names"] = np.array([c[0] for c in cases])
    np.savez_compressed(HERE / "conv2d_w8a8.npz", **conv)
    print("conv2d w8a8:", len(cases), "cases")
    return 0


if __name__ == "__main__":
    sys.exit(main())
