"""Test configuration: the ``gpu`` marker, import paths and shared fixtures.

``-m "not gpu"`` runs everywhere (oracle vs golden vectors, host logic, C-ABI
loading, gloo multi-process logic). ``-m gpu`` runs the CUDA parity tests on a
B200 and calls the kernels through libqpucuda's C-ABI.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parents[1]
PACKAGE_DIR = REPO / "qpu-xla-triton_b200"
GOLDEN = Path(__file__).resolve().parent / "golden"
for path in (str(PACKAGE_DIR), str(REPO)):
    if path not in sys.path:
        sys.path.insert(0, path)


def pytest_configure(config: pytest.Config) -> None:
    config.addinivalue_line("markers", "gpu: needs an NVIDIA B200 (sm_100a) and runs CUDA kernels")


def cuda_available() -> bool:
    try:
        import torch

        return bool(torch.cuda.is_available())
    except Exception:
        return False


def pytest_collection_modifyitems(config: pytest.Config, items: list[pytest.Item]) -> None:
    if cuda_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device in this environment")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def golden() -> dict[str, dict[str, np.ndarray]]:
    """All golden fixtures, loaded once."""
    result: dict[str, dict[str, np.ndarray]] = {}
    for path in sorted(GOLDEN.glob("*.npz")):
        with np.load(path) as data:
            result[path.stem] = {key: data[key] for key in data.files}
    return result


@pytest.fixture(scope="session")
def cuda_device():  # type: ignore[no-untyped-def]
    """One CUDA device (libqpucuda context on GPU 0) shared by the GPU tests."""
    from qpu_xla import Device

    device = Device.open(device_ordinal=0)
    yield device
    device.close()
