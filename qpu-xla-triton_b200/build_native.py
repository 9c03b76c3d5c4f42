"""Build libqpucuda.so (the CUDA kernels and the C-ABI) in-tree for sm_100a.

Usage: ``python qpu-xla-triton_b200/build_native.py [--force]``. Objects go to
``qpu-xla-triton_b200/_build/``; the library lands at
``qpu-xla-triton_b200/qpu_xla/_native/libqpucuda.so`` where the ``qpu_xla``
package loads it. Only the static CUDA runtime is linked, so the library loads
(and reports "device unavailable") on a machine without a GPU driver.
"""

from __future__ import annotations

import argparse
import hashlib
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PACKAGE_ROOT = Path(__file__).resolve().parent
REPO_ROOT = PACKAGE_ROOT.parent
CSRC = PACKAGE_ROOT / "csrc"
INCLUDE = REPO_ROOT / "include"
BUILD = PACKAGE_ROOT / "_build"
OUTPUT = PACKAGE_ROOT / "qpu_xla" / "_native" / "libqpucuda.so"
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
VERSION = "0.1.0"


def nvcc() -> str:
    candidates = [shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"]
    for candidate in candidates:
        if candidate and Path(candidate).exists():
            return candidate
    raise RuntimeError("nvcc not found; the CUDA toolkit is required to build libqpucuda.so")


Q4_0_KERNEL_SOURCES = ("q4_0_gemv.cu", "q4_0_mx_sm100.cu")


def q4_0_source_hash() -> str:
    """SHA-256 of the Q4_0 kernel sources (concatenated): the identity Q4_0 linears are prepared against."""
    return hashlib.sha256(b"".join((CSRC / name).read_bytes() for name in Q4_0_KERNEL_SOURCES)).hexdigest()


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def common_flags() -> list[str]:
    return [
        "-std=c++17",
        "-O3",
        "-lineinfo",
        *ARCH_FLAGS,
        "-Xcompiler",
        "-fPIC",
        "-Xcompiler",
        "-fvisibility=hidden",
        f"-I{INCLUDE}",
        f"-I{CSRC}",
        f'-DQPUCUDA_VERSION="{VERSION}"',
        f'-DQPUCUDA_Q4_0_SOURCE_HASH="{q4_0_source_hash()}"',
    ]


def _stamp() -> str:
    digest = hashlib.sha256()
    for path in sorted([*sources(), *CSRC.glob("*.h"), *CSRC.glob("*.cuh"), *INCLUDE.glob("*.h"), Path(__file__)]):
        digest.update(path.name.encode())
        digest.update(path.read_bytes())
    return digest.hexdigest()


def build(force: bool = False, verbose: bool = False) -> Path:
    stamp_file = BUILD / "stamp"
    stamp = _stamp()
    if not force and OUTPUT.exists() and stamp_file.exists() and stamp_file.read_text() == stamp:
        return OUTPUT
    BUILD.mkdir(parents=True, exist_ok=True)
    OUTPUT.parent.mkdir(parents=True, exist_ok=True)
    compiler = nvcc()
    flags = common_flags()

    def compile_one(source: Path) -> Path:
        obj = BUILD / (source.stem + ".o")
        command = [compiler, *flags, "-c", str(source), "-o", str(obj)]
        if verbose:
            print(" ".join(command), flush=True)
        result = subprocess.run(command, capture_output=True, text=True)
        if result.returncode != 0:
            raise RuntimeError(f"nvcc failed for {source.name}:\n{result.stdout}\n{result.stderr}")
        return obj

    workers = max(1, min(len(sources()), os.cpu_count() or 1))
    with ThreadPoolExecutor(max_workers=workers) as pool:
        objects = list(pool.map(compile_one, sources()))
    # The public C entry points are the only exported symbols.
    link = [compiler, *ARCH_FLAGS, "-shared", "-Xcompiler", "-fPIC", *map(str, objects), "-o", str(OUTPUT)]
    if verbose:
        print(" ".join(link), flush=True)
    result = subprocess.run(link, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"link failed:\n{result.stdout}\n{result.stderr}")
    stamp_file.write_text(stamp)
    return OUTPUT


def main(argv: list[str] | None = None) -> int:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--verbose", action="store_true")
    args = parser.parse_args(argv)
    path = build(force=args.force, verbose=args.verbose)
    print(path)
    return 0


if __name__ == "__main__":
    sys.exit(main())
