"""Builds libt2c_sm100.so in-tree with nvcc for sm_100a.

Usage: ``python -m torch2vk_b200.build`` (or ``__graft_entry__.build()``).
Objects go to ``torch2vk_b200/_build/``; the shared library lands next to this
file so it travels with the source tree.
"""

from __future__ import annotations

import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PACKAGE_DIR = Path(__file__).resolve().parent
CSRC = PACKAGE_DIR / "csrc"
BUILD_DIR = PACKAGE_DIR / "_build"
LIB_NAME = "libt2c_sm100.so"
LIB_PATH = PACKAGE_DIR / LIB_NAME

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler",
    "-fPIC",
    "--expt-relaxed-constexpr",
    "-Xptxas",
    "-v",
]
# Files whose arithmetic must be reproducible bit for bit (no FMA contraction).
NO_FMAD = {"quantize.cu"}


def _nvcc() -> str:
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    candidate = Path(cuda_home) / "bin" / "nvcc"
    return str(candidate) if candidate.exists() else "nvcc"


def _compile(source: Path) -> tuple[Path, str]:
    obj = BUILD_DIR / (source.stem + ".o")
    deps = [source, *CSRC.glob("*.cuh"), PACKAGE_DIR.parent / "include" / "t2c_sm100.h"]
    if obj.exists() and all(obj.stat().st_mtime >= d.stat().st_mtime for d in deps if d.exists()):
        return obj, ""
    flags = list(COMMON_FLAGS)
    if source.name in NO_FMAD:
        flags.append("--fmad=false")
    cmd = [_nvcc(), *ARCH_FLAGS, *flags, "-c", str(source), "-o", str(obj)]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed for {source.name}:\n{proc.stderr}")
    return obj, proc.stderr


def build(verbose: bool = False) -> Path:
    BUILD_DIR.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as pool:
        results = list(pool.map(_compile, sources))
    objects = [obj for obj, _ in results]
    if verbose:
        for _, log in results:
            if log:
                sys.stderr.write(log)
    newest = max(o.stat().st_mtime for o in objects)
    if not LIB_PATH.exists() or LIB_PATH.stat().st_mtime < newest:
        cmd = [_nvcc(), *ARCH_FLAGS, "-shared", "-o", str(LIB_PATH), *map(str, objects), "-lcudart"]
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            raise RuntimeError(f"link failed:\n{proc.stderr}")
    return LIB_PATH


if __name__ == "__main__":
    path = build(verbose="-v" in sys.argv)
    print(path)
