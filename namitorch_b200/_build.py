"""Builds ``libnamitorch_b200.so`` (sm_100a) in-tree with nvcc.

The library is compiled from ``namitorch_b200/csrc/*.cu`` against the public header in
``include/``. The output lives at ``namitorch_b200/lib/libnamitorch_b200.so`` so that it
travels with the source tree (nothing is installed into site-packages or a JIT cache).
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE_DIR = Path(__file__).resolve().parent
REPO_DIR = PACKAGE_DIR.parent
CSRC_DIR = PACKAGE_DIR / "csrc"
INCLUDE_DIR = REPO_DIR / "include"
LIB_DIR = PACKAGE_DIR / "lib"
LIB_PATH = LIB_DIR / "libnamitorch_b200.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
# No --use_fast_math: the optimizer kernels rely on IEEE division / square root and on
# subnormal support to stay bit-identical to the NumPy reference path.
COMMON_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-O2",
                "--expt-relaxed-constexpr"]


def _nvcc() -> str:
    candidates = [os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"]
    for candidate in candidates:
        if candidate and Path(candidate).exists():
            return candidate
    raise RuntimeError("nvcc was not found; set NVCC or add /usr/local/cuda/bin to PATH.")


def sources() -> list[Path]:
    return sorted(CSRC_DIR.glob("*.cu"))


def _inputs() -> list[Path]:
    return sources() + sorted(CSRC_DIR.glob("*.cuh")) + sorted(INCLUDE_DIR.glob("*.h")) + [Path(__file__)]


def is_stale() -> bool:
    if not LIB_PATH.exists():
        return True
    built = LIB_PATH.stat().st_mtime
    return any(path.stat().st_mtime > built for path in _inputs())


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> Path:
    """Compiles every .cu file into the shared library (skipped when it is up to date)."""
    if not force and not is_stale():
        return LIB_PATH
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [_nvcc(), *ARCH_FLAGS, *COMMON_FLAGS, f"-I{INCLUDE_DIR}", "-shared", "-o", str(tmp),
           *[str(path) for path in sources()]]
    if ptxas_info:
        cmd.insert(1, "-Xptxas=-v")
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"nvcc failed ({result.returncode}):\n{result.stdout}\n{result.stderr}")
    if ptxas_info or verbose:
        sys.stderr.write(result.stdout + result.stderr)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True, ptxas_info="--ptxas" in sys.argv)
    print(LIB_PATH)
