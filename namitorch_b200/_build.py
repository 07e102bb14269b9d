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
from concurrent.futures import ThreadPoolExecutor
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


def _compile(nvcc: str, source: Path, obj: Path, ptxas_info: bool) -> subprocess.CompletedProcess:
    cmd = [nvcc, *ARCH_FLAGS, *COMMON_FLAGS, f"-I{INCLUDE_DIR}", "-c", "-o", str(obj), str(source)]
    if ptxas_info:
        cmd.insert(1, "-Xptxas=-v")
    return subprocess.run(cmd, capture_output=True, text=True)


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> Path:
    """Compiles every .cu file into the shared library (skipped when it is up to date).

    Each translation unit is compiled by its own nvcc process (in parallel, one per host
    core at most) into ``_build/`` at the repository root; the objects are then linked into
    the library. Without ``force``, a translation unit is recompiled only when it, or any
    header, is newer than its object."""
    if not force and not is_stale():
        return LIB_PATH
    nvcc = _nvcc()
    obj_dir = REPO_DIR / "_build"
    obj_dir.mkdir(parents=True, exist_ok=True)
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    objects = [obj_dir / (path.stem + ".o") for path in sources()]
    headers = max((path.stat().st_mtime for path in _inputs() if path.suffix != ".cu"), default=0.0)
    todo = [(src, obj) for src, obj in zip(sources(), objects)
            if force or not obj.exists() or obj.stat().st_mtime < max(src.stat().st_mtime, headers)]
    workers = max(1, min(len(todo), os.cpu_count() or 1))
    with ThreadPoolExecutor(max_workers=workers) as pool:
        results = list(pool.map(lambda pair: _compile(nvcc, pair[0], pair[1], ptxas_info), todo))
    for (source, _), result in zip(todo, results):
        if verbose:
            print(" ".join(result.args), file=sys.stderr)
        if result.returncode != 0:
            raise RuntimeError(f"nvcc failed on {source.name} ({result.returncode}):\n{result.stdout}\n{result.stderr}")
        if ptxas_info or verbose:
            sys.stderr.write(result.stdout + result.stderr)
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [nvcc, *ARCH_FLAGS, "-shared", "-o", str(tmp), *[str(o) for o in objects]]
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"nvcc link failed ({result.returncode}):\n{result.stdout}\n{result.stderr}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True, ptxas_info="--ptxas" in sys.argv)
    print(LIB_PATH)
