"""Builds libjitcast_b200.so in-tree with nvcc for sm_100a.

Every ``csrc/*.cu`` file is compiled to an object under ``_build/`` (in parallel, skipped when
the object is newer than its sources and headers) and linked into ``libjitcast_b200.so`` next to
this file, so the library travels with the source tree. The CUDA runtime is linked statically.
"""

from __future__ import annotations

import concurrent.futures
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
BUILD = HERE / "_build"
LIB = HERE / "libjitcast_b200.so"
INCLUDE = HERE.parent / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr", "-Xptxas",
         "-warn-spills"]


def nvcc() -> str:
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(path).exists():
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build libjitcast_b200.so")
    return path


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.h")) + sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def _stale(obj: Path, src: Path, deps: list[Path]) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return any(p.stat().st_mtime > t for p in [src, *deps])


def _compile(src: Path, obj: Path, verbose: bool) -> None:
    cmd = [nvcc(), *ARCH, *FLAGS, "-I", str(INCLUDE), "-c", str(src), "-o", str(obj)]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
    if "spill" in r.stderr and "0 bytes spill" not in r.stderr:
        print(r.stderr, file=sys.stderr)


def build(verbose: bool = False, jobs: int | None = None) -> Path:
    """Compiles stale objects and relinks the library if anything changed; returns its path."""
    BUILD.mkdir(exist_ok=True)
    deps = _headers()
    sources = sorted(CSRC.glob("*.cu"))
    todo = [(s, BUILD / (s.stem + ".o")) for s in sources if _stale(BUILD / (s.stem + ".o"), s, deps)]
    if todo:
        workers = jobs or min(len(todo), os.cpu_count() or 4)
        with concurrent.futures.ThreadPoolExecutor(workers) as ex:
            list(ex.map(lambda so: _compile(so[0], so[1], verbose), todo))
    objs = [BUILD / (s.stem + ".o") for s in sources]
    if todo or not LIB.exists() or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objs):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *map(str, objs)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
