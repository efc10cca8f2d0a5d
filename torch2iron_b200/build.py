"""Build ``libt2b.so`` (the C-ABI library) from ``csrc/*.cu`` for sm_100a.

    python -m torch2iron_b200.build [--force]

Each translation unit is compiled in parallel with
``nvcc -gencode arch=compute_100a,code=sm_100a -O3 -lineinfo`` into
``_build/`` and linked into ``torch2iron_b200/libt2b.so`` (in-tree, so the
built library travels with the source tree).  Rebuilds only when a source or
header is newer than the library.
"""

from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = ROOT / "_build"
LIB = PKG / "libt2b.so"
TRACE_LIB = BUILD / "libt2b_trace.so"   # -DT2B_TRACE: device phase timestamps (diagnostics only, kept out of the package)

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC",
         "-Xcompiler", "-fvisibility=hidden", "-I", str(ROOT / "include")]


def nvcc() -> str:
    exe = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(exe).exists():
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libt2b.so")
    return exe


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _stale(lib: Path) -> bool:
    if not lib.exists():
        return True
    t = lib.stat().st_mtime
    deps = list(CSRC.glob("*")) + list((ROOT / "include").glob("*.h"))
    return any(p.stat().st_mtime > t for p in deps)


def _compile(src: Path, extra: list[str], suffix: str = "") -> Path:
    obj = BUILD / (src.stem + suffix + ".o")
    cmd = [nvcc(), *ARCH, *FLAGS, *extra, "-c", str(src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stderr}")
    if r.stderr.strip():
        sys.stderr.write(r.stderr)
    return obj


def build(force: bool = False, verbose_ptxas: bool = False, trace: bool = False) -> Path:
    lib = TRACE_LIB if trace else LIB
    if not force and not _stale(lib):
        return lib
    BUILD.mkdir(exist_ok=True)
    extra = ["-Xptxas", "-v"] if verbose_ptxas else []
    suffix = ""
    if trace:
        extra = extra + ["-DT2B_TRACE"]
        suffix = "_trace"
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(lambda s: _compile(s, extra, suffix), sources()))
    tmp = lib.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *map(str, objs)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stderr}")
    os.replace(tmp, lib)
    return lib


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose_ptxas="--ptxas-v" in sys.argv, trace="--trace" in sys.argv))
