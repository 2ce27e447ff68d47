"""Builds the sm_100a kernel library `foidfinder_b200/_lib/libfoidfinder_b200.so` with nvcc.

Same role as the reference's loader/build step (foidfinder/backends/cuda/kernels.py:22-35,
`foidfinder build-kernels`), but ahead of time, in-tree and for `compute_100a` only: each `.cu` in
`csrc/` is compiled to an object in parallel and linked into one shared library that exports the C ABI
declared in `include/foidfinder_b200.h`. The CUDA runtime is linked statically, so the library needs
only the driver at run time.

    python -m foidfinder_b200.build [--force] [--jobs N]
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
BUILD = ROOT / "_build"
LIB_DIR = PKG / "_lib"
LIB = LIB_DIR / "libfoidfinder_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden", f"-I{INCLUDE}"]


def nvcc() -> str:
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(path).exists():
        raise RuntimeError("nvcc not found; the CUDA 12.9 toolkit is required to build foidfinder_b200")
    return path


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(force: bool = False, jobs: int | None = None, verbose: bool = False) -> Path:
    """Compiles (incrementally) and links the library; returns its path."""
    BUILD.mkdir(exist_ok=True)
    LIB_DIR.mkdir(exist_ok=True)
    headers = sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE.glob("*.h"))
    cc = nvcc()
    todo = []
    objects = []
    for src in sources():
        obj = BUILD / (src.stem + ".o")
        objects.append(obj)
        if force or _stale(obj, [src, *headers]):
            todo.append((src, obj))

    def compile_one(item: tuple[Path, Path]) -> tuple[Path, str]:
        src, obj = item
        cmd = [cc, *ARCH, *FLAGS, "-c", str(src), "-o", str(obj)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
        return src, r.stderr

    with cf.ThreadPoolExecutor(max_workers=jobs or os.cpu_count() or 4) as ex:
        for src, log in ex.map(compile_one, todo):
            if verbose:
                print(f"compiled {src.name}", log, file=sys.stderr)
    if force or todo or _stale(LIB, objects):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [cc, *ARCH, "-shared", "-o", str(tmp), *map(str, objects), "-cudart", "static"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=None)
    args = ap.parse_args()
    print(build(force=args.force, jobs=args.jobs, verbose=True))


if __name__ == "__main__":
    main()
