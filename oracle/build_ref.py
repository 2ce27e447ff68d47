"""Compiles the reference's own CUDA kernels (foidfinder/backends/cuda/csrc/kernels.cu with its two headers,
the `torch.ops.foidfinder` extension of foidfinder/backends/cuda/kernels.py:21-35) for sm_100 into
oracle/_ref/pixai_kernels.so — test infrastructure only: the GPU parity tests load it as a second checker
next to the CPU oracle (same inputs through the reference's kernels and through this library's).

The sources are compiled where they lie (nothing is copied), with the reference's own compiler flags
(-O3 -std=c++20 --expt-relaxed-constexpr) plus sm_100 code generation, through
torch.utils.cpp_extension (ninja) into oracle/_ref/ only.

    python -m oracle.build_ref /path/to/reference       (or FOIDFINDER_REFERENCE=/path/to/reference)
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

OUT = Path(__file__).resolve().parent / "_ref"
NAME = "pixai_kernels"


def reference_root(ref_root: str | os.PathLike | None = None) -> Path | None:
    """The reference checkout: the argument, else $FOIDFINDER_REFERENCE, else None."""
    root = ref_root if ref_root is not None else os.environ.get("FOIDFINDER_REFERENCE")
    return Path(root) if root else None


def build(ref_root: str | os.PathLike | None = None, verbose: bool = False) -> Path | None:
    """Returns the built library, or None when no reference tree is given or found (e.g. on a GPU box)."""
    root = reference_root(ref_root)
    if root is None:
        return None
    csrc = root / "foidfinder" / "backends" / "cuda" / "csrc"
    if not (csrc / "kernels.cu").is_file():
        return None
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0")
    from torch.utils.cpp_extension import load

    OUT.mkdir(parents=True, exist_ok=True)
    load(
        name=NAME,
        sources=[str(csrc / "kernels.cu")],
        extra_include_paths=[str(csrc)],
        extra_cuda_cflags=["-O3", "-std=c++20", "--expt-relaxed-constexpr", "-lineinfo"],
        build_directory=str(OUT),
        is_python_module=False,
        verbose=verbose,
    )
    return OUT / f"{NAME}.so"


if __name__ == "__main__":
    print(build(sys.argv[1] if len(sys.argv) > 1 else None, verbose=True))
