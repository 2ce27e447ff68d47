"""foidfinder_b200: the int8 forward of foidfinder's `cuda` backend, rebuilt for NVIDIA B200 (sm_100a).

Kernels live in `csrc/` and are reached only through the C ABI of `libfoidfinder_b200.so`
(`include/foidfinder_b200.h`); `ops` wraps them per kernel, `engine.Engine` runs the whole model under
CUDA graphs, and `backend.CUDABackend` keeps the reference's `predict(image)` API.
"""

__version__ = "0.1.0"
