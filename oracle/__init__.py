"""CPU oracle for the foidfinder int8 forward — TEST INFRASTRUCTURE ONLY.

This package restates, in plain PyTorch on the CPU, the reference algorithm of every kernel on the hot
path (each function cites the reference file:line it follows). It is the checker for the CUDA library:
only `tests/`, `__graft_entry__.smoke()` and `bench.py`'s CPU-baseline / reference arm may import it,
and never as the thing measured or shipped. The product path (`foidfinder_b200`) must not import it.

Pinning: `tests/golden/` holds vectors produced by running the reference's own Python functions
(`tests/golden/make_golden.py`); `tests/test_oracle_golden.py` checks this oracle against them.
"""
