"""Kernel microbenchmarks on one B200 (BASELINE configs 1 and 2), timed with CUDA events on the launching
stream after warm-up. Also the entry point for ncu captures of single kernels.

    python -m foidfinder_b200.microbench gemm [--batch 64] [--shape 1024x3072] [--iters 20]
                                              [--epilogue bias|swiglu|residual|qkv_rope]
    python -m foidfinder_b200.microbench attention [--batch 64] [--seq 1025] [--iters 20]
    python -m foidfinder_b200.microbench rotate [--batch 64] [--tokens 1025] [--cols 1024 ...] [--iters 20]
    python -m foidfinder_b200.microbench peak      (measured dense int8 tensor-core TOPS)

PixAI-1008 shapes: `attention --batch 144 --seq 576` (16 images x 9 windows), `attention --batch 16 --seq
5184` (global blocks), `rotate --batch 16 --tokens 5184 --cols 1024 --cols 4864`.

Each prints one JSON line per case: shape, ms per launch, and achieved TFLOP/s (GEMM: 2*M*N*K int8 ops;
attention: 4*B*heads*T^2*64) or GB/s (rotation: algorithmic bytes read + written).
"""

from __future__ import annotations

import argparse
import json

import torch

from . import ops

GEMM_SHAPES = {  # (K, N) of BASELINE config 1; N of the gate|up GEMM is the interleaved padded 2 x 2816
    "1024x3072": (1024, 3072, "qkv"),
    "1024x1024": (1024, 1024, "proj"),
    "1024x5632": (1024, 5632, "gate|up (5460 unpadded)"),
    "2816x1024": (2816, 1024, "down (2730 unpadded)"),
}
TOKENS = 1025


def _time(fn, iters: int, warmup: int = 3) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters


def bench_gemm(batch: int, shapes: list[str], iters: int, epi: str, tile: int = 0) -> None:
    d = torch.device("cuda")
    g = torch.Generator(device=d).manual_seed(0)
    M = TOKENS * batch
    for name in shapes:
        K, N, what = GEMM_SHAPES[name]
        A = torch.randint(-127, 128, (M, K), generator=g, device=d, dtype=torch.int8)
        W = torch.randint(-127, 128, (N, K), generator=g, device=d, dtype=torch.int8)
        rs = torch.rand(M, generator=g, device=d) * 1e-2
        cs = torch.rand(N, generator=g, device=d) * 1e-3
        b = torch.randn(N, generator=g, device=d) * 0.02
        e = {"bias": ops.EPI_BIAS, "swiglu": ops.EPI_SWIGLU, "residual": ops.EPI_RESIDUAL,
             "qkv_rope": ops.EPI_QKV_ROPE}[epi]
        out = torch.zeros(M, N // 2 if e == ops.EPI_SWIGLU else N, device=d, dtype=torch.float16)
        rope = {}
        if e == ops.EPI_QKV_ROPE:
            from .weights import rope_tables

            cos, sin = (t.t().contiguous().to(d) for t in rope_tables(32, 16))  # angle-major
            rope = dict(rope_cos=cos, rope_sin=sin, rope_cols=2 * N // 3, tokens=TOKENS)
        ms = _time(lambda: ops.gemm_s8(A, W, rs, cs, b, out, e, tile_n=tile, **rope), iters)
        n_alg = {"1024x5632": 5460, "2816x1024": 1024}.get(name, N)
        k_alg = 2730 if name == "2816x1024" else K
        ops_alg = 2 * M * n_alg * k_alg
        print(json.dumps({"kernel": "gemm_s8", "shape": name, "what": what, "M": M, "N": N, "K": K, "epilogue": epi,
                          "tile_n": tile,
                          "ms": ms, "tflops": ops_alg / ms / 1e9,
                          "bytes": M * K + N * K + out.numel() * 2, "gbs": (M * K + N * K + out.numel() * 2) / ms / 1e6}))


def bench_attention(batch: int, iters: int, seq: int = TOKENS, heads: int = 16) -> None:
    d = torch.device("cuda")
    g = torch.Generator(device=d).manual_seed(0)
    qkv = torch.randn(batch * seq, 3 * heads * 64, generator=g, device=d).half()
    out = torch.empty(batch * seq, heads * 64, device=d, dtype=torch.float16)
    ms = _time(lambda: ops.attention(qkv, out, seq, heads, scale=0.125), iters)
    flops = 4 * batch * heads * seq * seq * 64
    print(json.dumps({"kernel": "attention", "batch": batch, "tokens": seq, "heads": heads,
                      "ms": ms, "tflops": flops / ms / 1e9}))


ROT_CASES = {  # cols -> the engine's rotations of that width: (valid, block, LayerNorm)
    1024: ((1024, 1024, True), (1024, 1024, False)),
    2816: ((2730, 128, True),),
    4864: ((4864, 128, False),),  # PixAI GELU hidden 4736 padded to 4864
}


def bench_rotate(batch: int, iters: int, tokens: int = TOKENS, widths: list[int] | None = None) -> None:
    d = torch.device("cuda")
    g = torch.Generator(device=d).manual_seed(0)
    M = tokens * batch
    cases = [(c, *v) for c in (widths or (1024, 2816)) for v in ROT_CASES[c]]
    for cols, valid, block, norm in cases:
        x = torch.randn(M, cols, generator=g, device=d).half()
        gamma = torch.ones(cols, device=d) if norm else None
        beta = torch.zeros(cols, device=d) if norm else None
        out = torch.empty(M, cols, device=d, dtype=torch.int8)
        rs = torch.empty(M, device=d)
        ms = _time(lambda: ops.rot_q8(x, gamma, beta, out, rs, block=block, valid_cols=valid), iters)
        nbytes = M * cols * 3 + M * 4
        print(json.dumps({"kernel": "rot_q8", "cols": cols, "block": block, "norm": norm, "M": M, "ms": ms,
                          "gbs": nbytes / ms / 1e6}))


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("kernel", choices=("gemm", "attention", "rotate", "peak"))
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--shape", action="append", choices=sorted(GEMM_SHAPES))
    ap.add_argument("--epilogue", default="bias", choices=("bias", "swiglu", "residual", "qkv_rope"))
    ap.add_argument("--tile", type=int, default=0, help="gemm: tile_n (0 auto, 128, 256, 512 = pair tiles)")
    ap.add_argument("--seq", type=int, default=TOKENS, help="attention: sequence length")
    ap.add_argument("--tokens", type=int, default=TOKENS, help="rotate: rows per image")
    ap.add_argument("--cols", type=int, action="append", choices=sorted(ROT_CASES), help="rotate: row widths")
    a = ap.parse_args()
    if a.kernel == "peak":
        for _ in range(3):
            print(json.dumps({"kernel": "int8_mma_peak", "tops": ops.int8_mma_peak()}))
    elif a.kernel == "gemm":
        bench_gemm(a.batch, a.shape or list(GEMM_SHAPES), a.iters, a.epilogue, a.tile)
    elif a.kernel == "attention":
        bench_attention(a.batch, a.iters, a.seq)
    else:
        bench_rotate(a.batch, a.iters, a.tokens, a.cols)
    torch.cuda.synchronize()
    err = ops.device_error(0)
    if err:
        raise SystemExit(f"device error word {err}")


if __name__ == "__main__":
    main()
