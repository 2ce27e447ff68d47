"""The allocation-free W8A8 linear (ff_linear_w8a8_noalloc) against the oracle and the ordinary entry points.

Callers that may not allocate device memory while running (hosts that own all GPU memory through their
own pool, serving loops that forbid cudaMalloc/cudaFree on the hot path, plugins that only receive
buffers) use this entry point: it keeps the int8 activation codes and row scales in a static device
array inside the library, and reports timeouts in an error word the caller passes. Its output must match
the oracle's rot_q8 -> int32 GEMM -> dequantisation -> epilogue (oracle/quant.py) within the tolerance
that allows a code to round the other way at a tie, and ff_rot_q8 followed by ff_gemm_s8 with
caller-allocated codes within fp16 rounding, on two calls in a row (the second call reuses the array the
first one left behind) — and the second call must not change the device's free memory. This file sorts
last so a failure here comes after every other test.
"""

import ctypes as C

import pytest
import torch

from oracle import quant as Q

pytestmark = pytest.mark.gpu


def _inputs(rows, cols, N, seed, norm=True):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(rows, cols, generator=g).half()
    gamma = (1 + 0.1 * torch.randn(cols, generator=g)) if norm else None
    beta = (0.1 * torch.randn(cols, generator=g)) if norm else None
    W = torch.randint(-127, 128, (N, cols), generator=g, dtype=torch.int8)
    cs = torch.rand(N, generator=g) * 1e-3 + 1e-5
    b = torch.randn(N, generator=g) * 0.02
    return x, gamma, beta, W, cs, b


def _oracle(x, gamma, beta, W, cs, b, base, block, epi_name):
    """oracle/quant.py: rot_q8 (LayerNorm eps 1e-6 when gamma is given) -> exact int32 GEMM -> dequant, then
    the epilogue: fp16 output (bias), fp16(base + fp16(y)) (residual), or silu(gate) * up over the
    [gate 64 | up 64] interleaved columns (SwiGLU)."""
    codes, scales = Q.rot_q8(x, gamma, beta, block=block, eps=1e-6)
    y = Q.dequant(Q.gemm_s8_acc(codes, W), scales, cs, b)
    if epi_name == "EPI_BIAS":
        return y.half()
    if epi_name == "EPI_RESIDUAL":
        return (base.float() + y.half().float()).half()
    g = y.view(y.shape[0], -1, 2, 64)
    return Q.silu_mul(g[:, :, 0], g[:, :, 1]).reshape(y.shape[0], -1).half()


def _call(lib, x, gamma, beta, rows, cols, block, W, cs, b, out, N, epi, err, stream):
    return lib.ff_linear_w8a8_noalloc(x.data_ptr(), gamma.data_ptr() if gamma is not None else None,
                                      beta.data_ptr() if beta is not None else None, C.c_float(1e-6), rows, cols,
                                      cols, block, W.data_ptr(), cs.data_ptr(), b.data_ptr(), out.data_ptr(), N, epi,
                                      err.data_ptr() if err is not None else None, stream)


@pytest.mark.parametrize(("rows", "cols", "N", "block", "epi_name", "norm"),
                         [(1025, 1024, 3072, 1024, "EPI_BIAS", True),
                          (2050, 2816, 1024, 128, "EPI_RESIDUAL", True),
                          (700, 1024, 5632, 1024, "EPI_SWIGLU", True),
                          (600, 4864, 1024, 128, "EPI_RESIDUAL", False)])
def test_noalloc_matches_oracle_and_caller_allocated_path(cuda_device, rows, cols, N, block, epi_name, norm):
    from foidfinder_b200 import _lib, ops

    lib = _lib.lib()
    d = cuda_device
    epi = getattr(ops, epi_name)
    out_cols = N // 2 if epi == ops.EPI_SWIGLU else N
    err = torch.zeros(1, dtype=torch.int32, device=d)
    stream = torch.cuda.current_stream(d).cuda_stream
    for call in range(2):
        host = _inputs(rows, cols, N, seed=call, norm=norm)
        x, gamma, beta, W, cs, b = (t.to(d) if t is not None else None for t in host)
        base_h = torch.randn(rows, out_cols, generator=torch.Generator().manual_seed(10 + call)).half()
        base = base_h.to(d)
        # ordinary path: caller-allocated codes and scales
        codes = torch.empty(rows, cols, dtype=torch.int8, device=d)
        scales = torch.empty(rows, device=d)
        ops.rot_q8(x, gamma, beta, codes, scales, block=block, eps=1e-6)
        ref = base.clone()
        ops.gemm_s8(codes, W, scales, cs, b, ref, epi)
        got = base.clone()
        torch.cuda.synchronize()
        free_before = torch.cuda.mem_get_info(d)[0]
        _lib.check(_call(lib, x, gamma, beta, rows, cols, block, W, cs, b, got, N, epi, err, stream),
                   "ff_linear_w8a8_noalloc")
        torch.cuda.synchronize()
        free_after = torch.cuda.mem_get_info(d)[0]
        assert err.item() == 0
        if call == 1:  # the first call may load the library's module (lazy loading); later calls take nothing
            assert free_after == free_before, f"device free memory moved by {free_before - free_after} bytes"
        torch.testing.assert_close(got.float().cpu(), ref.float().cpu(), atol=2e-3, rtol=3e-3)
        want = _oracle(*host, base_h, block, epi_name).float()
        diff = (got.float().cpu() - want).abs()
        # a code may round the other way at a tie (one step of |W| * row scale * col scale, <= 1e-2 here)
        assert diff.max().item() < 1e-2 + 1e-2 * want.abs().max().item(), diff.max().item()
        assert diff.mean().item() < 1e-3, diff.mean().item()


def test_noalloc_rejects_sizes_beyond_its_scratch(cuda_device):
    from foidfinder_b200 import _lib, ops

    lib = _lib.lib()
    d = cuda_device
    rows, cols, N = 8193, 1024, 128
    x = torch.zeros(rows, cols, dtype=torch.float16, device=d)
    W = torch.zeros(N, cols, dtype=torch.int8, device=d)
    cs = torch.ones(N, device=d)
    b = torch.zeros(N, device=d)
    out = torch.zeros(rows, N, dtype=torch.float16, device=d)
    err = torch.zeros(1, dtype=torch.int32, device=d)
    stream = torch.cuda.current_stream(d).cuda_stream
    rc = _call(lib, x, None, None, rows, cols, 1024, W, cs, b, out, N, ops.EPI_BIAS, err, stream)
    assert rc == _lib.FF_ERR_INVALID_ARGUMENT
    assert b"exceed the static scratch limit" in lib.ff_last_error()


def test_noalloc_requires_an_error_word(cuda_device):
    """Without a caller-owned error word a bounded-wait timeout would have nowhere to go: rejected."""
    from foidfinder_b200 import _lib, ops

    lib = _lib.lib()
    d = cuda_device
    rows, cols, N = 64, 1024, 128
    x = torch.zeros(rows, cols, dtype=torch.float16, device=d)
    W = torch.zeros(N, cols, dtype=torch.int8, device=d)
    cs = torch.ones(N, device=d)
    b = torch.zeros(N, device=d)
    out = torch.zeros(rows, N, dtype=torch.float16, device=d)
    rc = _call(lib, x, None, None, rows, cols, 1024, W, cs, b, out, N, ops.EPI_BIAS, None,
               torch.cuda.current_stream(d).cuda_stream)
    assert rc == _lib.FF_ERR_INVALID_ARGUMENT
    assert b"err is NULL" in lib.ff_last_error()
