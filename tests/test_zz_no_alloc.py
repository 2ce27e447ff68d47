"""The allocation-free W8A8 linear (ff_linear_w8a8_noalloc) against the ordinary entry points.

Callers that may not allocate device memory while running (hosts that own all GPU memory through their
own pool, serving loops that forbid cudaMalloc/cudaFree on the hot path, plugins that only receive
buffers) use this entry point: it keeps the int8 activation codes and row scales in a static device
array inside the library. Its output must match ff_rot_q8 followed by ff_gemm_s8 with caller-allocated
codes, within the tolerance the other GEMM tests use, on two calls in a row (the second call reuses the
array the first one left behind). This file sorts last so a failure here comes after every other test.
"""

import ctypes as C

import pytest
import torch

pytestmark = pytest.mark.gpu


def _inputs(rows, cols, N, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(rows, cols, generator=g).half()
    gamma = 1 + 0.1 * torch.randn(cols, generator=g)
    beta = 0.1 * torch.randn(cols, generator=g)
    W = torch.randint(-127, 128, (N, cols), generator=g, dtype=torch.int8)
    cs = torch.rand(N, generator=g) * 1e-3 + 1e-5
    b = torch.randn(N, generator=g) * 0.02
    return x, gamma, beta, W, cs, b


@pytest.mark.parametrize(("rows", "cols", "N", "block", "epi_name"), [(1025, 1024, 3072, 1024, "EPI_BIAS"),
                                                                      (2050, 2816, 1024, 128, "EPI_RESIDUAL"),
                                                                      (700, 1024, 5632, 1024, "EPI_SWIGLU")])
def test_noalloc_matches_caller_allocated_path(cuda_device, rows, cols, N, block, epi_name):
    from foidfinder_b200 import _lib, ops

    lib = _lib.lib()
    d = cuda_device
    epi = getattr(ops, epi_name)
    out_cols = N // 2 if epi == ops.EPI_SWIGLU else N
    err = torch.zeros(1, dtype=torch.int32, device=d)
    for call in range(2):
        x, gamma, beta, W, cs, b = (t.to(d) for t in _inputs(rows, cols, N, seed=call))
        base = torch.randn(rows, out_cols, generator=torch.Generator().manual_seed(10 + call)).half().to(d)
        # ordinary path: caller-allocated codes and scales
        codes = torch.empty(rows, cols, dtype=torch.int8, device=d)
        scales = torch.empty(rows, device=d)
        ops.rot_q8(x, gamma, beta, codes, scales, block=block, eps=1e-6)
        ref = base.clone()
        ops.gemm_s8(codes, W, scales, cs, b, ref, epi)
        # allocation-free path through the C ABI
        got = base.clone()
        stream = torch.cuda.current_stream(d).cuda_stream
        rc = lib.ff_linear_w8a8_noalloc(x.data_ptr(), gamma.data_ptr(), beta.data_ptr(), C.c_float(1e-6), rows, cols,
                                        cols, block, W.data_ptr(), cs.data_ptr(), b.data_ptr(), got.data_ptr(), N,
                                        epi, err.data_ptr(), stream)
        _lib.check(rc, "ff_linear_w8a8_noalloc")
        torch.cuda.synchronize()
        assert err.item() == 0
        torch.testing.assert_close(got.float().cpu(), ref.float().cpu(), atol=2e-3, rtol=3e-3)


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
    rc = lib.ff_linear_w8a8_noalloc(x.data_ptr(), None, None, C.c_float(1e-6), rows, cols, cols, 1024, W.data_ptr(),
                                    cs.data_ptr(), b.data_ptr(), out.data_ptr(), N, ops.EPI_BIAS, None,
                                    torch.cuda.current_stream(d).cuda_stream)
    assert rc == _lib.FF_ERR_INVALID_ARGUMENT
    assert b"exceed the static scratch limit" in lib.ff_last_error()
