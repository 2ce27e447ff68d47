"""tcgen05 GEMM vs the CPU oracle: int32 accumulators bit-exact, every epilogue within fp16 rounding.

Parity bar: int32 GEMM accumulators bit-exact; dequantised activations within
2e-2 absolute (the epilogue checks below are far tighter: f32 math then one fp16 rounding).
"""

import pytest
import torch

from oracle import quant as Q

pytestmark = pytest.mark.gpu


def _rand_i8(shape, gen):
    return torch.randint(-127, 128, shape, generator=gen, dtype=torch.int8)


# Smallest case first: a single 128 x 256 tile with one K stage.
S32_CASES = [
    (128, 256, 128, 256),
    (1, 256, 128, 256),
    (129, 128, 256, 128),
    (1025, 3072, 1024, 0),
    (1025, 1024, 2816, 128),
    (2050, 5632, 1024, 256),
    (777, 768, 768, 256),
    (4100, 2304, 768, 0),
]


PAIR = 512  # ops.TILE_PAIR256: 256 x 256 tiles over a cluster of two CTAs (tcgen05 cta_group::2)

# Pair tiles, smallest first: one pair tile, a ragged last 256-row tile, several tiles per cluster.
PAIR_S32_CASES = [
    (256, 256, 128, PAIR),
    (300, 256, 256, PAIR),
    (1025, 3072, 1024, PAIR),
    (2050, 5632, 1024, PAIR),
    (4100, 2304, 768, PAIR),
    (65600 // 4, 1024, 2816, PAIR),
]


@pytest.mark.parametrize(("M", "N", "K", "tile"), PAIR_S32_CASES + S32_CASES)
def test_gemm_s8_int32_bit_exact(cuda_device, no_device_error, M, N, K, tile):
    g = torch.Generator().manual_seed(M * 131 + N * 7 + K)
    A, W = _rand_i8((M, K), g), _rand_i8((N, K), g)
    from foidfinder_b200 import ops

    out = torch.full((M, N), -(2**31), dtype=torch.int32, device=cuda_device)
    ops.gemm_s8(A.to(cuda_device), W.to(cuda_device), None, None, None, out, ops.EPI_S32, tile_n=tile)
    torch.cuda.synchronize()
    assert torch.equal(out.cpu(), Q.gemm_s8_acc(A, W))


def _dequant_case(M, N, K, gen):
    A, W = _rand_i8((M, K), gen), _rand_i8((N, K), gen)
    rs = torch.rand(M, generator=gen) * 0.05 + 1e-3
    cs = torch.rand(N, generator=gen) * 1e-3 + 1e-5
    b = torch.randn(N, generator=gen) * 0.02
    return A, W, rs, cs, b


@pytest.mark.parametrize("tile", [128, 256, PAIR])
def test_gemm_s8_bias_epilogue(cuda_device, no_device_error, tile):
    from foidfinder_b200 import ops

    M, N, K = 1025, 1024, 1024
    A, W, rs, cs, b = _dequant_case(M, N, K, torch.Generator().manual_seed(1))
    ref = Q.dequant(Q.gemm_s8_acc(A, W), rs, cs, b)
    d = cuda_device
    out = torch.full((M, N), float("nan"), dtype=torch.float16, device=d)
    ops.gemm_s8(A.to(d), W.to(d), rs.to(d), cs.to(d), b.to(d), out, ops.EPI_BIAS, tile_n=tile)
    torch.cuda.synchronize()
    torch.testing.assert_close(out.float().cpu(), ref.half().float(), atol=1e-3, rtol=2e-3)


@pytest.mark.parametrize("tile", [128, 256, PAIR])
def test_gemm_s8_residual_epilogue(cuda_device, no_device_error, tile):
    """x = fp16(x + fp16(y)): the reference stages y in fp16 and adds with __hadd2
    (foidfinder/backends/cuda/csrc/gemm.cuh:153-169); here a TMA add-reduction does the same add."""
    from foidfinder_b200 import ops

    M, N, K = 1025, 1024, 2816
    A, W, rs, cs, b = _dequant_case(M, N, K, torch.Generator().manual_seed(2))
    x0 = torch.randn(M, N, generator=torch.Generator().manual_seed(3)).half()
    ref = (x0.float() + Q.dequant(Q.gemm_s8_acc(A, W), rs, cs, b).half().float()).half()
    d = cuda_device
    x = x0.to(d)
    ops.gemm_s8(A.to(d), W.to(d), rs.to(d), cs.to(d), b.to(d), x, ops.EPI_RESIDUAL, tile_n=tile)
    torch.cuda.synchronize()
    got = x.cpu()
    torch.testing.assert_close(got.float(), ref.float(), atol=2e-3, rtol=2e-3)
    # y's f32 rounding differs from torch's only at fp16 ties, so nearly every element is bit-identical.
    assert (got == ref).float().mean().item() > 0.999


@pytest.mark.parametrize("tile", [128, 256, PAIR])
def test_gemm_s8_swiglu_epilogue(cuda_device, no_device_error, tile):
    from foidfinder_b200 import ops

    M, N, K = 700, 2 * 2816, 1024
    A, W, rs, cs, b = _dequant_case(M, N, K, torch.Generator().manual_seed(4))
    y = Q.dequant(Q.gemm_s8_acc(A, W), rs, cs, b)
    # rows of W are [gate 64 | up 64] pairs
    yg = y.view(M, N // 128, 2, 64)
    ref = Q.silu_mul(yg[:, :, 0], yg[:, :, 1]).reshape(M, N // 2)
    d = cuda_device
    out = torch.full((M, N // 2), float("nan"), dtype=torch.float16, device=d)
    ops.gemm_s8(A.to(d), W.to(d), rs.to(d), cs.to(d), b.to(d), out, ops.EPI_SWIGLU, tile_n=tile)
    torch.cuda.synchronize()
    torch.testing.assert_close(out.float().cpu(), ref.half().float(), atol=2e-3, rtol=3e-3)


@pytest.mark.parametrize("tile", [0, PAIR])
def test_gemm_s8_qkv_rope_epilogue(cuda_device, no_device_error, tile):
    from foidfinder_b200 import ops

    tokens, dim = 1025, 1024
    M, N, K = 2 * tokens, 3 * dim, 1024
    A, W, rs, cs, b = _dequant_case(M, N, K, torch.Generator().manual_seed(5))
    g = torch.Generator().manual_seed(6)
    ang = torch.rand(tokens, 32, generator=g) * 6.28
    ang[0] = 0.0
    cos, sin = torch.cos(ang), torch.sin(ang)
    pos = torch.arange(M) % tokens
    ref = Q.apply_rope_pairs(Q.dequant(Q.gemm_s8_acc(A, W), rs, cs, b), cos, sin, pos, 2 * dim)
    d = cuda_device
    out = torch.full((M, N), float("nan"), dtype=torch.float16, device=d)
    ops.gemm_s8(
        A.to(d), W.to(d), rs.to(d), cs.to(d), b.to(d), out, ops.EPI_QKV_ROPE,
        rope_cos=cos.t().contiguous().to(d), rope_sin=sin.t().contiguous().to(d), rope_cols=2 * dim, tokens=tokens,
        tile_n=tile,
    )
    torch.cuda.synchronize()
    torch.testing.assert_close(out.float().cpu(), ref.half().float(), atol=2e-3, rtol=3e-3)


def test_gemm_f16_logits_epilogue(cuda_device, no_device_error):
    from foidfinder_b200 import ops

    g = torch.Generator().manual_seed(7)
    B, K, n_tags, n_pad = 5, 1024, 30877, 30976
    A = torch.randn(B, K, generator=g).half()
    W = (torch.randn(n_pad, K, generator=g) * 0.02).half()
    W[n_tags:] = 0
    bias = torch.randn(n_pad, generator=g) * 0.02
    ref = A.float() @ W.float().t() + bias
    d = cuda_device
    out = torch.full((B, n_tags), float("nan"), dtype=torch.float32, device=d)
    ops.gemm_f16(A.to(d), W.to(d), out, ops.EPI_LOGITS, bias=bias.to(d), n_valid=n_tags)
    torch.cuda.synchronize()
    torch.testing.assert_close(out.cpu(), ref[:, :n_tags], atol=1e-4, rtol=1e-4)


@pytest.mark.parametrize("M", [1025 * 3, 77])
def test_gemm_f16_bias_epilogue(cuda_device, no_device_error, M):
    """fp16 x fp16 -> f32 accumulation + bias -> fp16 (the tree pool's key/value projection shape)."""
    from foidfinder_b200 import ops

    g = torch.Generator().manual_seed(9)
    K, N = 768, 1536
    A = torch.randn(M, K, generator=g).half()
    W = (torch.randn(N, K, generator=g) * 0.05).half()
    bias = torch.randn(N, generator=g) * 0.1
    ref = (A.float() @ W.float().t() + bias).half()
    d = cuda_device
    out = torch.full((M, N), float("nan"), dtype=torch.float16, device=d)
    ops.gemm_f16(A.to(d), W.to(d), out, ops.EPI_BIAS, bias=bias.to(d))
    torch.cuda.synchronize()
    # f32 accumulation in a different order, then one fp16 rounding: at most one fp16 ulp apart.
    torch.testing.assert_close(out.cpu().float(), ref.float(), atol=2e-3, rtol=1e-3)


def test_gemm_f16_stem_epilogue(cuda_device, no_device_error):
    from foidfinder_b200 import ops

    g = torch.Generator().manual_seed(8)
    B, P, T, D, K = 3, 1024, 1025, 1024, 640
    A = torch.randn(B * P, K, generator=g).half()
    A[:, 588:] = 0
    W = (torch.randn(D, K, generator=g) * 0.02).half()
    pos_bias = torch.randn(P, D, generator=g) * 0.02
    ref = (A.float() @ W.float().t()).view(B, P, D) + pos_bias
    d = cuda_device
    x = torch.full((B * T, D), float("nan"), dtype=torch.float16, device=d)
    ops.gemm_f16(A.to(d), W.to(d), x, ops.EPI_STEM, pos_bias=pos_bias.to(d), patches=P, tokens=T)
    torch.cuda.synchronize()
    got = x.view(B, T, D).cpu()
    assert torch.isnan(got[:, 0]).all()  # the class-token row is not written by the stem
    torch.testing.assert_close(got[:, 1:].float(), ref.half().float(), atol=2e-3, rtol=3e-3)
