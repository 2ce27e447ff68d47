"""The kernels only the PixAI-1008 shape uses, each against the CPU oracle or a plain f32 restatement:
GELU fc1 epilogue, H128 rotation of the 4736-wide hidden, window-ordered patchify, pool LayerNorm +
position embedding, and the one-query attention pool."""

import math

import pytest
import torch
import torch.nn.functional as F

from oracle import eva02 as E
from oracle import pixai as PX
from oracle import quant as Q

pytestmark = pytest.mark.gpu


def _rand_i8(shape, gen):
    return torch.randint(-127, 128, shape, generator=gen, dtype=torch.int8)


@pytest.mark.parametrize(("N", "tile"), [(4736, 128), (4736, 0), (2048, 256), (4864, 512)])
def test_gemm_s8_gelu_epilogue(cuda_device, no_device_error, N, tile):
    """fp16 out = gelu_tanh(acc * rs * cs + b) (foidfinder/backends/cuda/csrc/gemm.cuh:137-140, common.cuh:56).
    4736 = 18.5 x 256 columns: only the 128-wide tile fits it."""
    from foidfinder_b200 import ops

    g = torch.Generator().manual_seed(11)
    M, K = 1100, 1024
    A, W = _rand_i8((M, K), g), _rand_i8((N, K), g)
    rs = torch.rand(M, generator=g) * 0.05 + 1e-3
    cs = torch.rand(N, generator=g) * 1e-3 + 1e-5
    b = torch.randn(N, generator=g) * 0.5
    ref = PX.gelu_tanh(Q.dequant(Q.gemm_s8_acc(A, W), rs, cs, b))
    d = cuda_device
    out = torch.full((M, N), float("nan"), dtype=torch.float16, device=d)
    ops.gemm_s8(A.to(d), W.to(d), rs.to(d), cs.to(d), b.to(d), out, ops.EPI_GELU, tile_n=tile)
    torch.cuda.synchronize()
    # tanh.approx.f32 carries ~2^-11 relative error: a few fp16 steps at most.
    torch.testing.assert_close(out.float().cpu(), ref.half().float(), atol=4e-3, rtol=4e-3)


@pytest.mark.parametrize(("rows", "cols"), [(1, 128), (333, 384), (1030, 4736), (64, 1152), (3, 4736), (41, 6272)])
def test_rot_q8_h128_any_width(cuda_device, no_device_error, rows, cols):
    """H128 + per-row int8 over widths outside the fixed set (PixAI's 4736 = 37 x 128), one, two and four
    warps per row, row counts that leave warps of the last CTA without a row."""
    from foidfinder_b200 import ops

    g = torch.Generator().manual_seed(rows + cols)
    x = torch.randn(rows, cols, generator=g)
    x = torch.where(torch.rand(rows, cols, generator=g) < 0.01, x * 20, x).half()
    ref_q, ref_s = Q.rot_q8(x, None, None, block=128)
    d = cuda_device
    out = torch.full((rows, cols), 99, dtype=torch.int8, device=d)
    rs = torch.full((rows,), float("nan"), device=d)
    ops.rot_q8_h128(x.to(d), out, rs)
    torch.cuda.synchronize()
    torch.testing.assert_close(rs.cpu(), ref_s, rtol=2e-5, atol=0)
    diff = (out.cpu().int() - ref_q.int()).abs()
    assert diff.max().item() <= 1
    assert diff.float().mean().item() < 1e-3


@pytest.mark.parametrize(("S", "window"), [(1008, 24), (336, 8), (448, 0)])
def test_patchify_windowed(cuda_device, no_device_error, S, window):
    """Rows in window order: windows row-major, patches row-major inside (reference.py:21-24, :103-107)."""
    from foidfinder_b200 import ops

    p, B = 14, 2
    G = S // p
    g = torch.Generator().manual_seed(S)
    img = torch.randint(0, 256, (B, S, S, 3), generator=g, dtype=torch.uint8)
    mean, std = (0.5, 0.5, 0.5), (0.5, 0.5, 0.5)
    ref = E.patchify(img, p, mean, std)  # row-major [B, G*G, 588]
    if window:
        ref = ref[:, PX.window_perm(G, window)]
    d = cuda_device
    out = torch.full((B * G * G, 640), float("nan"), dtype=torch.float16, device=d)
    ops.patchify_windowed(img.to(d), p, mean, std, window, out)
    torch.cuda.synchronize()
    got = out.cpu()
    assert torch.all(got[:, 588:] == 0)
    torch.testing.assert_close(got[:, :588].float(), ref.reshape(B * G * G, 588).half().float(), atol=0, rtol=1e-3)


def test_layernorm_pos(cuda_device, no_device_error):
    """fp16(LN(x)) + fp16 pos[row % L] in fp16: F.layer_norm on fp16 then the fp16 add (reference.py:135)."""
    from foidfinder_b200 import ops

    g = torch.Generator().manual_seed(5)
    B, L, D = 3, 5184, 1024
    x = (torch.randn(B * L, D, generator=g) * 3 + 0.5).half()
    gam, bet = 1 + 0.1 * torch.randn(D, generator=g), 0.1 * torch.randn(D, generator=g)
    pos = (0.2 * torch.randn(L, D, generator=g)).half()
    ref = (Q.layer_norm(x, gam, bet, 1e-5).half().view(B, L, D) + pos).view(B * L, D)
    d = cuda_device
    out = torch.full((B * L, D), float("nan"), dtype=torch.float16, device=d)
    ops.layernorm_pos(x.to(d), gam.to(d), bet.to(d), 1e-5, pos.to(d), out)
    torch.cuda.synchronize()
    torch.testing.assert_close(out.cpu().float(), ref.float(), atol=4e-3, rtol=2e-3)


@pytest.mark.parametrize(("B", "tokens", "heads"), [(1, 5184, 16), (3, 577, 16), (2, 100, 4), (1, 1, 2)])
def test_pool_query_attention(cuda_device, no_device_error, B, tokens, heads):
    """softmax(q k^T) v with one learned query per head (reference.py:136-138), q carrying the 1/8 scale."""
    from foidfinder_b200 import ops

    g = torch.Generator().manual_seed(B * tokens + heads)
    dim = heads * 64
    q = torch.randn(dim, generator=g) * (1.0 / math.sqrt(64)) * 2.0
    kv = torch.randn(B * tokens, 2 * dim, generator=g).half()
    k = kv[:, :dim].float().view(B, tokens, heads, 64).permute(0, 2, 1, 3)
    v = kv[:, dim:].float().view(B, tokens, heads, 64).permute(0, 2, 1, 3)
    qh = q.view(1, heads, 1, 64).expand(B, heads, 1, 64)
    ref = F.scaled_dot_product_attention(qh, k, v, scale=1.0).reshape(B, dim)
    d = cuda_device
    out = torch.full((B, dim), float("nan"), dtype=torch.float16, device=d)
    ops.pool_query_attention(q.to(d), kv.to(d), B, tokens, out)
    torch.cuda.synchronize()
    torch.testing.assert_close(out.cpu().float(), ref.half().float(), atol=2e-3, rtol=2e-3)
