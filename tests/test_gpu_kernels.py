"""Rotation/quantisation, attention, LayerNorm, patchify and top-k kernels vs the CPU oracle."""

import math

import pytest
import torch

from oracle import eva02 as E
from oracle import quant as Q

pytestmark = pytest.mark.gpu


def _activations(rows, cols, seed):
    """N(0, 1) with 1% outliers x20 (BASELINE config 1 activation model)."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(rows, cols, generator=g)
    mask = torch.rand(rows, cols, generator=g) < 0.01
    return torch.where(mask, x * 20, x).half()


ROT_CASES = [
    # (rows, cols, valid, block, norm)
    (1025, 1024, 1024, 1024, True),
    (1025, 1024, 1024, 1024, False),
    (2050, 2816, 2730, 128, True),
    (3, 2816, 2816, 128, True),  # an odd row count: the last CTA of the split kernel has a row without data
    (1, 2816, 2730, 128, True),
    (1025, 2816, 2816, 128, False),
    (777, 768, 768, 256, True),
    (300, 2048, 2048, 128, True),
    (513, 1024, 1024, 128, False),
    (7, 4096, 4096, 512, False),
    (1, 1024, 1024, 1024, True),
]


@pytest.mark.parametrize(("rows", "cols", "valid", "block", "norm"), ROT_CASES)
def test_rot_q8_matches_oracle(cuda_device, no_device_error, rows, cols, valid, block, norm):
    from foidfinder_b200 import ops

    x = _activations(rows, cols, rows + cols)
    g = torch.Generator().manual_seed(9)
    gamma = (1 + 0.1 * torch.randn(cols, generator=g)) if norm else None
    beta = (0.1 * torch.randn(cols, generator=g)) if norm else None
    ref_q, ref_s = Q.rot_q8(x, gamma, beta, block=block, eps=1e-6, valid_cols=valid)
    d = cuda_device
    out = torch.full((rows, cols), 99, dtype=torch.int8, device=d)
    rs = torch.full((rows,), float("nan"), device=d)
    ops.rot_q8(
        x.to(d), gamma.to(d) if norm else None, beta.to(d) if norm else None, out, rs, block=block, eps=1e-6,
        valid_cols=valid,
    )
    torch.cuda.synchronize()
    got_q, got_s = out.cpu(), rs.cpu()
    torch.testing.assert_close(got_s, ref_s, rtol=2e-5, atol=0)
    diff = (got_q.int() - ref_q.int()).abs()
    # FWHT add order and rsqrt differ from the oracle's f64 matmul: codes may move by one step at
    # rounding ties, nothing more.
    assert diff.max().item() <= 1
    assert diff.float().mean().item() < 1e-3
    if valid < cols:
        # padded columns are zero before rotation: the codes still carry the rotated valid part
        assert got_q.shape == (rows, cols)


def test_rot_q8_reference_entry_points(cuda_device, no_device_error):
    """ff_rot_q8_1024 / ff_rot_q8_h128 keep the reference's semantics (eps 1e-5, no-norm H128)."""
    from foidfinder_b200 import ops

    d = cuda_device
    x = _activations(300, 1024, 1)
    gamma, beta = torch.ones(1024), torch.zeros(1024)
    out, rs = torch.empty(300, 1024, dtype=torch.int8, device=d), torch.empty(300, device=d)
    ops.rot_q8_1024(x.to(d), gamma.to(d), beta.to(d), out, rs)
    ref_q, ref_s = Q.rot_q8(x, gamma, beta, block=1024, eps=1e-5)
    torch.cuda.synchronize()
    assert (out.cpu().int() - ref_q.int()).abs().max() <= 1
    torch.testing.assert_close(rs.cpu(), ref_s, rtol=2e-5, atol=0)
    h = _activations(300, 2816, 2)
    out2, rs2 = torch.empty(300, 2816, dtype=torch.int8, device=d), torch.empty(300, device=d)
    ops.rot_q8_h128(h.to(d), out2, rs2)
    ref_q2, ref_s2 = Q.rot_q8(h, None, None, block=128)
    torch.cuda.synchronize()
    assert (out2.cpu().int() - ref_q2.int()).abs().max() <= 1
    torch.testing.assert_close(rs2.cpu(), ref_s2, rtol=2e-5, atol=0)


def _ref_attention(qkv, seqs, T, heads, scale, rope=None):
    q, k, v = qkv.float().view(seqs, T, 3, heads, 64).permute(2, 0, 3, 1, 4)
    if rope is not None:
        cos, sin = rope

        def rot(t):
            t2 = t.reshape(*t.shape[:-1], 32, 2)
            x0, x1 = t2[..., 0], t2[..., 1]
            return torch.stack([x0 * cos - x1 * sin, x0 * sin + x1 * cos], -1).reshape(t.shape)

        q, k = rot(q.half().float()).half().float(), rot(k.half().float()).half().float()
    o = torch.softmax((q @ k.transpose(-1, -2)) * scale, -1) @ v
    return o.transpose(1, 2).reshape(seqs * T, heads * 64)


@pytest.mark.parametrize(("seqs", "T", "heads", "rope"), [(1, 1025, 16, False), (2, 1025, 16, True), (3, 65, 12, False),
                                                          (1, 1, 16, False), (2, 577, 16, True), (1, 128, 4, False),
                                                          # tensor-core path: masked ragged query tile (577),
                                                          # CUDA-core tail rows (259: 3 rows; 1540: 4 rows and
                                                          # more keys than one pass of the tail warps)
                                                          (2, 577, 16, False), (2, 259, 8, False), (1, 1540, 4, False),
                                                          # the keys of the ragged last key tile (and the
                                                          # CUDA-core tail rows) hold the row maximum by far
                                                          (2, 1025, 16, "dominant"), (1, 1540, 4, "dominant"),
                                                          # the running maximum grows past the rescale
                                                          # threshold in the second half of the first key
                                                          # tile (its first half's P is recomputed), in the
                                                          # second half of a later tile (O rescaled and the
                                                          # first half recomputed), in the first half of a
                                                          # later tile, and steadily over all tiles
                                                          (2, 1025, 16, ("dominant", 64, 128)),
                                                          (1, 1025, 16, ("dominant", 320, 384)),
                                                          (1, 1025, 16, ("dominant", 512, 560)),
                                                          (2, 1025, 8, "ramp"),
                                                          # 512 pairs of query tiles, 3.5 rounds over the
                                                          # SMs, tail rows on the items' own warps (the cases
                                                          # above with fewer items put each query tile in
                                                          # an item of its own and the tail rows in CTAs of
                                                          # their own)
                                                          (8, 1025, 16, False)])
def test_attention_matches_oracle(cuda_device, no_device_error, seqs, T, heads, rope):
    from foidfinder_b200 import ops

    g = torch.Generator().manual_seed(seqs * 1000 + T)
    qkv = torch.randn(seqs * T, 3 * heads * 64, generator=g).half()
    if rope == "dominant" or isinstance(rope, tuple):
        k0, k1 = (T - T % 128, T) if rope == "dominant" else rope[1:]
        rope = False
        x = qkv.view(seqs, T, 3, heads, 64)
        x[:, :, 0] = x[:, :, 0].abs()  # q >= 0
        x[:, k0:k1, 1] = 0.6 * (1 + torch.rand(seqs, k1 - k0, heads, 64, generator=g)).half()  # q k ~ 60
    elif rope == "ramp":
        rope = False
        x = qkv.view(seqs, T, 3, heads, 64)
        x[:, :, 0] = x[:, :, 0].abs()
        ramp = torch.linspace(0.0, 1.2, T).view(1, T, 1, 1)  # q k grows from ~0 to ~70 over the keys
        x[:, :, 1] = (ramp * (1 + torch.rand(seqs, T, heads, 64, generator=g))).half()
    scale = 1.0 / math.sqrt(64)
    tables = None
    if rope:
        grid = int(round(math.sqrt(T - 1)))
        cos, sin = E.rope_tables(grid, 16)
        tables = (cos[:T], sin[:T])
    ref = _ref_attention(qkv, seqs, T, heads, scale, tables)
    if rope:  # q and k arrive rotated, as the QKV GEMM epilogue leaves them
        x = qkv.float().view(seqs, T, 3, heads, 32, 2)
        cos, sin = (t[:, None, :] for t in tables)
        for s in (0, 1):
            x0, x1 = x[:, :, s, ..., 0].clone(), x[:, :, s, ..., 1].clone()
            x[:, :, s, ..., 0], x[:, :, s, ..., 1] = x0 * cos - x1 * sin, x0 * sin + x1 * cos
        qkv = x.reshape(seqs * T, -1).half()
    d = cuda_device
    out = torch.full((seqs * T, heads * 64), float("nan"), dtype=torch.float16, device=d)
    ops.attention(qkv.to(d), out, T, heads, scale=scale)
    torch.cuda.synchronize()
    torch.testing.assert_close(out.float().cpu(), ref, atol=4e-3, rtol=1e-2)


@pytest.mark.parametrize(("T", "heads", "seqs"), [(1025, 16, 10), (1540, 4, 8)])
def test_attention_tail_rows_batch_invariant(cuda_device, no_device_error, T, heads, seqs):
    """A sequence alone (at most one work item per CTA: the tail rows' burst schedule) and the same
    sequence among others (more items than CTAs: the steady schedule) give the same bits."""
    from foidfinder_b200 import ops

    g = torch.Generator().manual_seed(T + heads)
    qkv = torch.randn(seqs * T, 3 * heads * 64, generator=g).half().to(cuda_device)
    many = torch.empty(seqs * T, heads * 64, dtype=torch.float16, device=cuda_device)
    one = torch.empty(T, heads * 64, dtype=torch.float16, device=cuda_device)
    ops.attention(qkv, many, T, heads, scale=0.125)
    ops.attention(qkv[:T].contiguous(), one, T, heads, scale=0.125)
    torch.cuda.synchronize()
    assert torch.equal(one, many[:T])


def test_attention_rejects_rope_tables(cuda_device):
    """RoPE belongs to the QKV GEMM epilogue (as in the reference); the attention op refuses tables."""
    from foidfinder_b200 import ops

    d = cuda_device
    qkv = torch.zeros(128, 3 * 64, dtype=torch.float16, device=d)
    out = torch.zeros(128, 64, dtype=torch.float16, device=d)
    cos = torch.ones(128, 32, device=d)
    with pytest.raises(RuntimeError, match="RoPE tables must be NULL"):
        ops.attention(qkv, out, 128, 1, rope=(cos, cos))


def test_layernorm_patchify_fill_cls(cuda_device, no_device_error):
    from foidfinder_b200 import ops

    d = cuda_device
    g = torch.Generator().manual_seed(3)
    B, S, p = 3, 448, 14
    img = torch.randint(0, 256, (B, S, S, 3), generator=g, dtype=torch.uint8)
    mean, std = (0.485, 0.456, 0.406), (0.229, 0.224, 0.225)
    out = torch.full((B * 1024, 640), float("nan"), dtype=torch.float16, device=d)
    ops.patchify(img.to(d), p, mean, std, out)
    ref = E.patchify(img, p, mean, std).reshape(B * 1024, 588)
    torch.cuda.synchronize()
    got = out.cpu()
    assert torch.all(got[:, 588:] == 0)
    torch.testing.assert_close(got[:, :588].float(), ref.half().float(), atol=0, rtol=1e-3)

    T, D = 1025, 1024
    x = torch.randn(B * T, D, generator=g).half()
    cls = torch.randn(D, generator=g).half()
    xd = x.to(d)
    ops.fill_cls(cls.to(d), xd, B, T)
    x[0::T] = cls
    gam, bet = 1 + 0.1 * torch.randn(D, generator=g), 0.1 * torch.randn(D, generator=g)
    ln = torch.empty(B, D, dtype=torch.float16, device=d)
    ops.layernorm(xd, T * D, B, D, gam.to(d), bet.to(d), 1e-6, ln)
    torch.cuda.synchronize()
    assert torch.equal(xd.cpu(), x)
    torch.testing.assert_close(ln.cpu().float(), Q.layer_norm(x[0::T], gam, bet, 1e-6).half().float(), atol=2e-3, rtol=2e-3)


@pytest.mark.parametrize(("B", "n", "k"), [(1, 30877, 50), (5, 30877, 50), (3, 98782 // 4, 64), (2, 98782, 50), (2, 100, 1), (4, 64, 64)])
def test_topk_exact(cuda_device, no_device_error, B, n, k):
    from foidfinder_b200 import ops

    g = torch.Generator().manual_seed(B * n + k)
    logits = torch.randn(B, n, generator=g)
    logits[:, 10:20] = 2.5  # a block of exact ties
    logits[0, -1] = float("-inf")
    d = cuda_device
    idx = torch.full((B, k), -1, dtype=torch.int32, device=d)
    val = torch.empty(B, k, device=d)
    ops.topk(logits.to(d), k, idx, val)
    torch.cuda.synchronize()
    # reference order: value descending, index ascending among equals
    order = sorted(range(n), key=lambda j: (-logits[0, j].item(), j))[:k] if B == 1 else None
    for b in range(B):
        keys = sorted(range(n), key=lambda j, b=b: (-logits[b, j].item(), j))[:k]
        assert idx[b].cpu().tolist() == keys
        torch.testing.assert_close(val[b].cpu(), logits[b, keys])
    del order
