"""Teacher-forced parity of the whole forward: every kernel launch of the engine's sequence, for every
block, is run on the oracle's input for that stage and compared with the oracle's output.

Why teacher forcing: the int8 pipeline is chaotic with respect to ulp-level differences — a code that
sits on a rounding tie flips, the flip moves the fp16 residual stream, LayerNorm statistics shift, more
codes flip downstream. Changing nothing but the rounding of the oracle's own FWHT (f64 -> f32 matmul)
moves the logits of the 2-block test model by up to 0.055 (mean 0.0085). A free-running GPU-vs-CPU
comparison can therefore only be statistical (tests/test_gpu_engine.py); this test pins every kernel to
the oracle's function on identical inputs: codes within one step at ties, scales to 2e-5, fp16
activations to 1-2 ulps, logits to 1e-4.
"""

import pytest
import torch

from oracle import eva02 as E

pytestmark = pytest.mark.gpu


def _codes_close(got, ref, what):
    diff = (got.cpu().int() - ref.int()).abs()
    assert diff.max().item() <= 1, f"{what}: code off by {diff.max().item()}"
    assert diff.float().mean().item() < 1e-3, f"{what}: {diff.float().mean().item():.2e} of codes differ"


def _fp16_close(got, ref, what, atol=2e-3, rtol=2e-3):
    torch.testing.assert_close(got.cpu().float(), ref.float(), atol=atol, rtol=rtol, msg=lambda m: f"{what}: {m}")


def _teacher_forced(cfg, conv, imgs, d):
    from foidfinder_b200 import ops

    trace: list = []
    E.forward_int8(conv, cfg, imgs, trace=trace)
    fin = trace[-1]
    W = {k: v.to(d) for k, v in conv.items()}
    B, T, D, Hp = imgs.shape[0], cfg.tokens, cfg.dim, cfg.mlp_hidden_pad
    M = B * T
    eps = cfg.ln_eps

    patches = torch.empty(B * cfg.patches, cfg.k_pad, dtype=torch.float16, device=d)
    ops.patchify(imgs.to(d), cfg.patch, cfg.mean, cfg.std, patches)
    torch.cuda.synchronize()
    _fp16_close(patches[:, : cfg.k_patch], fin["patches"].reshape(B * cfg.patches, -1), "patchify", atol=0, rtol=1e-3)
    x = torch.empty(M, D, dtype=torch.float16, device=d)
    padded = torch.zeros(B * cfg.patches, cfg.k_pad, dtype=torch.float16, device=d)
    padded[:, : cfg.k_patch] = fin["patches"].reshape(B * cfg.patches, -1).to(d)
    ops.gemm_f16(padded, W["patch_w"], x, ops.EPI_STEM, pos_bias=W["pos_bias"], patches=cfg.patches, tokens=T)
    ops.fill_cls(W["cls_row"], x, B, T)
    torch.cuda.synchronize()
    _fp16_close(x, fin["x_stem"], "stem")

    a = torch.empty(M, D, dtype=torch.int8, device=d)
    ah = torch.empty(M, Hp, dtype=torch.int8, device=d)
    rs = torch.empty(M, device=d)
    qkv = torch.empty(M, 3 * D, dtype=torch.float16, device=d)
    o = torch.empty(M, D, dtype=torch.float16, device=d)
    h = torch.empty(M, Hp, dtype=torch.float16, device=d)
    for i, st in enumerate(trace[:-1]):
        p = f"blocks.{i}."
        tag = f"block {i}"
        ops.rot_q8(st["x_in"].to(d), W[p + "norm1.weight"], W[p + "norm1.bias"], a, rs, block=cfg.rot_block_dim, eps=eps)
        torch.cuda.synchronize()
        _codes_close(a, st["a8"], tag + " LN1+H+q8")
        torch.testing.assert_close(rs.cpu(), st["rs"], rtol=2e-5, atol=0)
        ops.gemm_s8(st["a8"].to(d), W[p + "qkv.qweight"], st["rs"].to(d), W[p + "qkv.wscale"], W[p + "qkv.bias"], qkv,
                    ops.EPI_QKV_ROPE, rope_cos=W["rope_cos"], rope_sin=W["rope_sin"], rope_cols=2 * D, tokens=T)
        ops.attention(st["qkv"].to(d), o, T, cfg.heads)
        torch.cuda.synchronize()
        _fp16_close(qkv, st["qkv"], tag + " qkv GEMM")
        _fp16_close(o, st["o"], tag + " attention", rtol=1e-2)
        ops.rot_q8(st["o"].to(d), None, None, a, rs, block=cfg.rot_block_dim)
        torch.cuda.synchronize()
        _codes_close(a, st["a8o"], tag + " H+q8(o)")
        xr = st["x_in"].to(d).clone()
        ops.gemm_s8(st["a8o"].to(d), W[p + "proj.qweight"], st["rso"].to(d), W[p + "proj.wscale"], W[p + "proj.bias"], xr,
                    ops.EPI_RESIDUAL)
        ops.rot_q8(st["x_attn"].to(d), W[p + "norm2.weight"], W[p + "norm2.bias"], a, rs, block=cfg.rot_block_dim, eps=eps)
        torch.cuda.synchronize()
        _fp16_close(xr, st["x_attn"], tag + " proj GEMM + residual")
        _codes_close(a, st["a8m"], tag + " LN2+H+q8")
        ops.gemm_s8(st["a8m"].to(d), W[p + "fc1.qweight"], st["rsm"].to(d), W[p + "fc1.wscale"], W[p + "fc1.bias"], h,
                    ops.EPI_SWIGLU)
        ops.rot_q8(st["h"].to(d), W[p + "mlp_norm.weight"], W[p + "mlp_norm.bias"], ah, rs, block=cfg.rot_block_hidden,
                   eps=eps, valid_cols=cfg.mlp_hidden)
        torch.cuda.synchronize()
        _fp16_close(h, st["h"], tag + " gate|up GEMM + SwiGLU")
        _codes_close(ah, st["a8h"], tag + " mlp LN+H128+q8")
        torch.testing.assert_close(rs.cpu(), st["rsh"], rtol=2e-5, atol=0)
        xr = st["x_attn"].to(d).clone()
        ops.gemm_s8(st["a8h"].to(d), W[p + "fc2.qweight"], st["rsh"].to(d), W[p + "fc2.wscale"], W[p + "fc2.bias"], xr,
                    ops.EPI_RESIDUAL)
        torch.cuda.synchronize()
        _fp16_close(xr, st["x_out"], tag + " down GEMM + residual")

    cls = torch.empty(B, cfg.head_in, dtype=torch.float16, device=d)
    if cfg.head == "tree":
        ops.tree_pool(cfg, W, fin["x_final"].to(d), cls)
        torch.cuda.synchronize()
        err = (cls.cpu().float() - fin["cls"].float()).abs().max().item()
        assert err <= 4e-3 * fin["cls"].float().abs().max().item(), f"tree pool: max err {err:.3e}"
    else:
        ops.layernorm(fin["x_final"].to(d), T * D, B, D, W["norm.weight"], W["norm.bias"], eps, cls)
        torch.cuda.synchronize()
        _fp16_close(cls, fin["cls"], "final LayerNorm")
    logits = torch.empty(B, cfg.num_tags, device=d)
    ops.gemm_f16(fin["cls"].to(d), W["head.weight"], logits, ops.EPI_LOGITS, bias=W["head.bias"], n_valid=cfg.num_tags)
    idx = torch.empty(B, cfg.topk, dtype=torch.int32, device=d)
    ops.topk(fin["logits"].to(d), cfg.topk, idx)
    torch.cuda.synchronize()
    torch.testing.assert_close(logits.cpu(), fin["logits"], atol=1e-4, rtol=1e-4)
    ref_idx = torch.sort(fin["logits"], dim=1, descending=True, stable=True).indices[:, : cfg.topk]
    assert torch.equal(idx.cpu().long(), ref_idx)


def test_teacher_forced_448_two_blocks(cuda_device, no_device_error):
    from foidfinder_b200.config import EVA02_L
    from foidfinder_b200.weights import convert, random_raw

    cfg = EVA02_L.with_(name="tf-448-2", depth=2)
    conv = convert(random_raw(cfg, seed=4), cfg)
    imgs = torch.randint(0, 256, (2, 448, 448, 3), generator=torch.Generator().manual_seed(1), dtype=torch.uint8)
    _teacher_forced(cfg, conv, imgs, cuda_device)


def test_teacher_forced_full_eva02_l(cuda_device, no_device_error):
    """Every launch of the BASELINE config-0 forward (24 blocks, 30,877 tags) at batch 1."""
    from foidfinder_b200.config import EVA02_L
    from foidfinder_b200.weights import convert, random_raw

    conv = convert(random_raw(EVA02_L, seed=0, device="cuda"), EVA02_L, "cpu")
    imgs = torch.randint(0, 256, (1, 448, 448, 3), generator=torch.Generator().manual_seed(0), dtype=torch.uint8)
    _teacher_forced(EVA02_L, conv, imgs, cuda_device)


def test_teacher_forced_eva02_b(cuda_device, no_device_error):
    """The Haruka shape (dim 768, H256 rotation, hidden 2048, ImageNet normalisation, tree pool head)."""
    from foidfinder_b200.config import EVA02_B
    from foidfinder_b200.weights import convert, random_raw

    cfg = EVA02_B.with_(name="tf-b-2", depth=2)
    conv = convert(random_raw(cfg, seed=6), cfg)
    imgs = torch.randint(0, 256, (2, 448, 448, 3), generator=torch.Generator().manual_seed(2), dtype=torch.uint8)
    _teacher_forced(cfg, conv, imgs, cuda_device)
