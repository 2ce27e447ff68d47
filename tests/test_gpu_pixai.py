"""PixAI Tagger v1.0 (the reference's own `cuda` workload, foidfinder/backends/cuda/engine.py:65-184) on the
engine: every launch of the PixAI forward teacher-forced against the int8 oracle, then the whole engine
free-running against it (statistical bounds, as tests/test_gpu_engine.py explains)."""

import pytest
import torch

from oracle import pixai as PX

pytestmark = pytest.mark.gpu


def _codes_close(got, ref, what):
    diff = (got.cpu().int() - ref.int()).abs()
    assert diff.max().item() <= 1, f"{what}: code off by {diff.max().item()}"
    assert diff.float().mean().item() < 1e-3, f"{what}: {diff.float().mean().item():.2e} of codes differ"


def _fp16_close(got, ref, what, atol=2e-3, rtol=2e-3):
    torch.testing.assert_close(got.cpu().float(), ref.float(), atol=atol, rtol=rtol, msg=lambda m: f"{what}: {m}")


def _images(B, S, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, 256, (B, S, S, 3), generator=g, dtype=torch.uint8)


def _cfg(image=1008, depth=2, window=24, global_blocks=(1,), **kw):
    from foidfinder_b200.config import PIXAI_1008

    return PIXAI_1008.with_(name=f"pixai-{image}-{depth}", image_size=image, depth=depth, window=window,
                            global_blocks=global_blocks, **kw)


@pytest.mark.parametrize(("image", "window", "B"), [(1008, 24, 1), (336, 8, 2)])
def test_pixai_teacher_forced(cuda_device, no_device_error, image, window, B):
    """Each launch of PixAICuda._forward's sequence (window block 0, global block 1, pool head) on the
    oracle's input for that stage, compared with the oracle's output."""
    from foidfinder_b200 import ops
    from foidfinder_b200.weights import convert_pixai, pixai_random_raw

    d = cuda_device
    cfg = _cfg(image, 2, window, (1,))
    conv = convert_pixai(pixai_random_raw(cfg, seed=7, device="cuda"), cfg, "cpu")
    imgs = _images(B, image, 3)
    trace: list = []
    PX.forward_int8(conv, cfg, imgs, trace=trace)
    fin = trace[-1]
    W = {k: v.to(d) for k, v in conv.items()}
    L, D, H, eps = cfg.patches, cfg.dim, cfg.mlp_hidden_pad, cfg.ln_eps
    M = B * L

    patches = torch.empty(M, cfg.k_pad, dtype=torch.float16, device=d)
    ops.patchify_windowed(imgs.to(d), cfg.patch, cfg.mean, cfg.std, cfg.window, patches)
    x = torch.empty(M, D, dtype=torch.float16, device=d)
    padded = torch.zeros(M, cfg.k_pad, dtype=torch.float16, device=d)
    padded[:, : cfg.k_patch] = fin["patches"].to(d)
    ops.gemm_f16(padded, W["patch_w"], x, ops.EPI_STEM, pos_bias=W["pos_bias"], patches=L, tokens=L)
    torch.cuda.synchronize()
    _fp16_close(patches[:, : cfg.k_patch], fin["patches"], "windowed patchify", atol=0, rtol=1e-3)
    _fp16_close(x, fin["x_stem"], "stem")
    xs = fin["x_stem"].to(d).clone()
    ops.layernorm(xs, D, M, D, W["ln_pre.weight"], W["ln_pre.bias"], eps, xs)  # in place, as the engine runs it
    torch.cuda.synchronize()
    _fp16_close(xs, fin["x_pre"], "ln_pre")

    a = torch.empty(M, D, dtype=torch.int8, device=d)
    ah = torch.empty(M, H, dtype=torch.int8, device=d)
    rs = torch.empty(M, device=d)
    qkv = torch.empty(M, 3 * D, dtype=torch.float16, device=d)
    o = torch.empty(M, D, dtype=torch.float16, device=d)
    h = torch.empty(M, H, dtype=torch.float16, device=d)
    for i, st in enumerate(trace[:-1]):
        p = f"blocks.{i}."
        glob = cfg.is_global(i)
        tag = f"block {i} ({'global' if glob else 'window'})"
        n = st["seq"]
        cos, sin = (W["rope_cos_global"], W["rope_sin_global"]) if glob else (W["rope_cos"], W["rope_sin"])
        ops.rot_q8(st["x_in"].to(d), W[p + "norm1.weight"], W[p + "norm1.bias"], a, rs, block=cfg.rot_block_dim, eps=eps)
        torch.cuda.synchronize()
        _codes_close(a, st["a8"], tag + " LN1+H+q8")
        torch.testing.assert_close(rs.cpu(), st["rs"], rtol=2e-5, atol=0)
        ops.gemm_s8(st["a8"].to(d), W[p + "qkv.qweight"], st["rs"].to(d), W[p + "qkv.wscale"], W[p + "qkv.bias"], qkv,
                    ops.EPI_QKV_ROPE, rope_cos=cos, rope_sin=sin, rope_cols=2 * D, tokens=n)
        ops.attention(st["qkv"].to(d), o, n, cfg.heads)
        torch.cuda.synchronize()
        _fp16_close(qkv, st["qkv"], tag + " qkv GEMM + RoPE")
        _fp16_close(o, st["o"], tag + " attention", rtol=1e-2)
        ops.rot_q8(st["o"].to(d), None, None, a, rs, block=cfg.rot_block_dim)
        torch.cuda.synchronize()
        _codes_close(a, st["a8o"], tag + " H+q8(o)")
        xr = st["x_in"].to(d).clone()
        ops.gemm_s8(st["a8o"].to(d), W[p + "proj.qweight"], st["rso"].to(d), W[p + "proj.wscale"], W[p + "proj.bias"],
                    xr, ops.EPI_RESIDUAL)
        ops.rot_q8(st["x_attn"].to(d), W[p + "norm2.weight"], W[p + "norm2.bias"], a, rs, block=cfg.rot_block_dim,
                   eps=eps)
        torch.cuda.synchronize()
        _fp16_close(xr, st["x_attn"], tag + " proj GEMM + residual")
        _codes_close(a, st["a8m"], tag + " LN2+H+q8")
        ops.gemm_s8(st["a8m"].to(d), W[p + "fc1.qweight"], st["rsm"].to(d), W[p + "fc1.wscale"], W[p + "fc1.bias"], h,
                    ops.EPI_GELU)
        ops.rot_q8_h128(st["h"].to(d), ah, rs)
        torch.cuda.synchronize()
        _fp16_close(h, st["h"], tag + " fc1 GEMM + GELU", atol=4e-3, rtol=4e-3)
        _codes_close(ah, st["a8h"], tag + " H128+q8 (4864 padded)")
        torch.testing.assert_close(rs.cpu(), st["rsh"], rtol=2e-5, atol=0)
        xr = st["x_attn"].to(d).clone()
        ops.gemm_s8(st["a8h"].to(d), W[p + "fc2.qweight"], st["rsh"].to(d), W[p + "fc2.wscale"], W[p + "fc2.bias"], xr,
                    ops.EPI_RESIDUAL)
        torch.cuda.synchronize()
        _fp16_close(xr, st["x_out"], tag + " fc2 GEMM + residual")

    xn = torch.empty(M, D, dtype=torch.float16, device=d)
    ops.layernorm_pos(fin["x_final"].to(d), W["pool.norm.weight"], W["pool.norm.bias"], eps, W["pool.pos"], xn)
    kv = torch.empty(M, 2 * D, dtype=torch.float16, device=d)
    ops.gemm_f16(fin["xn"].to(d), W["pool.kv.weight"], kv, ops.EPI_BIAS, bias=W["pool.kv.bias"])
    att = torch.empty(B, D, dtype=torch.float16, device=d)
    ops.pool_query_attention(W["pool.q"], fin["kv"].to(d), B, L, att)
    z = torch.empty(B, D, dtype=torch.float16, device=d)
    ops.gemm_f16(fin["att"].to(d), W["pool.proj.weight"], z, ops.EPI_BIAS, bias=W["pool.proj.bias"])
    logits = torch.empty(B, cfg.num_tags, device=d)
    ops.gemm_f16(fin["z"].to(d), W["head.weight"], logits, ops.EPI_LOGITS, bias=W["head.bias"], n_valid=cfg.num_tags)
    idx = torch.empty(B, cfg.topk, dtype=torch.int32, device=d)
    ops.topk(fin["logits"].to(d), cfg.topk, idx)
    torch.cuda.synchronize()
    _fp16_close(xn, fin["xn"], "pool LN + pos", atol=4e-3)
    _fp16_close(kv, fin["kv"], "pool kv GEMM")
    _fp16_close(att, fin["att"], "pool attention")
    _fp16_close(z, fin["z"], "pool proj GEMM")
    torch.testing.assert_close(logits.cpu(), fin["logits"], atol=1e-4, rtol=1e-4)
    ref_idx = torch.sort(fin["logits"], dim=1, descending=True, stable=True).indices[:, : cfg.topk]
    assert torch.equal(idx.cpu().long(), ref_idx)


@pytest.mark.parametrize(("image", "window", "depth", "B"), [(336, 8, 2, 3), (1008, 24, 2, 2)])
def test_pixai_engine_matches_int8_oracle(cuda_device, no_device_error, image, window, depth, B):
    from foidfinder_b200.engine import Engine
    from foidfinder_b200.weights import convert_pixai, pixai_random_raw

    from test_gpu_engine import _check_topk, _free_running_bounds

    cfg = _cfg(image, depth, window, (1,))
    raw = pixai_random_raw(cfg, seed=13, device="cuda")
    conv = convert_pixai(raw, cfg, "cpu")
    imgs = _images(B, image, 8)
    ref = PX.forward_int8(conv, cfg, imgs)
    eng = Engine(cfg, conv, device=0)
    assert eng.launches_per_forward == 3 + 9 * depth + 4 + 1 + 1
    logits, idx, val = eng.forward(imgs, graph=False)
    torch.cuda.synchronize()
    got = logits.cpu()
    assert torch.isfinite(got).all()
    _free_running_bounds(got, ref)
    _check_topk(idx.cpu(), ref, cfg.topk, slack=(got - ref).abs().max().item())
    torch.testing.assert_close(val.cpu(), torch.gather(got, 1, idx.cpu().long()))
    g1, i1, _ = eng.forward(imgs, graph=True)
    g2, _, _ = eng.forward(imgs, graph=True)
    torch.cuda.synchronize()
    assert torch.equal(g1.cpu(), got) and torch.equal(g2.cpu(), got)
    assert torch.equal(i1.cpu(), idx.cpu())
    # the f32 model of reference.py on the unquantised weights: int8 moves probabilities only slightly
    p32 = torch.sigmoid(PX.forward_fp32({k: v.cpu() for k, v in raw.items()}, cfg, imgs))
    assert (torch.sigmoid(got) - p32).abs().max().item() < 0.15
    eng.close()
