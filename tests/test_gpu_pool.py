"""Haruka tree attention pool head on the GPU (ff_tree_pool and the engine's tree head) against the
oracle (oracle/eva02.py:tree_pool, itself pinned to the model card's MHAttnPool by the golden vectors)."""

import pytest
import torch

from oracle import eva02 as E
from oracle import quant as Q

pytestmark = pytest.mark.gpu


def _cfg(**kw):
    from foidfinder_b200.config import EVA02_B

    return EVA02_B.with_(name="pool-test", depth=1, **kw)


@pytest.mark.parametrize(("image", "B"), [(448, 3), (112, 2)])
def test_tree_pool_matches_oracle(cuda_device, no_device_error, image, B):
    """Teacher-forced: the same fp16 backbone output into both; leaf features compared."""
    from foidfinder_b200 import ops
    from foidfinder_b200.weights import convert, random_raw

    cfg = _cfg(image_size=image)
    conv = convert(random_raw(cfg, seed=5), cfg)
    g = torch.Generator().manual_seed(17)
    x = (torch.randn(B * cfg.tokens, cfg.dim, generator=g) * 2.0 + 0.3).half()
    xf = Q.layer_norm(x.float(), conv["norm.weight"], conv["norm.bias"], cfg.ln_eps).half().float()
    ref = E.tree_pool(xf.view(B, cfg.tokens, cfg.dim), conv, cfg, half=True)
    d = cuda_device
    w = {k: v.to(d) for k, v in conv.items() if k.startswith("pool.") or k.startswith("norm.")}
    out = torch.full((B, cfg.head_in), float("nan"), dtype=torch.float16, device=d)
    ops.tree_pool(cfg, w, x.to(d), out)
    got = out.cpu().float()
    assert torch.isfinite(got).all()
    scale = ref.abs().max().item()
    assert scale > 1e-3
    err = (got - ref).abs()
    print(f"leaf features: max |ref| {scale:.3e}, max err {err.max().item():.3e}, mean err {err.mean().item():.3e}")
    # fp16 storage of the key/value projection differs by at most an ulp between f32 summation orders;
    # everything downstream is f32, so the features agree to a few fp16 ulps of their scale.
    assert err.max().item() <= 4e-3 * scale
    assert err.mean().item() <= 5e-4 * scale


def test_tree_pool_rejects_cls_config(cuda_device):
    from foidfinder_b200 import ops
    from foidfinder_b200.config import EVA02_L

    with pytest.raises(RuntimeError, match="no tree head"):
        ops.tree_pool(EVA02_L, {}, torch.zeros(1025, 1024, dtype=torch.float16, device=cuda_device),
                      torch.zeros(1, 1024, dtype=torch.float16, device=cuda_device))


@pytest.mark.parametrize(("image", "depth", "B"), [(112, 2, 3), (448, 2, 2)])
def test_engine_tree_head_matches_int8_oracle(cuda_device, no_device_error, image, depth, B):
    from foidfinder_b200.engine import Engine
    from foidfinder_b200.weights import convert, random_raw

    from test_gpu_engine import _check_topk, _free_running_bounds, _images

    cfg = _cfg(image_size=image).with_(depth=depth)
    raw = random_raw(cfg, seed=23)
    conv = convert(raw, cfg)
    imgs = _images(B, image, 29)
    ref = E.forward_int8(conv, cfg, imgs)
    eng = Engine(cfg, conv, device=0)
    assert eng.launches_per_forward == 3 + 9 * depth + 7 + 1 + 1
    logits, idx, val = eng.forward(imgs, graph=False)
    torch.cuda.synchronize()
    got = logits.cpu()
    assert torch.isfinite(got).all()
    _free_running_bounds(got, ref)
    _check_topk(idx.cpu(), ref, cfg.topk, slack=(got - ref).abs().max().item())
    g1, i1, _ = eng.forward(imgs, graph=True)
    torch.cuda.synchronize()
    assert torch.equal(g1.cpu(), got) and torch.equal(i1.cpu(), idx.cpu())
    # the unquantised fp32 model with the same weights
    p32 = torch.sigmoid(E.forward_fp32(raw, cfg, imgs))
    assert (torch.sigmoid(got) - p32).abs().max().item() < 0.15
    eng.close()
