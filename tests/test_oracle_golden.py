"""Pins the oracle (and the host-side weight preparation) to vectors produced by the reference's own
Python functions (tests/golden/make_golden.py). CPU only."""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT / "tests" / "golden"))

import make_golden  # noqa: E402

from foidfinder_b200 import weights as W  # noqa: E402
from oracle import eva02 as E  # noqa: E402
from oracle import fold as F  # noqa: E402
from oracle import pixai as P  # noqa: E402
from oracle import quant as Q  # noqa: E402

ROT_BLOCK = {"attn.qkv": 1024, "attn.proj": 1024, "mlp.fc1": 1024, "mlp.fc2": 128}


@pytest.fixture(scope="module")
def gold():
    with np.load(ROOT / "tests" / "golden" / "reference_vectors.npz") as z:
        return {k: z[k] for k in z.files}


@pytest.fixture(scope="module")
def inp():
    return make_golden.inputs()


@pytest.mark.parametrize("n", [128, 1024])
def test_hadamard(gold, n):
    sign = np.unpackbits(gold[f"hadamard{n}_sign"])[: n * n].reshape(n, n).astype(bool)
    h = Q.hadamard(n).numpy()
    assert np.array_equal(h > 0, sign)
    assert np.float32(np.abs(h).max()) == gold[f"hadamard{n}_abs"]
    # The weight converter rotates by the same float32 matrix.
    assert np.array_equal(W.hadamard(n).numpy(), h)
    assert np.array_equal(W.rotate_rows(torch.eye(n), n).numpy(), h)


@pytest.mark.parametrize("quant", [Q.quantize_rows_int8, W.quantize_rows_int8])
def test_quantize_rows_int8(gold, inp, quant):
    q, s = quant(torch.from_numpy(inp["quant_in"]))
    assert np.array_equal(q.numpy(), gold["quant_q"])
    assert np.array_equal(s.numpy(), gold["quant_scale"])


@pytest.mark.parametrize("name", list(make_golden.CONV_SHAPES))
def test_convert_checkpoint(gold, inp, name):
    """Rotated per-channel int8 weights are the reference's convert_checkpoint output bit for bit (codes and
    scales), both in the oracle and in the weight converter: the same float32 matmul by blockdiag(H)."""
    w = torch.from_numpy(inp[f"conv_{name}_w"])
    ref_q, ref_s = gold[f"conv_{name}_qweight"], gold[f"conv_{name}_wscale"]
    for rotated in (Q.rotate_weight(w, ROT_BLOCK[name]), W.rotate_rows(w, ROT_BLOCK[name])):
        q, s = W.quantize_rows_int8(rotated)
        assert np.array_equal(q.numpy(), ref_q)
        assert np.array_equal(s.numpy(), ref_s)


def test_pixai_convert_checkpoint_matches_reference(gold, inp):
    """The one-block checkpoint make_golden.py ran through the reference's convert_checkpoint: the
    converter's own copy of that step (`pixai_convert_checkpoint`) writes the same tensors under the same
    names, so a checkpoint written by `foidfinder convert` and one converted here are interchangeable."""
    raw = {}
    for name, shape in make_golden.CONV_SHAPES.items():
        raw[f"blocks.0.{name}.weight"] = torch.from_numpy(inp[f"conv_{name}_w"])
        raw[f"blocks.0.{name}.bias"] = torch.zeros(shape[0])
    from foidfinder_b200.config import PIXAI_1008

    conv = W.pixai_convert_checkpoint(raw, PIXAI_1008.with_(depth=1))
    assert W.is_pixai_int8(conv)
    for name in make_golden.CONV_SHAPES:
        assert conv[f"blocks.0.{name}.qweight"].dtype == torch.int8
        assert np.array_equal(conv[f"blocks.0.{name}.qweight"].numpy(), gold[f"conv_{name}_qweight"])
        assert np.array_equal(conv[f"blocks.0.{name}.wscale"].numpy(), gold[f"conv_{name}_wscale"])
        assert f"blocks.0.{name}.weight" not in conv


def test_pixai_engine_weights_from_reference_int8(inp):
    """convert_pixai on the official fp32 names and on the reference's int8 checkpoint of the same weights
    gives identical engine weights: codes unchanged, the 1/8 attention scale folded into the q rows'
    scale and bias (exact, a power of two), the hidden padded with zero rows/columns."""
    from foidfinder_b200.config import PIXAI_1008

    cfg = PIXAI_1008.with_(name="pixai-tiny", image_size=336, depth=2, window=8, global_blocks=(1,), dim=128,
                           heads=2, mlp_hidden=384, num_tags=300, rot_block_dim=128)
    raw = W.pixai_random_raw(cfg, seed=5, pre_grid=12)
    ref_int8 = W.pixai_convert_checkpoint(raw, cfg)
    a, b = W.convert_pixai(raw, cfg), W.convert_pixai(ref_int8, cfg)
    assert a.keys() == b.keys()
    for k in a:
        assert torch.equal(a[k], b[k]), k
    D, H, Hp = cfg.dim, cfg.mlp_hidden, cfg.mlp_hidden_pad
    for i in range(cfg.depth):
        p = f"blocks.{i}."
        assert torch.equal(a[p + "qkv.qweight"], ref_int8[p + "attn.qkv.qweight"])
        assert torch.equal(a[p + "qkv.wscale"][:D], ref_int8[p + "attn.qkv.wscale"][:D] * 0.125)
        assert torch.equal(a[p + "qkv.wscale"][D:], ref_int8[p + "attn.qkv.wscale"][D:])
        assert torch.equal(a[p + "fc1.qweight"][:H], ref_int8[p + "mlp.fc1.qweight"])
        assert not a[p + "fc1.qweight"][H:].any() and not a[p + "fc1.bias"][H:].any()
        assert torch.equal(a[p + "fc2.qweight"][:, :H], ref_int8[p + "mlp.fc2.qweight"])
        assert a[p + "fc2.qweight"].shape == (D, Hp) and not a[p + "fc2.qweight"][:, H:].any()


def test_pixai_axial_rope(gold, inp):
    cos, sin = P.axial_rope(24, 1.0)
    out = P.apply_rope(torch.from_numpy(inp["rope_in"]), cos, sin).numpy()
    np.testing.assert_allclose(out, gold["rope_out"], rtol=0, atol=1e-6)
    # The engine's epilogue convention (pairs 2i, 2i+1 of each 64-wide head) gives the same rotation.
    x = torch.from_numpy(inp["rope_in"]).reshape(-1, 64)
    pairs = Q.apply_rope_pairs(x, cos, sin, torch.arange(x.shape[0]), 64)
    np.testing.assert_allclose(pairs.numpy().reshape(out.shape), gold["rope_out"], rtol=0, atol=1e-6)


@pytest.mark.parametrize("tables", [E.rope_tables, W.rope_tables])
def test_eva02_rope_tables(gold, tables):
    assert bool(gold["eva_rope_pairs_equal"])  # the reference's tables repeat each angle over a pair
    cos, sin = tables(32, 16, 64)
    rows = make_golden.EVA_ROPE_ROWS
    np.testing.assert_allclose(cos.numpy()[rows], gold["eva_rope_cos_even"], rtol=0, atol=2e-6)
    np.testing.assert_allclose(sin.numpy()[rows], gold["eva_rope_sin_even"], rtol=0, atol=2e-6)
    csum, ssum, n = gold["eva_rope_checksum"]
    assert cos.shape[0] == int(n)
    # Full tables repeat each pair's value twice.
    assert abs(2 * cos.double().sum().item() - csum) < 1e-2
    assert abs(2 * sin.double().sum().item() - ssum) < 1e-2


def test_haruka_fold(gold):
    sd = make_golden.fold_inputs()
    out = F.fold(sd, dim=64, heads=2, patch=14, depth=1, pool_heads=make_golden.TREE["pool_heads"])
    for k in make_golden.FOLD_KEYS:
        np.testing.assert_allclose(out[k], gold["fold_out_" + k.replace(".", "_")], rtol=1e-5, atol=1e-7, err_msg=k)


def test_tree_pool_matches_model_card(gold):
    """The oracle's tree pool on the folded weights reproduces the model card's MHAttnPool (unfolded
    weights, f32, its LayerNorms at torch's default eps 1e-5)."""
    from foidfinder_b200.config import EVA02_B

    T = make_golden.TREE
    cfg = EVA02_B.with_(dim=T["dim"], pool_heads=T["pool_heads"], coarse_queries=T["coarse"],
                        leaf_queries=T["leaves"], leaf_dim=T["leaf_dim"])
    w = {k: torch.from_numpy(np.asarray(v)) for k, v in
         F.fold(make_golden.fold_inputs(), dim=T["dim"], heads=2, patch=14, depth=1, pool_heads=T["pool_heads"]).items()}
    x = torch.from_numpy(make_golden.tree_input())
    got = E.tree_pool(x, w, cfg, half=False, eps=1e-5).numpy()
    assert np.abs(gold["tree_leaf"]).max() > 0.05  # the pool is not degenerate at these scales
    np.testing.assert_allclose(got, gold["tree_leaf"], rtol=1e-4, atol=1e-5)
    # At the backbone's eps (what the MLX port and the engine use) the features move by far less than
    # the int8 noise.
    got6 = E.tree_pool(x, w, cfg, half=False).numpy()
    assert np.abs(got6 - gold["tree_leaf"]).max() < 1e-3


def test_fold_matches_engine_patch_convention(gold):
    """The folded patch embedding applied to raw pixels equals the unfolded one applied to normalised
    pixels — the equivalence the engine's stem (mean/std applied on the fly) relies on."""
    sd = make_golden.fold_inputs()
    rng = np.random.default_rng(3)
    px = rng.integers(0, 256, size=(4, 14, 14, 3)).astype(np.float32)
    w = sd["backbone.patch_embed.proj.weight"].transpose(0, 2, 3, 1).reshape(64, -1)
    b = sd["backbone.patch_embed.proj.bias"]
    norm = ((px / 255.0 - F.IMAGENET_MEAN) / F.IMAGENET_STD).reshape(4, -1)
    unfolded = norm @ w.T + b + sd["backbone.pos_embed"][0, 1:]
    folded = px.reshape(4, -1) @ gold["fold_out_patch_w"].T + gold["fold_out_patch_b"]
    np.testing.assert_allclose(folded, unfolded, rtol=1e-4, atol=1e-5)


# ---------------------------------------------------------------- PixAI Tagger v1.0


def _pixai_cfg():
    from foidfinder_b200.config import PIXAI_1008

    px = make_golden.PIXAI
    return PIXAI_1008.with_(name="pixai-golden", image_size=px["S"], dim=px["C"], heads=px["H"], depth=px["DEPTH"],
                            mlp_hidden=px["hidden"], num_tags=px["tags"], window=px["WIN"],
                            global_blocks=tuple(px["GLOBAL"]), rot_block_dim=px["C"])


def _pixai_raw():
    return {k: torch.from_numpy(v) for k, v in make_golden.pixai_checkpoint().items()}


def test_pixai_window_order_matches_reference_layout():
    """The window order of reference.py:21-24 (windows row-major, patches row-major inside)."""
    perm = P.window_perm(6, 3)
    assert perm[:9].tolist() == [0, 1, 2, 6, 7, 8, 12, 13, 14]
    assert perm[9:12].tolist() == [3, 4, 5]
    assert torch.equal(W.window_order(72, 24), P.window_perm(72, 24))
    assert torch.equal(torch.sort(P.window_perm(72, 24)).values, torch.arange(5184))


def test_pixai_forward_fp32_matches_reference(gold):
    """The oracle's f32 PixAI forward reproduces PixAITorch (reference.py:109-140) on the same checkpoint."""
    cfg = _pixai_cfg()
    imgs = torch.from_numpy(make_golden.pixai_images())
    got = P.forward_fp32(_pixai_raw(), cfg, imgs)
    np.testing.assert_allclose(got.numpy(), gold["pixai_logits"], atol=2e-5, rtol=1e-4)


def test_pixai_pool_head_matches_reference(gold):
    cfg = _pixai_cfg()
    got = P.pool_head_fp32(torch.from_numpy(make_golden.pixai_pool_input()), _pixai_raw(), cfg)
    np.testing.assert_allclose(got.numpy(), gold["pixai_pool_logits"], atol=2e-5, rtol=1e-4)


def test_pixai_int8_pipeline_tracks_fp32(gold):
    """The converted checkpoint through the int8 oracle (the engine's arithmetic) stays within the int8
    pipeline's error of the reference's f32 logits and keeps their top tags."""
    cfg = _pixai_cfg()
    conv = W.convert_pixai(_pixai_raw(), cfg)
    got = P.forward_int8(conv, cfg, torch.from_numpy(make_golden.pixai_images()))
    ref = torch.from_numpy(gold["pixai_logits"])
    err = (got - ref).abs().max().item()
    assert err < 0.05 * ref.abs().max().item(), err
    top = lambda t: set(torch.topk(t, 5).indices.tolist())  # noqa: E731
    for b in range(ref.shape[0]):
        assert len(top(got[b]) & top(ref[b])) >= 4
