"""CUDABackend's model-directory handling on the CPU: config.json decides the model as the reference's
CUDABackend does (foidfinder/backends/cuda/__init__.py:21-22), and a PixAI directory holding the official
fp32 checkpoint or the reference's `foidfinder convert` int8 output (engine.py:66-72) gives the same engine
weights."""

import json

import pytest
import torch

from foidfinder_b200 import backend as BK
from foidfinder_b200 import weights as W
from foidfinder_b200.config import EVA02_B, PIXAI_1008


def _tiny_pixai():
    return PIXAI_1008.with_(name="pixai-tiny", image_size=336, depth=2, window=8, global_blocks=(1,), dim=128,
                            heads=2, mlp_hidden=384, num_tags=300, rot_block_dim=128)


def _write(dirpath, tensors, config, metadata=None):
    from safetensors.torch import save_file

    dirpath.mkdir(parents=True, exist_ok=True)
    save_file({k: v.contiguous() for k, v in tensors.items()}, str(dirpath / "model.safetensors"), metadata)
    (dirpath / "config.json").write_text(json.dumps(config))


def test_pixai_directory_fp32_and_reference_int8(tmp_path):
    cfg = _tiny_pixai()
    raw = W.pixai_random_raw(cfg, seed=2, pre_grid=12)
    ref_int8 = W.pixai_convert_checkpoint(raw, cfg)
    _write(tmp_path / "official", raw, {"num_classes": cfg.num_tags})
    _write(tmp_path / "converted", ref_int8, {"num_classes": cfg.num_tags}, {"format": W.PIXAI_INT8_FORMAT})
    assert BK.model_kind(tmp_path / "official") == "pixai"
    assert BK.model_kind(tmp_path / "converted") == "pixai"
    c1, w1 = BK.load_weights(tmp_path / "official", cfg, torch.device("cpu"))
    c2, w2 = BK.load_weights(tmp_path / "converted", cfg, torch.device("cpu"))
    assert c1 == c2 == cfg
    assert w1.keys() == w2.keys()
    for k in w1:
        assert torch.equal(w1[k], w2[k]), k


def test_pixai_directory_default_shape_from_checkpoint(tmp_path):
    """Without an explicit config a PixAI directory runs the reference's PixAI-1008 shape, tags from the head."""
    cfg = _tiny_pixai()
    raw = W.pixai_random_raw(cfg, seed=3, pre_grid=12)
    _write(tmp_path / "m", {"head.weight": raw["head.weight"], "patch_embed.proj.weight": raw["patch_embed.proj.weight"]},
           {})
    from safetensors.torch import load_file

    got = load_file(str(tmp_path / "m" / "model.safetensors"))
    assert "patch_embed.proj.weight" in got
    assert BK.model_kind(tmp_path / "m") == "pixai"
    with pytest.raises(KeyError):  # the partial checkpoint stops at the first missing tensor, after picking PixAI
        BK.load_weights(tmp_path / "m", None, torch.device("cpu"))


def test_haruka_directory_is_recognised(tmp_path):
    """A Haruka Tagger directory (config.json with "categories") selects the EVA02-B engine instead of being
    refused (the reference runs it on MLX only)."""
    cfg = EVA02_B.with_(name="haruka-tiny", image_size=56, depth=1, num_tags=40)
    raw = W.random_raw(cfg, seed=1)
    folded = {k: v for k, v in raw.items() if k not in ("pos_embed", "patch_b", "cls_token")}
    folded["patch_b"] = (raw["patch_b"][None, :] + raw["pos_embed"][1:]).contiguous()
    folded["cls"] = (raw["cls_token"] + raw["pos_embed"][0])[None].contiguous()
    _write(tmp_path / "h", folded, {"categories": {"general": 0}})
    assert BK.model_kind(tmp_path / "h") == "haruka"
    got_cfg, conv = BK.load_weights(tmp_path / "h", cfg, torch.device("cpu"))
    ref = W.convert(raw, cfg)
    assert got_cfg == cfg
    for k in ("blocks.0.qkv.qweight", "blocks.0.fc1.qweight", "pos_bias", "cls_row", "head.weight"):
        torch.testing.assert_close(conv[k], ref[k], rtol=0, atol=1e-6 if conv[k].is_floating_point() else 0)
