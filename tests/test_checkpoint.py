"""The int8 checkpoint format: save/load round trip (bit-identical tensors, config restored), format
tag checks, and the backend's loader choosing it (CPU)."""

import pytest
import torch

from foidfinder_b200 import checkpoint, weights
from foidfinder_b200.config import EVA02_B, EVA02_L


@pytest.mark.parametrize("cfg", [EVA02_L.with_(name="ckpt-l", image_size=56, depth=1),
                                 EVA02_B.with_(name="ckpt-b", image_size=56, depth=1, num_tags=300)])
def test_round_trip(tmp_path, cfg):
    conv = weights.convert(weights.random_raw(cfg, seed=2), cfg)
    checkpoint.save(conv, cfg, tmp_path)
    assert checkpoint.is_int8_checkpoint(tmp_path)
    cfg2, conv2 = checkpoint.load(tmp_path)
    assert cfg2 == cfg
    assert conv2.keys() == conv.keys()
    for k in conv:
        assert conv2[k].dtype == conv[k].dtype and torch.equal(conv2[k], conv[k]), k


def test_rejects_other_formats(tmp_path):
    from safetensors.torch import save_file

    save_file({"x": torch.zeros(2)}, str(tmp_path / "model.safetensors"), {"format": "foidfinder-pixai-int8-v1"})
    assert not checkpoint.is_int8_checkpoint(tmp_path)
    with pytest.raises(ValueError, match="expected"):
        checkpoint.load(tmp_path)


def test_backend_loader_prefers_int8_checkpoint(tmp_path):
    from foidfinder_b200.backend import load_weights

    cfg = EVA02_L.with_(name="ckpt-loader", image_size=56, depth=1)
    conv = weights.convert(weights.random_raw(cfg, seed=3), cfg)
    checkpoint.save(conv, cfg, tmp_path)
    got_cfg, got = load_weights(tmp_path, EVA02_L, torch.device("cpu"))
    assert got_cfg == cfg and torch.equal(got["blocks.0.qkv.qweight"], conv["blocks.0.qkv.qweight"])
