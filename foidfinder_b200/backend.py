"""`CUDABackend`: the reference's `Backend` protocol (foidfinder/backends/__init__.py:17-23) on the B200
engine. `predict(image)` returns [num_tags] float32 probabilities; call it from one thread only, as the
protocol states (foidfinder/web.py runs it on a single-thread executor).

It replaces `foidfinder/backends/cuda/__init__.py:15-43`: where that class builds `PixAICuda` for compute
capability 8.0+, this one builds `Engine` on compute capability 10.x and refuses anything else (there is no
fallback). Preprocessing is the reference's letterbox (foidfinder/backends/cuda/preprocess.py:16-32):
transparency composited onto white (foidfinder/image.py:41-48), aspect-preserving antialiased bilinear
resize, centred on black — done on the host into the engine's uint8 input, outside the hot path.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import torch

from .config import CONFIGS, EVA02_L, ModelConfig
from .engine import Engine
from . import weights as W


def rgb_on_white(image):
    """RGB with any transparency composited onto white (foidfinder/image.py:41-48)."""
    from PIL import Image

    if image.mode == "RGB":
        return image
    rgba = image.convert("RGBA")
    canvas = Image.new("RGBA", rgba.size, (255, 255, 255, 255))
    canvas.alpha_composite(rgba)
    return canvas.convert("RGB")


def letterbox(image, size: int) -> np.ndarray:
    """PIL image -> uint8 [size, size, 3]: the longer side scaled to `size` (antialiased bilinear), the
    rest black, centred (preprocess.py:16-32; black is -1 after the mean/std 0.5 normalisation)."""
    from PIL import Image

    rgb = rgb_on_white(image)
    w, h = rgb.size
    r = min(size / h, size / w)
    nh, nw = int(h * r), int(w * r)
    if (nh, nw) != (h, w):
        rgb = rgb.resize((nw, nh), Image.BILINEAR, reducing_gap=None)
    out = np.zeros((size, size, 3), np.uint8)
    top, left = (size - nh) // 2, (size - nw) // 2
    out[top : top + nh, left : left + nw] = np.asarray(rgb, dtype=np.uint8)
    return out


def load_weights(model_dir: str | Path | None, cfg: ModelConfig, device: torch.device, seed: int = 0):
    """`model_dir/model.safetensors` in the folded layout (haruka.py:fold) or this package's raw layout ->
    engine weights on `device`; None -> the seeded synthetic model."""
    if model_dir is None:
        return W.synthetic(cfg, seed, device)
    from safetensors.torch import load_file

    raw = W.from_folded(load_file(str(Path(model_dir) / "model.safetensors")), cfg, device)
    return W.convert(raw, cfg, device)


class CUDABackend:
    name = "cuda"

    def __init__(self, model_dir: str | Path | None = None, *, config: ModelConfig | str = EVA02_L, device: int = 0,
                 seed: int = 0):
        if not torch.cuda.is_available():
            raise RuntimeError("CUDA backend: no NVIDIA GPU visible")
        cap = torch.cuda.get_device_capability(device)
        if cap[0] != 10:
            raise RuntimeError(f"foidfinder_b200 runs on compute capability 10.x (B200); device {device} is {cap}")
        self.cfg = CONFIGS[config] if isinstance(config, str) else config
        dev = torch.device("cuda", device)
        self.engine = Engine(self.cfg, load_weights(model_dir, self.cfg, dev, seed), device=device)
        self.device = torch.cuda.get_device_name(device)

    @torch.no_grad()
    def predict(self, image) -> np.ndarray:
        x = torch.from_numpy(letterbox(image, self.cfg.image_size))[None]
        return torch.sigmoid(self.engine(x))[0].cpu().numpy()

    @torch.no_grad()
    def predict_batch(self, images: list) -> np.ndarray:
        """Several decoded images in one graph replay -> [B, num_tags] probabilities."""
        x = torch.from_numpy(np.stack([letterbox(im, self.cfg.image_size) for im in images]))
        return torch.sigmoid(self.engine(x)).cpu().numpy()
