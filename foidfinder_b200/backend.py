"""`CUDABackend`: the reference's `Backend` protocol (foidfinder/backends/__init__.py:17-23) on the B200
engine. `predict(image)` returns [num_tags] float32 probabilities; call it from one thread only, as the
protocol states (foidfinder/web.py runs it on a single-thread executor).

It replaces `foidfinder/backends/cuda/__init__.py:15-43`: where that class builds `PixAICuda` for compute
capability 8.0+, this one builds `Engine` on compute capability 10.x and refuses anything else (there is no
fallback). Preprocessing is the reference's letterbox (foidfinder/backends/cuda/preprocess.py:16-32):
transparency composited onto white (foidfinder/image.py:41-48) on the host, then the aspect-preserving
resize (bilinear on black for the PixAI shape, bicubic on white for Haruka) on the GPU with Pillow's
fixed-point arithmetic (ff_resize_pad), written straight into the engine's uint8 input.
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


def letterbox_size(h: int, w: int, size: int) -> tuple[int, int]:
    """Resized (h, w) with the longer side at `size` (preprocess.py:24-26; at least 1 pixel as in
    mlx/haruka.py:67-73)."""
    r = min(size / h, size / w)
    return max(1, int(h * r)), max(1, int(w * r))


def letterbox(image, size: int, resample: str = "bilinear", pad: int = 0) -> np.ndarray:
    """PIL image -> uint8 [size, size, 3] on the host: transparency on white, the longer side scaled to
    `size` (Pillow bilinear or bicubic, antialiased when reducing), centred on a `pad` canvas — PixAI's
    preprocessing (preprocess.py:16-32; black is -1 after the mean/std 0.5 normalisation) or Haruka's
    (bicubic on white)."""
    from PIL import Image

    rgb = rgb_on_white(image)
    w, h = rgb.size
    nh, nw = letterbox_size(h, w, size)
    if (nh, nw) != (h, w):
        flt = Image.BICUBIC if resample == "bicubic" else Image.BILINEAR
        rgb = rgb.resize((nw, nh), flt, reducing_gap=None)
    out = np.full((size, size, 3), pad, np.uint8)
    top, left = (size - nh) // 2, (size - nw) // 2
    out[top : top + nh, left : left + nw] = np.asarray(rgb, dtype=np.uint8)
    return out


def letterbox_gpu(image, size: int, resample: str, pad: int, device: torch.device) -> torch.Tensor:
    """The same letterbox with the resize on the GPU (ff_resize_pad, bit-exact with Pillow):
    PIL image -> uint8 [size, size, 3] on `device`."""
    from . import ops

    rgb = torch.from_numpy(np.array(rgb_on_white(image), dtype=np.uint8)).to(device)
    h, w = rgb.shape[:2]
    nh, nw = letterbox_size(h, w, size)
    out = torch.empty(size, size, 3, dtype=torch.uint8, device=device)
    ops.resize_pad(rgb, nh, nw, size, out, bicubic=resample == "bicubic", fill=pad)
    return out


def load_weights(model_dir: str | Path | None, cfg: ModelConfig, device: torch.device, seed: int = 0):
    """`model_dir/model.safetensors` -> (config, engine weights on `device`): an int8 checkpoint written by
    `checkpoint.save` is used as is (its stored config wins); a folded checkpoint (haruka.py:fold layout)
    or this package's raw layout is converted. None -> the seeded synthetic model."""
    if model_dir is None:
        return cfg, W.synthetic(cfg, seed, device)
    from . import checkpoint

    if checkpoint.is_int8_checkpoint(model_dir):
        return checkpoint.load(model_dir, device)
    from safetensors.torch import load_file

    raw = W.from_folded(load_file(str(Path(model_dir) / "model.safetensors")), cfg, device)
    return cfg, W.convert(raw, cfg, device)


class CUDABackend:
    name = "cuda"

    def __init__(self, model_dir: str | Path | None = None, *, config: ModelConfig | str = EVA02_L, device: int = 0,
                 seed: int = 0):
        if not torch.cuda.is_available():
            raise RuntimeError("CUDA backend: no NVIDIA GPU visible")
        cap = torch.cuda.get_device_capability(device)
        if cap[0] != 10:
            raise RuntimeError(f"foidfinder_b200 runs on compute capability 10.x (B200); device {device} is {cap}")
        cfg = CONFIGS[config] if isinstance(config, str) else config
        dev = torch.device("cuda", device)
        self.cfg, w = load_weights(model_dir, cfg, dev, seed)
        self.engine = Engine(self.cfg, w, device=device)
        self.device = torch.cuda.get_device_name(device)

    def prepare(self, image) -> torch.Tensor:
        """Decoded image -> the engine's uint8 [S, S, 3] input on this backend's GPU (resize on the GPU)."""
        c = self.cfg
        return letterbox_gpu(image, c.image_size, c.resample, c.pad, self.engine.device)

    @torch.no_grad()
    def predict(self, image) -> np.ndarray:
        return torch.sigmoid(self.engine(self.prepare(image)[None]))[0].cpu().numpy()

    @torch.no_grad()
    def predict_batch(self, images: list) -> np.ndarray:
        """Several decoded images in one graph replay -> [B, num_tags] probabilities."""
        x = torch.stack([self.prepare(im) for im in images])
        return torch.sigmoid(self.engine(x)).cpu().numpy()
