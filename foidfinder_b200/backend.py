"""`CUDABackend`: the reference's `Backend` protocol (foidfinder/backends/__init__.py:17-23) on the B200
engine. `predict(image)` returns [num_tags] float32 probabilities; call it from one thread only, as the
protocol states (foidfinder/web.py runs it on a single-thread executor).

It replaces `foidfinder/backends/cuda/__init__.py:15-43`: where that class builds `PixAICuda` for compute
capability 8.0+, this one builds `Engine` on compute capability 10.x and refuses anything else (there is no
fallback). `CUDABackend(model_dir)` reads `model_dir/config.json` as the reference does (`__init__.py:21`):
a Haruka Tagger directory ("categories" in the config; the reference runs it on MLX only) loads the folded
EVA02-B checkpoint, any other directory is PixAI Tagger v1.0 — the official fp32 checkpoint or the
reference's own `foidfinder convert` int8 output, both through `weights.convert_pixai`. This package's own
int8 checkpoint (`checkpoint.save`) carries its config and loads as is.

Preprocessing: transparency composited onto white (foidfinder/image.py:41-48) on the host, then on the GPU
either PixAI's float letterbox (`preprocess`: antialiased bilinear in f32, x * 2 - 1 in fp16 on a -1
canvas, foidfinder/backends/cuda/preprocess.py:16-32) into the engine's fp16 pixel input, or for the
EVA02 shapes Pillow's 8-bit resize (bicubic on white for Haruka, mlx/kernels.py:75-186) into its uint8
input.
"""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import torch

from .config import CONFIGS, EVA02_B, EVA02_L, PIXAI_1008, ModelConfig
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


def preprocess(images: list, size: int, device: torch.device) -> torch.Tensor:
    """PIL images -> [B, size, size, 3] fp16 normalised pixels on `device`: PixAI's letterbox
    (foidfinder/backends/cuda/preprocess.py:16-32) with the resize on the GPU (ff_letterbox_aa_f16)."""
    from . import ops

    out = torch.empty(len(images), size, size, 3, dtype=torch.float16, device=device)
    for b, image in enumerate(images):
        rgb = torch.from_numpy(np.array(rgb_on_white(image), dtype=np.uint8)).to(device)
        h, w = rgb.shape[:2]
        r = min(size / h, size / w)
        ops.letterbox_aa_f16(rgb, max(1, int(h * r)), max(1, int(w * r)), size, out[b])
    return out


def model_kind(model_dir: str | Path) -> str:
    """"b200-int8" (checkpoint.save output), "haruka" (config.json has "categories", foidfinder/backends/cuda/
    __init__.py:21) or "pixai" (the official checkpoint or the reference's `foidfinder convert` output)."""
    from . import checkpoint

    if checkpoint.is_int8_checkpoint(model_dir):
        return "b200-int8"
    cfg_file = Path(model_dir) / "config.json"
    if cfg_file.is_file() and "categories" in json.loads(cfg_file.read_text()):
        return "haruka"
    return "pixai"


def load_weights(model_dir: str | Path | None, cfg: ModelConfig | None, device: torch.device, seed: int = 0):
    """Model directory -> (config, engine weights on `device`); `cfg` is the model shape to use when the
    directory does not determine it (None: from the directory). None model_dir -> the seeded synthetic
    model of `cfg`."""
    if model_dir is None:
        cfg = cfg or EVA02_L
        return cfg, W.synthetic(cfg, seed, device)
    from safetensors.torch import load_file

    from . import checkpoint

    kind = model_kind(model_dir)
    if kind == "b200-int8":
        return checkpoint.load(model_dir, device)
    raw = load_file(str(Path(model_dir) / "model.safetensors"), device=str(device))
    if kind == "haruka":
        cfg = cfg or EVA02_B
        return cfg, W.convert(W.from_folded(raw, cfg, device), cfg, device)
    if "patch_embed.proj.weight" not in raw:  # this package's folded EVA02 layout (no reference counterpart)
        cfg = cfg or EVA02_L
        return cfg, W.convert(W.from_folded(raw, cfg, device), cfg, device)
    cfg = cfg or PIXAI_1008.with_(num_tags=int(raw["head.weight"].shape[0]))
    return cfg, W.convert_pixai(raw, cfg, device)


class CUDABackend:
    name = "cuda"

    def __init__(self, model_dir: str | Path | None = None, *, config: ModelConfig | str | None = None, device: int = 0,
                 seed: int = 0):
        """model_dir: a PixAI or Haruka model directory (see the module docstring), or None for the seeded
        synthetic model of `config` (default EVA02-L/448). config: the model shape (a name of CONFIGS or a
        ModelConfig); None = what the directory holds."""
        if not torch.cuda.is_available():
            raise RuntimeError("CUDA backend: no NVIDIA GPU visible")
        cap = torch.cuda.get_device_capability(device)
        if cap[0] != 10:
            raise RuntimeError(f"foidfinder_b200 runs on compute capability 10.x (B200); device {device} is {cap}")
        cfg = CONFIGS[config] if isinstance(config, str) else config
        dev = torch.device("cuda", device)
        torch.cuda.set_device(dev)
        self.cfg, w = load_weights(model_dir, cfg, dev, seed)
        self.engine = Engine(self.cfg, w, device=device)
        self.device = torch.cuda.get_device_name(device)

    def prepare(self, image) -> torch.Tensor:
        """Decoded image -> the engine's input [S, S, 3] on this backend's GPU (resize on the GPU): fp16
        normalised pixels for PixAI, uint8 for the EVA02 shapes."""
        c = self.cfg
        if c.arch == "pixai":
            return preprocess([image], c.image_size, self.engine.device)[0]
        return letterbox_gpu(image, c.image_size, c.resample, c.pad, self.engine.device)

    @torch.no_grad()
    def predict(self, image) -> np.ndarray:
        return torch.sigmoid(self.engine(self.prepare(image)[None]))[0].cpu().numpy()

    @torch.no_grad()
    def predict_batch(self, images: list) -> np.ndarray:
        """Several decoded images in one graph replay -> [B, num_tags] probabilities."""
        x = torch.stack([self.prepare(im) for im in images])
        return torch.sigmoid(self.engine(x)).cpu().numpy()
