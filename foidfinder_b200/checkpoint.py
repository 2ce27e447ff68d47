"""The engine's int8 checkpoint on disk: what `weights.convert` produces (rotated per-channel int8 block
linears with interleaved gate|up rows and the padded SwiGLU width, fp16 stem/head, f32 norms, RoPE tables,
tree-pool tensors), saved once so serving skips the load-time conversion.

Counterpart of the reference's `foidfinder convert` (foidfinder/cli.py:143-161), which writes
`convert_checkpoint` (foidfinder/backends/cuda/engine.py:49-62) to `model.safetensors` tagged with
metadata {"format": "foidfinder-pixai-int8-v1"}. This format carries the same `.qweight/.wscale/.bias`
tensor names and adds what that one has no room for: the SwiGLU layout and the model shape, stored as
metadata so `load` can rebuild the `ModelConfig`.

    python -m foidfinder_b200.checkpoint --config eva02-b-448 --src folded.safetensors --out model_dir
"""

from __future__ import annotations

import argparse
import dataclasses
import json
from pathlib import Path

import torch

from .config import CONFIGS, ModelConfig
from . import weights as W

FORMAT = "foidfinder-b200-eva02-int8-v1"
FILE = "model.safetensors"


def save(conv: dict[str, torch.Tensor], cfg: ModelConfig, out_dir: str | Path) -> Path:
    from safetensors.torch import save_file

    out = Path(out_dir)
    out.mkdir(parents=True, exist_ok=True)
    meta = {"format": FORMAT, "config": json.dumps(dataclasses.asdict(cfg))}
    save_file({k: v.detach().contiguous().cpu() for k, v in conv.items()}, str(out / FILE), meta)
    return out / FILE


def is_int8_checkpoint(model_dir: str | Path) -> bool:
    from safetensors import safe_open

    path = Path(model_dir) / FILE
    if not path.is_file():
        return False
    with safe_open(str(path), framework="pt") as f:
        return (f.metadata() or {}).get("format") == FORMAT


def load(model_dir: str | Path, device: str | torch.device = "cpu") -> tuple[ModelConfig, dict[str, torch.Tensor]]:
    """-> (config, engine-format weights on `device`). Raises ValueError for another format."""
    from safetensors import safe_open

    path = Path(model_dir) / FILE
    with safe_open(str(path), framework="pt", device=str(device)) as f:
        meta = f.metadata() or {}
        if meta.get("format") != FORMAT:
            raise ValueError(f"{path}: format {meta.get('format')!r}, expected {FORMAT!r}")
        fields = json.loads(meta["config"])
        fields = {k: tuple(v) if isinstance(v, list) else v for k, v in fields.items()}  # JSON lists -> tuples
        cfg = ModelConfig(**fields)
        conv = {k: f.get_tensor(k) for k in f.keys()}
    return cfg, conv


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--config", choices=sorted(CONFIGS), required=True)
    ap.add_argument("--src", help="folded fp32/fp16 safetensors (foidfinder/haruka.py:fold layout); "
                    "omitted: the seeded synthetic model")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--out", required=True)
    a = ap.parse_args()
    cfg = CONFIGS[a.config]
    if a.src:
        from safetensors.torch import load_file

        raw = W.from_folded(load_file(a.src), cfg)
    else:
        raw = W.random_raw(cfg, a.seed)
    print(save(W.convert(raw, cfg), cfg, a.out))


if __name__ == "__main__":
    main()
