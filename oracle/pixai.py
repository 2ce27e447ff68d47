"""Oracle restatement of the reference's PixAI layout helpers (CPU, torch) — test infrastructure only.

- `axial_rope`   foidfinder/backends/cuda/reference.py:27-34 (x bands then y bands, fp32)
- `apply_rope`   reference.py:37-41 (interleaved pairs, fp32, cast back)
"""

from __future__ import annotations

import torch

D = 64


def axial_rope(end: int, scale: float) -> tuple[torch.Tensor, torch.Tensor]:
    freqs = 1.0 / (10000.0 ** (torch.arange(0, D, 4)[: D // 4].float() / D))
    t = torch.arange(end * end, dtype=torch.float32)
    tx = (t % end) * scale
    ty = torch.div(t, end, rounding_mode="floor") * scale
    ang = torch.cat([torch.outer(tx, freqs), torch.outer(ty, freqs)], dim=-1)
    return torch.cos(ang), torch.sin(ang)


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    xf = x.float().unflatten(-1, (D // 2, 2))
    x0, x1 = xf[..., 0], xf[..., 1]
    return torch.stack([x0 * cos - x1 * sin, x0 * sin + x1 * cos], dim=-1).flatten(-2).to(x.dtype)

