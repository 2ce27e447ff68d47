"""Oracle restatement of the reference's int8 building blocks (CPU, torch) — test infrastructure only.

- `hadamard`             foidfinder/backends/cuda/engine.py:29-34 (normalised Sylvester matrix)
- `quantize_rows_int8`   engine.py:37-41 (symmetric per-output-channel int8)
- `rotate_weight`        engine.py:58-60 (W' = W · blockdiag(H_n))
- `rot_q8`               csrc/kernels.cu:49-108 and :112-160 (optional LayerNorm, FWHT, per-row int8);
                         quantiser semantics csrc/common.cuh:45-48 (rint, clamp ±127); the EVA02
                         LayerNorm eps and masked SwiGLU width: mlx/haruka.py:19, mlx/kernels.py:32-72
- `gemm_s8_acc`          csrc/gemm.cuh:43-117 (exact int32 accumulation of int8 x int8)
- `dequant`              csrc/gemm.cuh:134-136 (acc * row_scale * col_scale + bias)
"""

from __future__ import annotations

import math

import torch


def hadamard(n: int, dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """Normalised Sylvester Hadamard matrix H_n / sqrt(n) (engine.py:29-34)."""
    h = torch.ones(1, 1, dtype=torch.float64)
    while h.shape[0] < n:
        h = torch.cat([torch.cat([h, h], 1), torch.cat([h, -h], 1)], 0)
    return (h / math.sqrt(n)).to(dtype)


def blockdiag_hadamard(cols: int, block: int, dtype: torch.dtype = torch.float64) -> torch.Tensor:
    return torch.block_diag(*[hadamard(block, torch.float64)] * (cols // block)).to(dtype)


def quantize_rows_int8(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-output-channel symmetric int8 (engine.py:37-41): w ~= q * scale[:, None]."""
    scale = w.abs().amax(1).clamp_min(1e-12) / 127.0
    q = torch.round(w / scale[:, None]).clamp(-127, 127).to(torch.int8)
    return q.contiguous(), scale.float().contiguous()


def rotate_weight(w: torch.Tensor, block: int) -> torch.Tensor:
    """W' = W · blockdiag(H_block) in float32, as convert_checkpoint does (engine.py:58-60)."""
    rot = blockdiag_hadamard(w.shape[1], block, torch.float32)
    return w.float() @ rot


def layer_norm(x: torch.Tensor, w: torch.Tensor | None, b: torch.Tensor | None, eps: float) -> torch.Tensor:
    """f32 LayerNorm over the last dim (F.layer_norm semantics)."""
    x = x.float()
    mean = x.mean(-1, keepdim=True)
    var = ((x - mean) ** 2).mean(-1, keepdim=True)
    y = (x - mean) * torch.rsqrt(var + eps)
    if w is not None:
        y = y * w.float() + b.float()
    return y


def rot_q8(
    x: torch.Tensor,
    gamma: torch.Tensor | None,
    beta: torch.Tensor | None,
    *,
    block: int,
    eps: float = 1e-6,
    valid_cols: int | None = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """fp16 rows -> [LayerNorm over the first valid_cols columns; the rest set to 0] -> blockdiag(H_block)
    -> scale = max(amax, 1e-12) / 127 -> codes clamp(rint(v * (1/scale)), ±127).

    Follows rot_q8_1024_kernel (kernels.cu:49-108) / rot_q8_h128_kernel (kernels.cu:112-160), including
    the multiplication by the f32 reciprocal of the scale (kernels.cu:94, :147) and round-half-even.
    Returns (codes int8 [T, C], row_scale f32 [T]).
    """
    T, cols = x.shape
    valid = valid_cols or cols
    v = x.float().clone()
    if gamma is not None:
        v[:, :valid] = layer_norm(v[:, :valid], gamma[:valid], beta[:valid], eps)
    v[:, valid:] = 0.0
    r = (v.double().view(T, cols // block, block) @ hadamard(block, torch.float64).to(v.device)).view(T, cols).float()
    amax = r.abs().amax(1)
    scale = amax.clamp_min(1e-12) / 127.0
    inv = (1.0 / scale).float()
    q = torch.round(r * inv[:, None]).clamp(-127, 127).to(torch.int8)
    return q, scale.float()


def rot_q8_f32_fwht(x, gamma, beta, *, block, eps=1e-6, valid_cols=None):
    """`rot_q8` with the Hadamard product rounded in f32 instead of f64. Not a reference algorithm: the
    tests use it only to measure how far the int8 pipeline moves when nothing but rounding order
    changes (the calibration of the free-running GPU-vs-oracle tolerance)."""
    T, cols = x.shape
    valid = valid_cols or cols
    v = x.float().clone()
    if gamma is not None:
        v[:, :valid] = layer_norm(v[:, :valid], gamma[:valid], beta[:valid], eps)
    v[:, valid:] = 0.0
    r = (v.view(T, cols // block, block) @ hadamard(block, torch.float32).to(v.device)).view(T, cols)
    scale = r.abs().amax(1).clamp_min(1e-12) / 127.0
    q = torch.round(r * (1.0 / scale)[:, None]).clamp(-127, 127).to(torch.int8)
    return q, scale.float()


def gemm_s8_acc(A: torch.Tensor, W: torch.Tensor) -> torch.Tensor:
    """Exact int32 accumulators of int8 A [M, K] x int8 W [N, K]^T (gemm.cuh:43-117)."""
    if A.shape[0] >= 17 and A.shape[1] % 8 == 0 and W.shape[0] % 8 == 0:
        return torch._int_mm(A.contiguous(), W.t().contiguous())  # exact on the CPU and on CUDA devices
    return (A.long() @ W.long().t()).to(torch.int32)


def dequant(acc: torch.Tensor, row_scale: torch.Tensor, col_scale: torch.Tensor, bias: torch.Tensor) -> torch.Tensor:
    """y = acc * row_scale[m] * col_scale[n] + bias[n] in f32 (gemm.cuh:134-136)."""
    return acc.float() * row_scale.float()[:, None] * col_scale.float()[None, :] + bias.float()[None, :]


def silu_mul(g: torch.Tensor, u: torch.Tensor) -> torch.Tensor:
    """SwiGLU gate: silu(g) * u (mlx/kernels.py:45-47, timm SwiGLU)."""
    return g / (1.0 + torch.exp(-g)) * u


def apply_rope_pairs(y: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, pos: torch.Tensor, cols: int) -> torch.Tensor:
    """Rotates interleaved pairs (2i, 2i+1) of every 64-wide head in columns [0, cols) of y [M, N] by the
    angle of pair i % 32 at row position pos[m] (mlx/kernels.py:12-29; reference.py:37-41 for the pair
    convention). cos/sin: [positions, 32]."""
    out = y.clone()
    part = y[:, :cols].reshape(y.shape[0], cols // 64, 32, 2)
    pos = pos.to(y.device)
    c = cos.to(y.device)[pos][:, None, :]
    s = sin.to(y.device)[pos][:, None, :]
    x0, x1 = part[..., 0], part[..., 1]
    rot = torch.stack([x0 * c - x1 * s, x0 * s + x1 * c], dim=-1)
    out[:, :cols] = rot.reshape(y.shape[0], cols)
    return out
