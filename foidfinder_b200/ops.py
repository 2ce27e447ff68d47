"""Per-kernel entry points on torch CUDA tensors, mirroring the reference's `torch.ops.foidfinder` ops
(foidfinder/backends/cuda/csrc/kernels.cu:267-281): outputs are caller-allocated and written in place,
shape/dtype violations raise, and every launch goes on the current CUDA stream. Each call goes through
the C ABI of `libfoidfinder_b200.so`; torch is only the memory and stream plumbing.
"""

from __future__ import annotations

import ctypes as C

import torch

from . import _lib
from ._lib import (
    EPI_BIAS, EPI_GELU, EPI_LOGITS, EPI_QKV_ROPE, EPI_RESIDUAL, EPI_S32, EPI_STEM, EPI_SWIGLU, TILE_PAIR256, check, lib,
)

__all__ = [
    "EPI_QKV_ROPE", "EPI_RESIDUAL", "EPI_SWIGLU", "EPI_BIAS", "EPI_S32", "EPI_STEM", "EPI_LOGITS", "EPI_GELU", "TILE_PAIR256",
    "gemm_s8", "gemm_f16", "rot_q8", "rot_q8_1024", "rot_q8_h128", "attention", "patchify", "fill_cls",
    "layernorm", "topk", "tree_pool", "resize_pad", "patchify_windowed", "layernorm_pos", "pool_query_attention",
]


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _need(cond: bool, msg: str) -> None:
    if not cond:
        raise RuntimeError(msg)


def _cuda(*ts: torch.Tensor | None) -> None:
    for t in ts:
        if t is not None:
            _need(t.is_cuda and t.is_contiguous(), "expected contiguous CUDA tensors")


def gemm_s8(
    A: torch.Tensor,
    W: torch.Tensor,
    row_scale: torch.Tensor | None,
    col_scale: torch.Tensor | None,
    bias: torch.Tensor | None,
    out: torch.Tensor,
    epi: int,
    tile_n: int = 0,
    rope_cos: torch.Tensor | None = None,
    rope_sin: torch.Tensor | None = None,
    rope_cols: int = 0,
    tokens: int = 1,
) -> None:
    """A [M, K] int8 x W [N, K] int8 -> epilogue into out (see include/foidfinder_b200.h). RoPE tables
    for EPI_QKV_ROPE are angle-major [32, tokens]."""
    _cuda(A, W, row_scale, col_scale, bias, out, rope_cos, rope_sin)
    _need(A.dtype == torch.int8 and W.dtype == torch.int8, "gemm_s8: A and W must be int8")
    M, K = A.shape
    N = W.shape[0]
    _need(W.shape[1] == K, "gemm_s8: K mismatch")
    if epi == EPI_S32:
        _need(out.dtype == torch.int32 and tuple(out.shape) == (M, N), "gemm_s8: S32 out must be int32 [M, N]")
    else:
        cols = N // 2 if epi == EPI_SWIGLU else N
        _need(out.dtype == torch.float16 and tuple(out.shape) == (M, cols), f"gemm_s8: out must be fp16 [{M}, {cols}]")
        _need(row_scale.numel() == M and col_scale.numel() == N and bias.numel() == N, "gemm_s8: scale/bias sizes")
    with torch.cuda.device(A.device):
        check(
            lib().ff_gemm_s8(
                _ptr(A), _ptr(W), _ptr(row_scale), _ptr(col_scale), _ptr(bias), _ptr(out), M, N, K, epi,
                _ptr(rope_cos), _ptr(rope_sin), rope_cols, tokens, tile_n, _stream(A),
            ),
            "gemm_s8",
        )


def gemm_f16(
    A: torch.Tensor,
    W: torch.Tensor,
    out: torch.Tensor,
    epi: int,
    bias: torch.Tensor | None = None,
    n_valid: int | None = None,
    pos_bias: torch.Tensor | None = None,
    patches: int = 0,
    tokens: int = 0,
    tile_n: int = 0,
) -> None:
    """fp16 A [M, K] x W [N, K] with f32 accumulation: EPI_STEM into the token rows of x, EPI_LOGITS into f32."""
    _cuda(A, W, out, bias, pos_bias)
    _need(A.dtype == torch.float16 and W.dtype == torch.float16, "gemm_f16: A and W must be fp16")
    M, K = A.shape
    N = W.shape[0]
    ldo = out.shape[-1]
    nv = n_valid if n_valid is not None else min(N, ldo)
    with torch.cuda.device(A.device):
        check(
            lib().ff_gemm_f16(
                _ptr(A), _ptr(W), _ptr(bias), _ptr(out), M, N, K, epi, ldo, nv, _ptr(pos_bias), patches, tokens,
                tile_n, _stream(A),
            ),
            "gemm_f16",
        )


def rot_q8(
    x: torch.Tensor,
    gamma: torch.Tensor | None,
    beta: torch.Tensor | None,
    out: torch.Tensor,
    row_scale: torch.Tensor,
    *,
    block: int,
    eps: float = 1e-6,
    valid_cols: int | None = None,
) -> None:
    """x [T, C] fp16 -> (LayerNorm) -> block Hadamard -> int8 codes out [T, C] + row_scale [T]."""
    _cuda(x, gamma, beta, out, row_scale)
    _need(x.dtype == torch.float16 and out.dtype == torch.int8 and out.shape == x.shape, "rot_q8: dtypes/shapes")
    T, Ccols = x.shape
    with torch.cuda.device(x.device):
        check(
            lib().ff_rot_q8(
                _ptr(x), _ptr(gamma), _ptr(beta), eps, T, Ccols, valid_cols or Ccols, block, _ptr(out),
                _ptr(row_scale), _stream(x),
            ),
            "rot_q8",
        )


def rot_q8_1024(x, gamma, beta, out, row_scale) -> None:
    """Reference signature (kernels.cu:220): LayerNorm eps 1e-5 if gamma is given, H1024, int8."""
    rot_q8(x, gamma, beta, out, row_scale, block=1024, eps=1e-5)


def rot_q8_h128(x, out, row_scale) -> None:
    """Reference signature (kernels.cu:238): block-H128 rotation and int8, no norm."""
    rot_q8(x, None, None, out, row_scale, block=128)


def attention(
    qkv: torch.Tensor,
    out: torch.Tensor,
    seq_len: int,
    heads: int | None = None,
    rope: tuple[torch.Tensor, torch.Tensor] | None = None,
    scale: float = 1.0,
) -> None:
    """qkv [S * seq_len, 3 * heads * 64] fp16 -> out [S * seq_len, heads * 64] fp16 (non-causal). `rope` must be
    None: q and k arrive rotated, as in the reference (its QKV GEMM epilogue rotates them; here EPI_QKV_ROPE)."""
    _cuda(qkv, out)
    _need(qkv.dtype == torch.float16 and out.dtype == torch.float16, "attention: fp16 tensors expected")
    heads = heads or qkv.shape[1] // 192
    _need(qkv.shape[1] == 3 * heads * 64 and out.shape[1] == heads * 64, "attention: column sizes")
    _need(qkv.shape[0] % seq_len == 0 and out.shape[0] == qkv.shape[0], "attention: row sizes")
    cos, sin = rope if rope is not None else (None, None)
    _cuda(cos, sin)
    with torch.cuda.device(qkv.device):
        check(
            lib().ff_attention(
                _ptr(qkv), _ptr(out), qkv.shape[0] // seq_len, seq_len, heads, _ptr(cos), _ptr(sin), scale,
                _stream(qkv),
            ),
            "attention",
        )


def patchify(images: torch.Tensor, patch: int, mean, std, out: torch.Tensor) -> None:
    _cuda(images, out)
    _need(images.dtype == torch.uint8 and images.dim() == 4, "patchify: uint8 [B, S, S, 3] expected")
    B, S = images.shape[:2]
    m = (C.c_float * 3)(*map(float, mean))
    s = (C.c_float * 3)(*map(float, std))
    with torch.cuda.device(images.device):
        check(lib().ff_patchify(_ptr(images), B, S, patch, m, s, _ptr(out), out.shape[1], _stream(images)), "patchify")


def fill_cls(cls_row: torch.Tensor, x: torch.Tensor, B: int, tokens: int) -> None:
    _cuda(cls_row, x)
    with torch.cuda.device(x.device):
        check(lib().ff_fill_cls(_ptr(cls_row), _ptr(x), B, tokens, x.shape[-1], _stream(x)), "fill_cls")


def layernorm(x: torch.Tensor, row_stride: int, rows: int, cols: int, gamma, beta, eps: float, out: torch.Tensor) -> None:
    _cuda(x, gamma, beta, out)
    with torch.cuda.device(x.device):
        check(
            lib().ff_layernorm(_ptr(x), row_stride, _ptr(gamma), _ptr(beta), eps, rows, cols, _ptr(out), _stream(x)),
            "layernorm",
        )


def topk(logits: torch.Tensor, k: int, idx: torch.Tensor, val: torch.Tensor | None = None) -> None:
    _cuda(logits, idx, val)
    B, n = logits.shape
    with torch.cuda.device(logits.device):
        check(lib().ff_topk(_ptr(logits), B, n, k, _ptr(idx), _ptr(val), _stream(logits)), "topk")


def device_error(device: int = 0, clear: bool = True) -> int:
    """Error code left by a kernel whose bounded wait ran out (0 = none); synchronises the device."""
    return _lib.device_error(device, clear)


def tree_pool(cfg, weights: dict[str, torch.Tensor], x: torch.Tensor, leaf_out: torch.Tensor) -> None:
    """Haruka tree attention pool head: x [B * tokens, dim] fp16 (backbone output before its final
    LayerNorm) -> leaf_out [B, leaf_queries * leaf_dim] fp16. `weights` in the engine format
    (`weights.convert`), on x's device."""
    from .engine import _POOL_KEYS, c_config

    _cuda(x, leaf_out)
    _need(cfg.head == "tree", "tree_pool: config has no tree head")
    _need(x.dtype == torch.float16 and leaf_out.dtype == torch.float16, "tree_pool: fp16 tensors expected")
    B = x.shape[0] // cfg.tokens
    _need(x.shape == (B * cfg.tokens, cfg.dim) and leaf_out.shape == (B, cfg.head_in), "tree_pool: bad shapes")
    c = c_config(cfg)
    mw = _lib.ModelWeights()
    for field, key in {"norm_w": "norm.weight", "norm_b": "norm.bias"}.items():
        setattr(mw, field, weights[key].data_ptr())
    for field, key in _POOL_KEYS.items():
        setattr(mw, field, weights[key].data_ptr())
    nbytes = int(lib().ff_tree_pool_workspace_bytes(C.byref(c), B))
    ws = torch.empty(nbytes, dtype=torch.uint8, device=x.device)
    with torch.cuda.device(x.device):
        check(lib().ff_tree_pool(C.byref(c), C.byref(mw), _ptr(x), B, _ptr(ws), nbytes, _ptr(leaf_out), _stream(x)),
              "tree_pool")
        torch.cuda.current_stream(x.device).synchronize()  # keeps the workspace alive until the pool has run


def resize_pad(image: torch.Tensor, new_h: int, new_w: int, size: int, out: torch.Tensor, *, bicubic: bool = True,
               fill: int = 255) -> None:
    """uint8 [h, w, 3] CUDA image -> out uint8 [size, size, 3]: Pillow-exact resize (bicubic or bilinear) to
    (new_h, new_w), centred on a `fill` canvas."""
    _cuda(image, out)
    _need(image.dtype == torch.uint8 and image.dim() == 3 and image.shape[2] == 3, "resize_pad: uint8 [h, w, 3]")
    _need(out.dtype == torch.uint8 and tuple(out.shape) == (size, size, 3), "resize_pad: out must be [size, size, 3]")
    h, w = image.shape[:2]
    flt = _lib.RESAMPLE_BICUBIC if bicubic else _lib.RESAMPLE_BILINEAR
    nbytes = int(lib().ff_resize_pad_workspace_bytes(h, w, new_h, new_w, flt))
    _need(nbytes > 0, "resize_pad: bad geometry")
    ws = torch.empty(nbytes, dtype=torch.uint8, device=image.device)
    with torch.cuda.device(image.device):
        check(lib().ff_resize_pad(_ptr(image), h, w, new_h, new_w, size, flt, fill, _ptr(out), _ptr(ws), nbytes,
                                  _stream(image)), "resize_pad")
        torch.cuda.current_stream(image.device).synchronize()  # the workspace is freed on return


def letterbox_aa_f16(image: torch.Tensor, new_h: int, new_w: int, size: int, out: torch.Tensor) -> None:
    """uint8 [h, w, 3] CUDA image -> out fp16 [size, size, 3] normalised pixels: PixAI's float letterbox
    (foidfinder/backends/cuda/preprocess.py:16-32): /255, antialiased bilinear resize to (new_h, new_w) in
    f32, x * 2 - 1, centred on a canvas of -1."""
    _cuda(image, out)
    _need(image.dtype == torch.uint8 and image.dim() == 3 and image.shape[2] == 3, "letterbox_aa_f16: uint8 [h, w, 3]")
    _need(out.dtype == torch.float16 and tuple(out.shape[-3:]) == (size, size, 3) and out.is_contiguous(),
          "letterbox_aa_f16: out must be contiguous fp16 [size, size, 3]")
    image = image.contiguous()
    h, w = image.shape[:2]
    with torch.cuda.device(image.device):
        check(lib().ff_letterbox_aa_f16(_ptr(image), h, w, new_h, new_w, size, _ptr(out), _stream(image)),
              "letterbox_aa_f16")


def patchify_windowed(images: torch.Tensor, patch: int, mean, std, window: int, out: torch.Tensor) -> None:
    """uint8 [B, S, S, 3] -> fp16 patch rows [B * (S/patch)^2, k_pad] in window order (window x window tiles)."""
    _cuda(images, out)
    B, S = images.shape[:2]
    m = (C.c_float * 3)(*map(float, mean))
    s = (C.c_float * 3)(*map(float, std))
    with torch.cuda.device(images.device):
        check(lib().ff_patchify_windowed(_ptr(images), B, S, patch, m, s, _ptr(out), out.shape[1], window,
                                         _stream(images)), "patchify_windowed")


def layernorm_pos(x: torch.Tensor, gamma, beta, eps: float, pos: torch.Tensor, out: torch.Tensor) -> None:
    """LayerNorm of fp16 rows to fp16, then + pos[row % pos.shape[0]] in fp16."""
    _cuda(x, gamma, beta, pos, out)
    rows, cols = x.shape
    with torch.cuda.device(x.device):
        check(lib().ff_layernorm_pos(_ptr(x), cols, _ptr(gamma), _ptr(beta), eps, rows, cols, _ptr(pos), pos.shape[0],
                                     _ptr(out), _stream(x)), "layernorm_pos")


def pool_query_attention(q: torch.Tensor, kv: torch.Tensor, B: int, tokens: int, out: torch.Tensor) -> None:
    """q [heads * 64] f32 (scaled), kv [B * tokens, 2 * dim] fp16 -> out [B, dim] fp16."""
    _cuda(q, kv, out)
    heads = q.numel() // 64
    with torch.cuda.device(kv.device):
        check(lib().ff_pool_query_attention(_ptr(q), _ptr(kv), B, tokens, heads, _ptr(out), _stream(kv)),
              "pool_query_attention")


def int8_mma_peak(device: int = 0, iters: int = 200_000) -> float:
    """Measured dense int8 tensor-core throughput of `device` in TOPS (back-to-back tcgen05 MMAs on
    resident operands, one CTA per SM; about 50 ms)."""
    ms, ops = C.c_float(), C.c_double()
    with torch.cuda.device(device):
        check(lib().ff_int8_mma_peak(iters, C.byref(ms), C.byref(ops), torch.cuda.current_stream(device).cuda_stream),
              "int8_mma_peak")
    return ops.value / (ms.value * 1e-3) / 1e12
