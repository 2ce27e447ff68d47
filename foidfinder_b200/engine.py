"""`Engine`: the whole int8 forward on one B200, through the C ABI's engine object.

Replaces `PixAICuda` (foidfinder/backends/cuda/engine.py:65-184): `engine(images)` returns fp32 logits
[B, num_tags], the first call for a batch size allocates that size's activation buffers and captures the
forward in a CUDA graph (engine.py:163-184), later calls replay it. The input is what PixAICuda takes —
normalised pixels [B, S, S, 3] of any float dtype, cast to fp16 as the reference's static input does
(engine.py:170, :182) — or uint8 images [B, S, S, 3], normalised on the GPU with the config's mean/std.
Weights stay owned by this object (torch tensors) and are handed to the library as device pointers.
"""

from __future__ import annotations

import ctypes as C

import torch

from . import _lib
from .config import ModelConfig
from .weights import synthetic

_LAYER_KEYS = {
    "norm1_w": "norm1.weight",
    "norm1_b": "norm1.bias",
    "qkv_w": "qkv.qweight",
    "qkv_s": "qkv.wscale",
    "qkv_b": "qkv.bias",
    "proj_w": "proj.qweight",
    "proj_s": "proj.wscale",
    "proj_b": "proj.bias",
    "norm2_w": "norm2.weight",
    "norm2_b": "norm2.bias",
    "fc1_w": "fc1.qweight",
    "fc1_s": "fc1.wscale",
    "fc1_b": "fc1.bias",
    "mlp_norm_w": "mlp_norm.weight",
    "mlp_norm_b": "mlp_norm.bias",
    "fc2_w": "fc2.qweight",
    "fc2_s": "fc2.wscale",
    "fc2_b": "fc2.bias",
}


def c_config(cfg: ModelConfig) -> _lib.ModelConfig:
    c = _lib.ModelConfig()
    c.image_size, c.patch, c.dim, c.depth, c.heads = cfg.image_size, cfg.patch, cfg.dim, cfg.depth, cfg.heads
    c.mlp_hidden, c.mlp_hidden_pad = cfg.mlp_hidden, cfg.mlp_hidden_pad
    c.num_tags, c.num_tags_pad = cfg.num_tags, cfg.num_tags_pad
    c.rot_block_dim, c.rot_block_hidden, c.topk, c.ln_eps = cfg.rot_block_dim, cfg.rot_block_hidden, cfg.topk, cfg.ln_eps
    c.mean = (C.c_float * 3)(*cfg.mean)
    c.std = (C.c_float * 3)(*cfg.std)
    c.head_kind = {"cls": _lib.HEAD_CLS, "tree": _lib.HEAD_TREE, "pool": _lib.HEAD_POOL}[cfg.head]
    c.pool_heads, c.coarse_queries, c.leaf_queries, c.leaf_dim = (
        cfg.pool_heads, cfg.coarse_queries, cfg.leaf_queries, cfg.leaf_dim)
    c.arch = _lib.ARCH_PIXAI if cfg.arch == "pixai" else _lib.ARCH_EVA02
    c.window = cfg.window
    c.global_blocks = sum(1 << i for i in cfg.global_blocks if i < 64)
    return c


_POOL_KEYS = {
    "pool_norm_w": "pool.norm.weight",
    "pool_norm_b": "pool.norm.bias",
    "pool_kv_w": "pool.kv.weight",
    "pool_kv_b": "pool.kv.bias",
    "q_coarse": "pool.q_coarse",
    "q_coarse_bias": "pool.q_coarse_bias",
    "q_child": "pool.q_child",
    "q_child_bias": "pool.q_child_bias",
    "trunk_norm_w": "pool.trunk_norm.weight",
    "trunk_norm_b": "pool.trunk_norm.bias",
    "child_q_norm_w": "pool.child_q_norm.weight",
    "child_q_norm_b": "pool.child_q_norm.bias",
    "leaf_norm_w": "pool.leaf_norm.weight",
    "leaf_norm_b": "pool.leaf_norm.bias",
    "leaf_w": "pool.leaf.weight",
    "leaf_b": "pool.leaf.bias",
}

_PIXAI_KEYS = {
    "ln_pre_w": "ln_pre.weight",
    "ln_pre_b": "ln_pre.bias",
    "rope_cos_global": "rope_cos_global",
    "rope_sin_global": "rope_sin_global",
    "pool_norm_w": "pool.norm.weight",
    "pool_norm_b": "pool.norm.bias",
    "pool_kv_w": "pool.kv.weight",
    "pool_kv_b": "pool.kv.bias",
    "pool_pos": "pool.pos",
    "pool_q": "pool.q",
    "pool_proj_w": "pool.proj.weight",
    "pool_proj_b": "pool.proj.bias",
}


def c_weights(cfg: ModelConfig, L: dict[str, torch.Tensor], layers) -> _lib.ModelWeights:
    """Device tensors in the engine format -> the C weight struct (pointers only; `L` must stay alive)."""
    def ptr(key: str) -> int | None:
        t = L.get(key)
        return t.data_ptr() if t is not None else None

    for i in range(cfg.depth):
        for field, key in _LAYER_KEYS.items():
            setattr(layers[i], field, ptr(f"blocks.{i}.{key}"))
    mw = _lib.ModelWeights()
    mw.patch_w, mw.pos_bias, mw.cls_row = ptr("patch_w"), ptr("pos_bias"), ptr("cls_row")
    mw.rope_cos, mw.rope_sin = ptr("rope_cos"), ptr("rope_sin")
    mw.layers = C.cast(layers, C.POINTER(_lib.LayerWeights))
    mw.norm_w, mw.norm_b = ptr("norm.weight"), ptr("norm.bias")
    mw.head_w, mw.head_b = ptr("head.weight"), ptr("head.bias")
    extra = {"tree": _POOL_KEYS, "pool": _PIXAI_KEYS}.get(cfg.head, {})
    for field, key in extra.items():
        setattr(mw, field, ptr(key))
    return mw


class Engine:
    def __init__(self, cfg: ModelConfig, weights: dict[str, torch.Tensor] | None = None, *, device: int | str = 0,
                 seed: int = 0):
        """weights: the output of `weights.convert` (any device; moved here). None = seeded random init."""
        self.cfg = cfg
        self.device = torch.device("cuda", torch.device(device).index if isinstance(device, str) else device)
        if weights is None:
            weights = synthetic(cfg, seed, self.device)
        self.w = {k: v.to(self.device).contiguous() for k, v in weights.items()}
        self._c_cfg = c_config(cfg)
        self._layers = (_lib.LayerWeights * cfg.depth)()
        mw = c_weights(cfg, self.w, self._layers)
        self._c_w = mw
        handle = C.c_void_p()
        _lib.check(
            _lib.lib().ff_engine_create(C.byref(self._c_cfg), C.byref(mw), self.device.index, C.byref(handle)),
            "ff_engine_create",
        )
        self._h = handle

    def workspace_bytes(self, B: int) -> int:
        return int(_lib.lib().ff_engine_workspace_bytes(C.byref(self._c_cfg), B))

    @torch.no_grad()
    def forward(
        self,
        images: torch.Tensor,
        *,
        logits: torch.Tensor | None = None,
        topk: bool = True,
        graph: bool = True,
    ) -> tuple[torch.Tensor, torch.Tensor | None, torch.Tensor | None]:
        """images [B, S, S, 3] uint8, or normalised float pixels (any float dtype, used as fp16) ->
        (logits [B, tags] f32, top-k indices [B, k] int32, values [B, k] f32)."""
        cfg = self.cfg
        pixels = images.is_floating_point()
        if (images.dtype != torch.uint8 and not pixels) or images.dim() != 4 or \
                tuple(images.shape[1:]) != (cfg.image_size,) * 2 + (3,):
            raise ValueError(f"images must be uint8 or normalised float pixels [B, {cfg.image_size}, "
                             f"{cfg.image_size}, 3]")
        if pixels:
            images = images.to(self.device, torch.float16, non_blocking=True).contiguous()
        else:
            images = images.to(self.device, non_blocking=True).contiguous()
        B = images.shape[0]
        if logits is None:
            logits = torch.empty(B, cfg.num_tags, device=self.device, dtype=torch.float32)
        idx = torch.empty(B, cfg.topk, device=self.device, dtype=torch.int32) if topk and cfg.topk else None
        val = torch.empty(B, cfg.topk, device=self.device, dtype=torch.float32) if idx is not None else None
        lib = _lib.lib()
        ip = idx.data_ptr() if idx is not None else None
        vp = val.data_ptr() if val is not None else None
        with torch.cuda.device(self.device):
            stream = torch.cuda.current_stream(self.device).cuda_stream
            if pixels:
                rc = lib.ff_engine_forward_pixels(self._h, images.data_ptr(), B, logits.data_ptr(), ip, vp,
                                                  1 if graph else 0, stream)
            else:
                fn = lib.ff_engine_forward if graph else lib.ff_engine_forward_eager
                rc = fn(self._h, images.data_ptr(), B, logits.data_ptr(), ip, vp, stream)
            _lib.check(rc, "ff_engine_forward")
        return logits, idx, val

    def __call__(self, images: torch.Tensor) -> torch.Tensor:
        """images [B, S, S, 3] normalised float pixels or uint8 -> logits [B, num_tags] f32 (PixAICuda.__call__,
        engine.py:163-184)."""
        return self.forward(images, topk=False)[0]

    @property
    def launches_per_forward(self) -> int:
        return int(_lib.lib().ff_engine_launches_per_forward(C.byref(self._c_cfg)))

    @torch.no_grad()
    def profile(self, images: torch.Tensor, iters: int = 3) -> dict[str, tuple[float, int]]:
        """Mean ms per forward and launches per forward of each kernel class (eager launches, CUDA events)."""
        images = images.to(self.device).contiguous()
        ms = (C.c_float * len(_lib.PROF_CLASSES))()
        n = (C.c_int * len(_lib.PROF_CLASSES))()
        with torch.cuda.device(self.device):
            stream = torch.cuda.current_stream(self.device).cuda_stream
            _lib.check(
                _lib.lib().ff_engine_profile(self._h, images.data_ptr(), images.shape[0], iters, ms, n, stream),
                "ff_engine_profile",
            )
        return {k: (ms[i], n[i]) for i, k in enumerate(_lib.PROF_CLASSES)}

    def device_error(self) -> int:
        return _lib.device_error(self.device.index, clear=True)

    def close(self) -> None:
        if getattr(self, "_h", None):
            _lib.lib().ff_engine_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
