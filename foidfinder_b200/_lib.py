"""ctypes binding of `libfoidfinder_b200.so` (the C ABI of include/foidfinder_b200.h).

Plays the role of the reference's kernel loader (foidfinder/backends/cuda/kernels.py:38-48): a prebuilt
library named by $FOIDFINDER_B200_LIB, else the in-tree build. There is no fallback: if the library is
missing or cannot load, `lib()` raises, so nothing silently runs on the CPU.
"""

from __future__ import annotations

import ctypes as C
import os
from functools import cache
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libfoidfinder_b200.so"

FF_OK = 0
FF_ERR_INVALID_ARGUMENT = 1
STATUS = {
    1: "invalid argument",
    2: "unsupported device",
    3: "launch failure",
    4: "device timeout",
    5: "out of memory",
}

# Epilogue ids (include/foidfinder_b200.h); the first two keep the reference's numbering
# (foidfinder/backends/cuda/csrc/gemm.cuh:8-12).
EPI_QKV_ROPE, EPI_RESIDUAL, EPI_SWIGLU, EPI_BIAS, EPI_S32, EPI_STEM, EPI_LOGITS = 0, 1, 3, 4, 5, 6, 7
EPI_GELU = 2
TILE_PAIR256 = 512  # ff_gemm_s8 tile_n: 256 x 256 tiles over a cluster of two CTAs (FF_TILE_PAIR256)

# ff_engine_profile kernel classes (FF_PROF_*).
PROF_CLASSES = ("stem_prep", "stem_gemm", "rotate", "gemm_qkv", "attention", "gemm_proj", "gemm_fc1", "gemm_fc2", "head")

vp, i32, i64, f32 = C.c_void_p, C.c_int, C.c_int64, C.c_float


class ModelConfig(C.Structure):
    _fields_ = [
        ("image_size", i32),
        ("patch", i32),
        ("dim", i32),
        ("depth", i32),
        ("heads", i32),
        ("mlp_hidden", i32),
        ("mlp_hidden_pad", i32),
        ("num_tags", i32),
        ("num_tags_pad", i32),
        ("rot_block_dim", i32),
        ("rot_block_hidden", i32),
        ("topk", i32),
        ("ln_eps", f32),
        ("mean", f32 * 3),
        ("std", f32 * 3),
        ("head_kind", i32),
        ("pool_heads", i32),
        ("coarse_queries", i32),
        ("leaf_queries", i32),
        ("leaf_dim", i32),
        ("arch", i32),
        ("window", i32),
        ("global_blocks", C.c_uint64),
    ]


HEAD_CLS, HEAD_TREE, HEAD_POOL = 0, 1, 2
ARCH_EVA02, ARCH_PIXAI = 0, 1
RESAMPLE_BILINEAR, RESAMPLE_BICUBIC = 0, 1
POOL_FIELDS = (
    "pool_norm_w", "pool_norm_b", "pool_kv_w", "pool_kv_b", "q_coarse", "q_coarse_bias", "q_child", "q_child_bias",
    "trunk_norm_w", "trunk_norm_b", "child_q_norm_w", "child_q_norm_b", "leaf_norm_w", "leaf_norm_b", "leaf_w", "leaf_b",
)
PIXAI_FIELDS = (
    "ln_pre_w", "ln_pre_b", "rope_cos_global", "rope_sin_global", "pool_pos", "pool_q", "pool_proj_w", "pool_proj_b",
)


class LayerWeights(C.Structure):
    _fields_ = [
        (name, vp)
        for name in (
            "norm1_w", "norm1_b", "qkv_w", "qkv_s", "qkv_b", "proj_w", "proj_s", "proj_b", "norm2_w", "norm2_b",
            "fc1_w", "fc1_s", "fc1_b", "mlp_norm_w", "mlp_norm_b", "fc2_w", "fc2_s", "fc2_b",
        )
    ]


class ModelWeights(C.Structure):
    _fields_ = [
        ("patch_w", vp),
        ("pos_bias", vp),
        ("cls_row", vp),
        ("rope_cos", vp),
        ("rope_sin", vp),
        ("layers", C.POINTER(LayerWeights)),
        ("norm_w", vp),
        ("norm_b", vp),
        ("head_w", vp),
        ("head_b", vp),
    ] + [(name, vp) for name in POOL_FIELDS + PIXAI_FIELDS]


_SIGNATURES = {
    "ff_last_error": (C.c_char_p, []),
    "ff_version": (i32, []),
    "ff_device_error": (i32, [i32, C.POINTER(i32), i32]),
    "ff_int8_mma_peak": (i32, [i32, C.POINTER(f32), C.POINTER(C.c_double), vp]),
    "ff_gemm_s8": (i32, [vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, vp, vp, i32, i32, i32, vp]),
    "ff_gemm_f16": (i32, [vp, vp, vp, vp, i32, i32, i32, i32, i32, i32, vp, i32, i32, i32, vp]),
    "ff_rot_q8": (i32, [vp, vp, vp, f32, i32, i32, i32, i32, vp, vp, vp]),
    "ff_linear_w8a8_noalloc": (i32, [vp, vp, vp, f32, i32, i32, i32, i32, vp, vp, vp, vp, i32, i32, vp, vp]),
    "ff_rot_q8_1024": (i32, [vp, vp, vp, i32, vp, vp, vp]),
    "ff_rot_q8_h128": (i32, [vp, i32, i32, vp, vp, vp]),
    "ff_attention": (i32, [vp, vp, i32, i32, i32, vp, vp, f32, vp]),
    "ff_patchify": (i32, [vp, i32, i32, i32, C.POINTER(f32), C.POINTER(f32), vp, i32, vp]),
    "ff_fill_cls": (i32, [vp, vp, i32, i32, i32, vp]),
    "ff_layernorm": (i32, [vp, i64, vp, vp, f32, i32, i32, vp, vp]),
    "ff_topk": (i32, [vp, i32, i32, i32, vp, vp, vp]),
    "ff_tree_pool": (i32, [C.POINTER(ModelConfig), C.POINTER(ModelWeights), vp, i32, vp, i64, vp, vp]),
    "ff_resize_pad": (i32, [vp, i32, i32, i32, i32, i32, i32, i32, vp, vp, i64, vp]),
    "ff_letterbox_aa_f16": (i32, [vp, i32, i32, i32, i32, i32, vp, vp]),
    "ff_patchify_windowed": (i32, [vp, i32, i32, i32, C.POINTER(f32), C.POINTER(f32), vp, i32, i32, vp]),
    "ff_layernorm_pos": (i32, [vp, i64, vp, vp, f32, i32, i32, vp, i32, vp, vp]),
    "ff_pool_query_attention": (i32, [vp, vp, i32, i32, i32, vp, vp]),
    "ff_resize_pad_workspace_bytes": (i64, [i32, i32, i32, i32, i32]),
    "ff_tree_pool_workspace_bytes": (i64, [C.POINTER(ModelConfig), i32]),
    "ff_engine_create": (i32, [C.POINTER(ModelConfig), C.POINTER(ModelWeights), i32, C.POINTER(vp)]),
    "ff_engine_forward": (i32, [vp, vp, i32, vp, vp, vp, vp]),
    "ff_engine_forward_eager": (i32, [vp, vp, i32, vp, vp, vp, vp]),
    "ff_engine_forward_pixels": (i32, [vp, vp, i32, vp, vp, vp, i32, vp]),
    "ff_engine_workspace_bytes": (i64, [C.POINTER(ModelConfig), i32]),
    "ff_engine_profile": (i32, [vp, vp, i32, i32, C.POINTER(f32), C.POINTER(i32), vp]),
    "ff_engine_launches_per_forward": (i32, [C.POINTER(ModelConfig)]),
    "ff_engine_destroy": (i32, [vp]),
}


def exported_symbols() -> list[str]:
    """Every entry point the C header declares (kept in sync by tests/test_capi.py)."""
    return sorted(_SIGNATURES)


@cache
def lib() -> C.CDLL:
    path = Path(os.environ.get("FOIDFINDER_B200_LIB", LIB_PATH))
    if not path.is_file():
        raise RuntimeError(
            f"foidfinder_b200 kernel library not found at {path}; build it with `python -m foidfinder_b200.build`"
        )
    handle = C.CDLL(str(path), mode=C.RTLD_LOCAL)
    for name, (res, args) in _SIGNATURES.items():
        fn = getattr(handle, name)
        fn.restype = res
        fn.argtypes = args
    return handle


class KernelError(RuntimeError):
    pass


def check(rc: int, what: str = "") -> None:
    """Maps a non-zero status to KernelError with the library's message (the reference's TORCH_CHECK role)."""
    if rc != FF_OK:
        msg = lib().ff_last_error().decode(errors="replace")
        raise KernelError(f"{what or 'foidfinder_b200'}: {STATUS.get(rc, rc)}: {msg}")


def device_error(device: int, clear: bool = True) -> int:
    code = i32(0)
    check(lib().ff_device_error(device, C.byref(code), int(clear)), "ff_device_error")
    return code.value
