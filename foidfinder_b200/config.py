"""Model shapes the engine runs (a runtime struct rather than the reference's hard-coded constants,
foidfinder/backends/cuda/reference.py:12-17).

- EVA02_L: BASELINE config 0/3, "PixAI-shaped EVA02-L/14": 448 px, patch 14, 1024 patches + class token,
  24 blocks, dim 1024, 16 heads of 64, SwiGLU hidden 2730 with the EVA02 hidden LayerNorm, 2-D RoPE,
  final LayerNorm, class-token linear head to 30,877 tags, pixel mean/std 0.5.
- EVA02_B: the Haruka Tagger shape (foidfinder/haruka.py:13-27): dim 768, 12 blocks, 12 heads,
  hidden 2048, ImageNet mean/std, the tree attention pool head (16 pool heads, 6 coarse and 18 leaf
  queries, leaf dim 64; foidfinder/backends/mlx/haruka.py:104-136) and a linear head from the 1152 leaf
  features to 98,782 tags.
"""

from __future__ import annotations

from dataclasses import dataclass, replace

IMAGENET_MEAN = (0.485, 0.456, 0.406)
IMAGENET_STD = (0.229, 0.224, 0.225)


def _ceil(a: int, b: int) -> int:
    return (a + b - 1) // b * b


@dataclass(frozen=True)
class ModelConfig:
    name: str
    image_size: int = 448
    patch: int = 14
    dim: int = 1024
    depth: int = 24
    heads: int = 16
    mlp_hidden: int = 2730
    num_tags: int = 30877
    rope_ref_grid: int = 16
    ln_eps: float = 1e-6
    mean: tuple[float, float, float] = (0.5, 0.5, 0.5)
    std: tuple[float, float, float] = (0.5, 0.5, 0.5)
    rot_block_dim: int = 1024  # Hadamard block of the dim-wide GEMM inputs (qkv, proj, fc1)
    rot_block_hidden: int = 128  # Hadamard block of the hidden-wide GEMM input (fc2)
    topk: int = 50
    arch: str = "eva02"  # "eva02": class token, SwiGLU + hidden LN, EVA02 RoPE; "pixai": see PIXAI_1008
    window: int = 0  # window attention size in patches (0: every block global)
    global_blocks: tuple[int, ...] = ()  # blocks that attend over the whole image when window > 0
    resample: str = "bilinear"  # letterbox filter: PixAI's antialiased bilinear on black
    pad: int = 0  # letterbox canvas value
    head: str = "cls"  # "cls": class-token linear head; "tree": the Haruka tree attention pool; "pool": PixAI's
    # one-query attention pool (LN + position embedding -> kv -> attention -> proj)
    pool_heads: int = 16
    coarse_queries: int = 6
    leaf_queries: int = 18
    leaf_dim: int = 64

    @property
    def head_in(self) -> int:
        """K of the tag head: dim (class token, attention pool) or leaf_queries * leaf_dim (tree pool)."""
        return self.leaf_queries * self.leaf_dim if self.head == "tree" else self.dim

    @property
    def grid(self) -> int:
        return self.image_size // self.patch

    @property
    def patches(self) -> int:
        return self.grid * self.grid

    @property
    def cls_token(self) -> bool:
        return self.arch == "eva02"

    @property
    def tokens(self) -> int:
        return self.patches + (1 if self.cls_token else 0)

    def is_global(self, block: int) -> bool:
        return self.window == 0 or block in self.global_blocks

    @property
    def head_dim(self) -> int:
        return self.dim // self.heads

    @property
    def mlp_hidden_pad(self) -> int:
        """Hidden width the GEMMs run at: a multiple of 256 so the up-projection takes 256-wide tiles (zero
        rows/columns in the padding; 2730 -> 2816, 4736 -> 4864)."""
        return _ceil(self.mlp_hidden, 256)

    @property
    def num_tags_pad(self) -> int:
        return _ceil(self.num_tags, 256)

    @property
    def k_patch(self) -> int:
        return self.patch * self.patch * 3

    @property
    def k_pad(self) -> int:
        return _ceil(self.k_patch, 64)

    def gemm_ops_per_image(self, padded: bool = False) -> int:
        """Int8 multiply-adds x 2 of the four block GEMMs per image (qkv, proj, gate|up or fc1, down)."""
        h = self.mlp_hidden_pad if padded else self.mlp_hidden
        up = 2 * h if self.arch == "eva02" else h
        per_token = self.dim * 3 * self.dim + self.dim * self.dim + self.dim * up + h * self.dim
        return 2 * self.tokens * self.depth * per_token

    def attention_flops_per_image(self) -> int:
        total = 0
        for i in range(self.depth):
            n = self.tokens if self.is_global(i) else self.window * self.window
            total += 4 * self.heads * self.tokens * n * self.head_dim
        return total

    def with_(self, **kw) -> ModelConfig:
        return replace(self, **kw)


EVA02_L = ModelConfig("eva02-l-448")
EVA02_B = ModelConfig(
    "eva02-b-448",
    dim=768,
    depth=12,
    heads=12,
    mlp_hidden=2048,
    num_tags=98782,
    mean=IMAGENET_MEAN,
    std=IMAGENET_STD,
    rot_block_dim=256,
    resample="bicubic",  # the model card's preprocessing: bicubic, composited and padded on white
    pad=255,
    head="tree",
)

# The reference's real `cuda` workload, PixAI Tagger v1.0 (foidfinder/backends/cuda/reference.py:12-17):
# 1008 px, patch 14 -> 72 x 72 = 5184 tokens in window order (no class token), 32 blocks of dim 1024 with
# 24 x 24 windowed attention except blocks 7, 15, 23, 31 (global), axial 2-D RoPE, GELU MLP 4736,
# LayerNorm eps 1e-5 and an ln_pre after the stem, a one-query attention-pool head, 30,877 tags.
PIXAI_1008 = ModelConfig(
    "pixai-1008",
    image_size=1008,
    depth=32,
    mlp_hidden=4736,
    ln_eps=1e-5,
    rot_block_dim=1024,
    rot_block_hidden=128,
    arch="pixai",
    window=24,
    global_blocks=(7, 15, 23, 31),
    head="pool",
)

CONFIGS = {c.name: c for c in (EVA02_L, EVA02_B, PIXAI_1008)}
