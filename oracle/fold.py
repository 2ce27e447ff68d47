"""Oracle restatement of the Haruka checkpoint folding (foidfinder/haruka.py:40-61) — test
infrastructure only. Covers what the EVA02 engine's weight layout depends on: the patch embedding over
(kh, kw, c)-ordered raw pixels with the ImageNet normalisation folded in (haruka.py:40-46), the class
token and position embedding split (haruka.py:45-46), the fused qkv with the attention scale in the
q rows and a zero k bias plus the fused gate|up matrix (haruka.py:48-61), and the tree pool's tensors
with the 1/sqrt(pool head dim) logit scale in the key rows (haruka.py:71-88).
"""

from __future__ import annotations

import numpy as np

IMAGENET_MEAN = np.array([0.485, 0.456, 0.406], np.float32)
IMAGENET_STD = np.array([0.229, 0.224, 0.225], np.float32)


def fold(sd: dict[str, np.ndarray], dim: int, heads: int, patch: int, depth: int,
         pool_heads: int = 16) -> dict[str, np.ndarray]:
    bb = "backbone."
    w = sd[bb + "patch_embed.proj.weight"].transpose(0, 2, 3, 1)
    b = sd[bb + "patch_embed.proj.bias"] - (w * (IMAGENET_MEAN / IMAGENET_STD)).sum(axis=(1, 2, 3))
    pos = sd[bb + "pos_embed"][0]
    out = {
        "patch_w": (w / (255.0 * IMAGENET_STD)).reshape(dim, patch * patch * 3),
        "cls": sd[bb + "cls_token"].reshape(1, dim) + pos[:1],
        "patch_b": b + pos[1:],
    }
    scale = (dim // heads) ** -0.5
    for i in range(depth):
        a, m = f"{bb}blocks.{i}.attn.", f"{bb}blocks.{i}.mlp."
        out[f"blocks.{i}.qkv.weight"] = np.concatenate(
            [sd[a + "q_proj.weight"] * scale, sd[a + "k_proj.weight"], sd[a + "v_proj.weight"]]
        )
        out[f"blocks.{i}.qkv.bias"] = np.concatenate(
            [sd[a + "q_proj.bias"] * scale, np.zeros(dim, np.float32), sd[a + "v_proj.bias"]]
        )
        out[f"blocks.{i}.fc1.weight"] = np.concatenate([sd[m + "fc1_g.weight"], sd[m + "fc1_x.weight"]])
        out[f"blocks.{i}.fc1.bias"] = np.concatenate([sd[m + "fc1_g.bias"], sd[m + "fc1_x.bias"]])
    hp = "head_pool."
    if hp + "kv.weight" in sd:
        ps = (dim // pool_heads) ** -0.5
        wk, wv = np.split(sd[hp + "kv.weight"], 2)
        bk, bv = np.split(sd[hp + "kv.bias"], 2)
        out["pool.kv.weight"] = np.concatenate([wk * ps, wv])
        out["pool.kv.bias"] = np.concatenate([bk * ps, bv])
        for name in ("norm", "trunk_norm", "child_q_norm", "leaf_norm"):
            out[f"pool.{name}.weight"], out[f"pool.{name}.bias"] = sd[hp + name + ".weight"], sd[hp + name + ".bias"]
        out["pool.q_coarse"] = sd[hp + "q_coarse"].reshape(-1, dim)
        out["pool.q_coarse_bias"] = sd[hp + "q_coarse_bias"].reshape(-1)
        out["pool.q_child"] = sd[hp + "q_child"].reshape(-1, dim)
        out["pool.q_child_bias"] = sd[hp + "q_child_bias"].reshape(-1)
        out["pool.leaf.weight"] = sd[hp + "leaf_proj_weight"]
        out["pool.leaf.bias"] = sd[hp + "leaf_proj_bias"]
    return out
