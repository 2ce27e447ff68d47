"""Generates tests/golden/reference_vectors.npz by running the reference's own Python functions.

Run where the reference project is importable (it is not needed at test time):

    python tests/golden/make_golden.py /path/to/foidfinder-reference

What it records (inputs are seeded; every function is the reference's, unmodified):
- `foidfinder.backends.cuda.engine.hadamard(128)` and `(1024)` sign patterns (bit-packed) and scale;
- `quantize_rows_int8` on a seeded matrix;
- `convert_checkpoint` on a seeded one-block checkpoint (its block count, `DEPTH`, is set to 1 for the
  call; the four block linears keep the reference's K and rotation sizes);
- `apply_rope` of `foidfinder.backends.cuda.reference` on seeded x with `axial_rope(24, 1.0)` tables
  (the interleaved-pair rotation convention);
- `rope_tables(32, 16, 64)` of `foidfinder/backends/mlx/haruka.py` (the EVA02 RoPE), executed from the
  function's source text because that module imports MLX at load time;
- `foidfinder.haruka.fold` on a seeded tiny timm-style checkpoint (model dims shrunk through its
  `MODEL` dict): the folded patch embedding (pixel normalisation inside the weights), the fused qkv with
  the q scale and zero k bias, and the tree-pool tensors (key rows scaled);
- the model card's tree attention pool `MHAttnPool` (defined inside the `haruka` fixture of
  `tests/test_haruka.py`, executed from its source text) on seeded tokens with the same checkpoint;
- `PixAITorch` of `foidfinder.backends.cuda.reference` (f32, CPU) on a seeded tiny PixAI checkpoint under
  the official tensor names: the whole forward (window-ordered patchify, tiled position embedding, ln_pre,
  window and global blocks with their RoPE tables, GELU MLP, attention-pool head) on seeded images, and
  `pool_head` alone on seeded tokens. The module's shape constants are set to the tiny model (`PIXAI`)
  for the call and restored after.
"""

from __future__ import annotations

import ast
import sys
from pathlib import Path

import numpy as np


TREE = {"dim": 64, "pool_heads": 4, "coarse": 6, "leaves": 18, "leaf_dim": 8, "tokens": 9, "images": 2}
CONV_SHAPES = {"attn.qkv": (24, 1024), "attn.proj": (8, 1024), "mlp.fc1": (16, 1024), "mlp.fc2": (8, 256)}
EVA_ROPE_ROWS = np.r_[0:40, 40:1025:37, 1024]


def inputs() -> dict[str, np.ndarray]:
    """Seeded inputs (numpy's PCG64 stream is stable across versions, so tests regenerate them)."""
    rng = np.random.default_rng(1234)
    inp = {"quant_in": (rng.standard_normal((64, 256)) * 0.02).astype(np.float32)}
    for name, shape in CONV_SHAPES.items():
        inp[f"conv_{name}_w"] = (rng.standard_normal(shape) * 0.02).astype(np.float32)
    inp["rope_in"] = rng.standard_normal((1, 1, 576, 64)).astype(np.float32)
    return inp


def main(ref_root: str) -> None:
    sys.path.insert(0, ref_root)
    import torch

    from foidfinder import haruka
    from foidfinder.backends.cuda import engine, reference

    out: dict[str, np.ndarray] = {}
    inp = inputs()

    for n in (128, 1024):
        h = engine.hadamard(n, "cpu")
        out[f"hadamard{n}_sign"] = np.packbits((h > 0).numpy())
        out[f"hadamard{n}_abs"] = np.float32(h.abs().max().item())

    q, s = engine.quantize_rows_int8(torch.from_numpy(inp["quant_in"]))
    out["quant_q"], out["quant_scale"] = q.numpy(), s.numpy()

    raw = {}
    for name in CONV_SHAPES:
        raw[f"blocks.0.{name}.weight"] = torch.from_numpy(inp[f"conv_{name}_w"])
        raw[f"blocks.0.{name}.bias"] = torch.zeros(CONV_SHAPES[name][0])
    saved_depth = engine.DEPTH
    engine.DEPTH = 1
    try:
        conv = engine.convert_checkpoint(raw)
    finally:
        engine.DEPTH = saved_depth
    for name in CONV_SHAPES:
        key = f"blocks.0.{name}"
        out[f"conv_{name}_qweight"] = conv[key + ".qweight"].numpy()
        out[f"conv_{name}_wscale"] = conv[key + ".wscale"].numpy()

    cos, sin = reference.axial_rope(24, 1.0)
    out["rope_out"] = reference.apply_rope(torch.from_numpy(inp["rope_in"]), cos, sin).numpy()

    src = (Path(ref_root) / "foidfinder/backends/mlx/haruka.py").read_text()
    fn = next(node for node in ast.parse(src).body if isinstance(node, ast.FunctionDef) and node.name == "rope_tables")
    ns: dict = {"np": np}
    exec(compile(ast.Module(body=[fn], type_ignores=[]), "haruka_rope_tables", "exec"), ns)
    ecos, esin = ns["rope_tables"](32, 16, 64)
    rows = EVA_ROPE_ROWS
    out["eva_rope_cos_even"] = ecos[rows, 0::2].astype(np.float32)
    out["eva_rope_sin_even"] = esin[rows, 0::2].astype(np.float32)
    out["eva_rope_pairs_equal"] = np.array(
        bool(np.array_equal(ecos[:, 0::2], ecos[:, 1::2]) and np.array_equal(esin[:, 0::2], esin[:, 1::2]))
    )
    out["eva_rope_checksum"] = np.array([ecos.astype(np.float64).sum(), esin.astype(np.float64).sum(), ecos.shape[0]])

    saved_model = dict(haruka.MODEL)
    haruka.MODEL.update(dim=64, heads=2, depth=1, pool_heads=TREE["pool_heads"])
    try:
        sd = fold_inputs()
        folded = haruka.fold(sd)
    finally:
        haruka.MODEL.clear()
        haruka.MODEL.update(saved_model)
    for k in FOLD_KEYS:
        out["fold_out_" + k.replace(".", "_")] = folded[k]

    # The model card's tree pool (MHAttnPool, defined inside the `haruka` fixture of tests/test_haruka.py),
    # executed from its source text with the same seeded weights.
    src = (Path(ref_root) / "tests/test_haruka.py").read_text()
    fixture = next(n for n in ast.parse(src).body if isinstance(n, ast.FunctionDef) and n.name == "haruka")
    cls_def = next(n for n in ast.walk(fixture) if isinstance(n, ast.ClassDef) and n.name == "MHAttnPool")
    ns = {"torch": torch, "nn": torch.nn}
    exec(compile(ast.Module(body=[cls_def], type_ignores=[]), "model_card_MHAttnPool", "exec"), ns)
    pool = ns["MHAttnPool"](dim=TREE["dim"], num_heads=TREE["pool_heads"], num_queries=TREE["leaves"],
                            leaf_dim=TREE["leaf_dim"])
    pool.load_state_dict({k[len("head_pool."):]: torch.from_numpy(v) for k, v in sd.items() if k.startswith("head_pool.")})
    with torch.no_grad():
        out["tree_leaf"] = pool(torch.from_numpy(tree_input())).numpy()

    # PixAI Tagger v1.0 (reference.py), shrunk through its module constants.
    px = PIXAI
    consts = {"S": px["S"], "P": px["P"], "C": px["C"], "H": px["H"], "DEPTH": px["DEPTH"], "WIN": px["WIN"],
              "G": px["S"] // px["P"], "NW": px["S"] // px["P"] // px["WIN"], "L": (px["S"] // px["P"]) ** 2,
              "LW": px["WIN"] ** 2, "GLOBAL": frozenset(px["GLOBAL"]), "PRE": px["PRE"]}
    saved = {k: getattr(reference, k) for k in consts}
    for k, v in consts.items():
        setattr(reference, k, v)
    try:
        sd = {k: torch.from_numpy(v) for k, v in pixai_checkpoint().items()}
        model = reference.PixAITorch(".", dtype=torch.float32, device="cpu", raw=sd)
        with torch.no_grad():
            out["pixai_logits"] = model(torch.from_numpy(pixai_pixels())).numpy()
            out["pixai_pool_logits"] = model.pool_head(torch.from_numpy(pixai_pool_input())).numpy()
    finally:
        for k, v in saved.items():
            setattr(reference, k, v)

    dst = Path(__file__).resolve().parent / "reference_vectors.npz"
    np.savez_compressed(dst, **out)
    print(f"wrote {dst} ({dst.stat().st_size} bytes, {len(out)} arrays)")


FOLD_KEYS = ("patch_w", "patch_b", "cls", "blocks.0.qkv.weight", "blocks.0.qkv.bias", "blocks.0.fc1.weight",
             "blocks.0.fc1.bias", "pool.kv.weight", "pool.kv.bias", "pool.q_coarse", "pool.q_coarse_bias",
             "pool.q_child", "pool.q_child_bias", "pool.leaf.weight", "pool.leaf.bias", "pool.trunk_norm.weight")


def tree_input() -> np.ndarray:
    """Seeded final-normed tokens [images, tokens, dim] for the tree pool."""
    rng = np.random.default_rng(11)
    return rng.standard_normal((TREE["images"], TREE["tokens"], TREE["dim"])).astype(np.float32)


def fold_inputs() -> dict[str, np.ndarray]:
    """A seeded tiny timm-style Haruka checkpoint: dim 64, 2 heads, 1 block, 4 patches."""
    rng = np.random.default_rng(7)
    D, p = 64, 14

    def r(*shape, std=0.02):
        return (rng.standard_normal(shape) * std).astype(np.float32)

    bb = "backbone."
    sd = {
        bb + "patch_embed.proj.weight": r(D, 3, p, p),
        bb + "patch_embed.proj.bias": r(D),
        bb + "pos_embed": r(1, 5, D),
        bb + "cls_token": r(1, 1, D),
        bb + "norm.weight": r(D),
        bb + "norm.bias": r(D),
        "head.weight": r(3, TREE["leaves"] * TREE["leaf_dim"]),
        "head.bias": r(3),
    }
    for nm in ("norm", "trunk_norm", "child_q_norm", "leaf_norm"):
        sd[f"head_pool.{nm}.weight"], sd[f"head_pool.{nm}.bias"] = 1.0 + r(D), r(D)
    C, Qn, L = TREE["coarse"], TREE["leaves"], TREE["leaf_dim"]
    sd.update({"head_pool.q_coarse": r(1, C, D, std=1.0), "head_pool.q_coarse_bias": -2.0 + r(1, 1, C, 1),
               "head_pool.q_child": r(1, C, Qn // C, D, std=1.0), "head_pool.q_child_bias": -2.0 + r(1, 1, Qn, 1),
               "head_pool.leaf_proj_weight": r(Qn, D, L, std=0.1), "head_pool.leaf_proj_bias": r(Qn, L),
               "head_pool.kv.weight": r(2 * D, D, std=0.2), "head_pool.kv.bias": r(2 * D)})
    a, m = bb + "blocks.0.attn.", bb + "blocks.0.mlp."
    for nm in ("q_proj", "k_proj", "v_proj", "proj"):
        sd[a + nm + ".weight"], sd[a + nm + ".bias"] = r(D, D), r(D)
    for nm in ("fc1_g", "fc1_x"):
        sd[m + nm + ".weight"], sd[m + nm + ".bias"] = r(96, D), r(96)
    sd[m + "fc2.weight"], sd[m + "fc2.bias"] = r(D, 96), r(D)
    sd[m + "norm.weight"], sd[m + "norm.bias"] = r(96), r(96)
    for nm in ("norm1", "norm2"):
        sd[bb + f"blocks.0.{nm}.weight"], sd[bb + f"blocks.0.{nm}.bias"] = r(D), r(D)
    return sd


PIXAI = {"S": 336, "P": 14, "C": 128, "H": 2, "DEPTH": 2, "WIN": 8, "GLOBAL": (1,), "PRE": 12, "hidden": 256,
         "tags": 50, "images": 2}


def pixai_checkpoint() -> dict[str, np.ndarray]:
    """A seeded tiny PixAI checkpoint under the official names (the tensors reference.py:68-98 reads)."""
    rng = np.random.default_rng(21)
    px = PIXAI
    C, Hd, p, L = px["C"], px["hidden"], px["P"], (px["S"] // px["P"]) ** 2

    def r(*shape, std=0.02, base=0.0):
        return (base + rng.standard_normal(shape) * std).astype(np.float32)

    sd = {
        "patch_embed.proj.weight": r(C, 3, p, p),
        "pos_embed": r(1, 1 + px["PRE"] ** 2, C, std=0.1),
        "ln_pre.weight": r(C, base=1.0), "ln_pre.bias": r(C),
        "head_pool.norm.weight": r(C, base=1.0), "head_pool.norm.bias": r(C),
        "head_pool.pos_embed": r(L, C, std=0.1), "head_pool.q": r(1, 1, C, std=1.0),
        "head_pool.kv.weight": r(2 * C, C, std=0.1), "head_pool.kv.bias": r(2 * C),
        "head_pool.proj.weight": r(C, C, std=0.1), "head_pool.proj.bias": r(C),
        "head.weight": r(px["tags"], C, std=0.1), "head.bias": r(px["tags"]),
    }
    for i in range(px["DEPTH"]):
        b = f"blocks.{i}."
        sd.update({
            b + "norm1.weight": r(C, base=1.0), b + "norm1.bias": r(C),
            b + "attn.qkv.weight": r(3 * C, C, std=0.1), b + "attn.qkv.bias": r(3 * C),
            b + "attn.proj.weight": r(C, C, std=0.1), b + "attn.proj.bias": r(C),
            b + "norm2.weight": r(C, base=1.0), b + "norm2.bias": r(C),
            b + "mlp.fc1.weight": r(Hd, C, std=0.1), b + "mlp.fc1.bias": r(Hd),
            b + "mlp.fc2.weight": r(C, Hd, std=0.1), b + "mlp.fc2.bias": r(C),
        })
    return sd


def pixai_images() -> np.ndarray:
    """Seeded uint8 images [images, S, S, 3]."""
    rng = np.random.default_rng(22)
    return rng.integers(0, 256, (PIXAI["images"], PIXAI["S"], PIXAI["S"], 3), dtype=np.uint8)


def pixai_pixels() -> np.ndarray:
    """The images normalised as the engine's patchify does: (u8 * f32(1/255) - 0.5) * (1 / 0.5), f32."""
    x = pixai_images().astype(np.float32) * np.float32(1.0 / 255.0)
    return ((x - np.float32(0.5)) * np.float32(2.0)).astype(np.float32)


def pixai_pool_input() -> np.ndarray:
    """Seeded window-ordered tokens [images, L, C] for the pool head alone."""
    rng = np.random.default_rng(23)
    return rng.standard_normal((PIXAI["images"], (PIXAI["S"] // PIXAI["P"]) ** 2, PIXAI["C"])).astype(np.float32)


if __name__ == "__main__":
    import os

    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("FOIDFINDER_REFERENCE")
    if not root:
        sys.exit("usage: make_golden.py /path/to/foidfinder-reference (or set FOIDFINDER_REFERENCE)")
    main(root)
