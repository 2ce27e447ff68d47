"""Checkpoint handling: synthetic EVA02 and PixAI weights, RoPE tables, and the int8 conversion the kernels read.

`convert` plays the role of the reference's `convert_checkpoint` (foidfinder/backends/cuda/engine.py:49-62):
each block linear becomes `<name>.qweight` (int8, W' = W · blockdiag(H_n)), `<name>.wscale` (f32 per
output channel, `quantize_rows_int8`, engine.py:37-41) and `<name>.bias` (f32). On top of the reference
it lays the weights out for the sm_100a kernels:
- gate|up rows interleaved in groups of 64 ([gate 64 | up 64] per 128 rows) so one GEMM tile holds
  matching gate and up columns and the SwiGLU runs in the epilogue;
- the SwiGLU width padded (2730 -> 2816) with zero rows/columns so every GEMM K is a multiple of 128;
- head rows padded to a multiple of 256 tags; patch-embedding columns padded to a multiple of 64.

The raw layout is the folded one foidfinder/haruka.py:fold writes (q rows and bias pre-scaled by
head_dim**-0.5, zero k bias, fused qkv and gate|up matrices, patch bias + position embedding).
"""

from __future__ import annotations

import math

import numpy as np
import torch

from .config import ModelConfig

LINEARS = ("qkv", "proj", "fc1", "fc2")


def rope_tables(grid: int, ref_grid: int, head_dim: int = 64) -> tuple[torch.Tensor, torch.Tensor]:
    """EVA02 2-D RoPE (timm RotaryEmbeddingCat as restated in foidfinder/backends/mlx/haruka.py:22-33):
    axial bands, positions t / grid * ref_grid, y bands then x bands, interleaved pairs, class token
    (row 0) unrotated. Returns per-pair cos/sin [1 + grid*grid, head_dim/2] f32."""
    nb = head_dim // 4
    bands = 1.0 / (10000.0 ** (np.arange(nb, dtype=np.float32) / nb))
    t = np.arange(grid, dtype=np.float32) / grid * ref_grid
    ty, tx = np.meshgrid(t, t, indexing="ij")
    ang = np.concatenate([ty.reshape(-1, 1) * bands, tx.reshape(-1, 1) * bands], axis=1)  # [N, head_dim/2]
    cos = np.concatenate([np.ones((1, head_dim // 2), np.float32), np.cos(ang)]).astype(np.float32)
    sin = np.concatenate([np.zeros((1, head_dim // 2), np.float32), np.sin(ang)]).astype(np.float32)
    return torch.from_numpy(cos), torch.from_numpy(sin)


def random_raw(cfg: ModelConfig, seed: int = 0, device: str | torch.device = "cpu") -> dict[str, torch.Tensor]:
    """Seeded random-init weights in the folded layout: linear weights, position/class embeddings and
    biases ~ N(0, 0.02); LayerNorm weight 1 + N(0, 0.02), bias N(0, 0.02)."""
    g = torch.Generator(device=device).manual_seed(seed)
    D, H, P = cfg.dim, cfg.mlp_hidden, cfg.patches

    def n(*shape, std=0.02):
        return torch.randn(*shape, generator=g, device=device) * std

    raw = {
        "patch_w": n(D, cfg.k_patch),
        "patch_b": n(D),
        "pos_embed": n(P + 1, D),
        "cls_token": n(D),
        "norm.weight": 1.0 + n(D),
        "norm.bias": n(D),
        "head.weight": n(cfg.num_tags, cfg.head_in),
        "head.bias": n(cfg.num_tags),
    }
    if cfg.head == "tree":
        raw.update(random_pool(cfg, n))
    q_scale = cfg.head_dim**-0.5
    for i in range(cfg.depth):
        p = f"blocks.{i}."
        qkv_w, qkv_b = n(3 * D, D), n(3 * D)
        qkv_w[:D] *= q_scale  # attention scale folded into q (haruka.py:48-57)
        qkv_b[:D] *= q_scale
        qkv_b[D : 2 * D] = 0.0
        raw.update(
            {
                p + "norm1.weight": 1.0 + n(D),
                p + "norm1.bias": n(D),
                p + "qkv.weight": qkv_w,
                p + "qkv.bias": qkv_b,
                p + "proj.weight": n(D, D),
                p + "proj.bias": n(D),
                p + "norm2.weight": 1.0 + n(D),
                p + "norm2.bias": n(D),
                p + "fc1.weight": n(2 * H, D),  # gate rows then up rows (haruka.py:58-59)
                p + "fc1.bias": n(2 * H),
                p + "mlp_norm.weight": 1.0 + n(H),
                p + "mlp_norm.bias": n(H),
                p + "fc2.weight": n(D, H),
                p + "fc2.bias": n(D),
            }
        )
    return raw


def random_pool(cfg: ModelConfig, n) -> dict[str, torch.Tensor]:
    """Tree-pool weights in the folded layout (foidfinder/haruka.py:fold:66-80). Linear weights and biases
    ~ N(0, 0.02) (key rows then scaled by pool_head_dim^-0.5 as the folding does); LayerNorm weights
    1 + N(0, 0.02); the learned queries ~ N(0, 1) (the scale of trained query embeddings, so the slot
    softmax is not uniform); query biases -2 + N(0, 0.02) (the model card's initial value)."""
    D, C, Qn, L = cfg.dim, cfg.coarse_queries, cfg.leaf_queries, cfg.leaf_dim
    kv_w, kv_b = n(2 * D, D), n(2 * D)
    scale = (D // cfg.pool_heads) ** -0.5
    kv_w[:D] *= scale
    kv_b[:D] *= scale
    out = {"pool.kv.weight": kv_w, "pool.kv.bias": kv_b}
    for nm in ("norm", "trunk_norm", "child_q_norm", "leaf_norm"):
        out[f"pool.{nm}.weight"], out[f"pool.{nm}.bias"] = 1.0 + n(D), n(D)
    out["pool.q_coarse"], out["pool.q_coarse_bias"] = n(C, D, std=1.0), -2.0 + n(C)
    out["pool.q_child"], out["pool.q_child_bias"] = n(Qn, D, std=1.0), -2.0 + n(Qn)
    out["pool.leaf.weight"], out["pool.leaf.bias"] = n(Qn, D, L), n(Qn, L)
    return out


def hadamard(n: int, device: str | torch.device = "cpu") -> torch.Tensor:
    """Normalised Sylvester Hadamard matrix H_n / sqrt(n) as float32 (engine.py:29-34): built in float64 by
    doubling, divided by sqrt(n) in float64, then rounded once to float32."""
    h = torch.ones(1, 1, dtype=torch.float64)
    while h.shape[0] < n:
        h = torch.cat([torch.cat([h, h], 1), torch.cat([h, -h], 1)], 0)
    return (h / math.sqrt(n)).to(device=device, dtype=torch.float32)


_ROT_CACHE: dict[tuple[int, int, str], torch.Tensor] = {}


def rotate_rows(w: torch.Tensor, block: int) -> torch.Tensor:
    """w [N, K] -> w · blockdiag(H_block) as convert_checkpoint computes it (engine.py:58-60): one float32
    matmul by the full K x K block-diagonal matrix on w's device. The same torch call on the same device
    gives the reference's float32 sums bit for bit, so the int8 codes derived from them are the
    reference's codes, ties included (a shorter per-block product or an FWHT rounds differently)."""
    K = w.shape[1]
    key = (K, block, str(w.device))
    rot = _ROT_CACHE.get(key)
    if rot is None:
        rot = torch.block_diag(*[hadamard(block, w.device)] * (K // block))
        _ROT_CACHE.clear()  # keep one matrix (K = 2816 or 4864 takes 32-95 MB)
        _ROT_CACHE[key] = rot
    return w.float() @ rot


def quantize_rows_int8(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Symmetric per-output-channel int8 (engine.py:37-41)."""
    scale = w.abs().amax(1).clamp_min(1e-12) / 127.0
    q = torch.round(w / scale[:, None]).clamp(-127, 127).to(torch.int8)
    return q.contiguous(), scale.float().contiguous()


def interleave_gate_up(w: torch.Tensor, hidden: int, hidden_pad: int) -> torch.Tensor:
    """[gate (hidden) ; up (hidden)] rows -> [gate 64 | up 64] groups over hidden_pad (zero padding)."""
    rest = w.shape[1:]
    gate = torch.zeros(hidden_pad, *rest, dtype=w.dtype, device=w.device)
    up = torch.zeros_like(gate)
    gate[:hidden], up[:hidden] = w[:hidden], w[hidden:]
    return torch.stack([gate.view(hidden_pad // 64, 64, *rest), up.view(hidden_pad // 64, 64, *rest)], 1).reshape(
        2 * hidden_pad, *rest
    )


def convert(raw: dict[str, torch.Tensor], cfg: ModelConfig, device: str | torch.device | None = None) -> dict[str, torch.Tensor]:
    """Folded fp32 weights -> the engine format on `device` (default: where raw lives)."""
    dev = torch.device(device) if device is not None else raw["patch_w"].device
    D, H, Hp = cfg.dim, cfg.mlp_hidden, cfg.mlp_hidden_pad
    out: dict[str, torch.Tensor] = {}

    def put(name: str, t: torch.Tensor) -> None:
        out[name] = t.to(dev).contiguous()

    pw = torch.zeros(D, cfg.k_pad, device=raw["patch_w"].device)
    pw[:, : cfg.k_patch] = raw["patch_w"].float()
    put("patch_w", pw.half())
    pos = raw["pos_embed"].float()
    put("pos_bias", raw["patch_b"].float()[None, :] + pos[1:])
    put("cls_row", (raw["cls_token"].float() + pos[0]).half())
    cos, sin = rope_tables(cfg.grid, cfg.rope_ref_grid, cfg.head_dim)
    put("rope_cos", cos.t())  # angle-major [32, tokens], the QKV epilogue's layout
    put("rope_sin", sin.t())
    put("norm.weight", raw["norm.weight"].float())
    put("norm.bias", raw["norm.bias"].float())
    hw = torch.zeros(cfg.num_tags_pad, cfg.head_in, device=raw["head.weight"].device)
    hw[: cfg.num_tags] = raw["head.weight"].float()
    hb = torch.zeros(cfg.num_tags_pad, device=hw.device)
    hb[: cfg.num_tags] = raw["head.bias"].float()
    put("head.weight", hw.half())
    put("head.bias", hb)
    if cfg.head == "tree":
        for k, v in raw.items():
            if k.startswith("pool."):
                put(k, v.half() if k == "pool.kv.weight" else v.float())
    for i in range(cfg.depth):
        p = f"blocks.{i}."
        for n in ("norm1", "norm2"):
            put(p + n + ".weight", raw[p + n + ".weight"].float())
            put(p + n + ".bias", raw[p + n + ".bias"].float())
        mw = torch.zeros(Hp, device=hw.device)
        mb = torch.zeros(Hp, device=hw.device)
        mw[:H], mb[:H] = raw[p + "mlp_norm.weight"].float(), raw[p + "mlp_norm.bias"].float()
        put(p + "mlp_norm.weight", mw)
        put(p + "mlp_norm.bias", mb)
        lin = {
            "qkv": (raw[p + "qkv.weight"].float(), raw[p + "qkv.bias"].float(), cfg.rot_block_dim),
            "proj": (raw[p + "proj.weight"].float(), raw[p + "proj.bias"].float(), cfg.rot_block_dim),
            "fc1": (
                interleave_gate_up(raw[p + "fc1.weight"].float(), H, Hp),
                interleave_gate_up(raw[p + "fc1.bias"].float()[:, None], H, Hp)[:, 0],
                cfg.rot_block_dim,
            ),
            "fc2": (
                torch.nn.functional.pad(raw[p + "fc2.weight"].float(), (0, Hp - H)),
                raw[p + "fc2.bias"].float(),
                cfg.rot_block_hidden,
            ),
        }
        for name, (w, b, block) in lin.items():
            q, s = quantize_rows_int8(rotate_rows(w, block))
            put(f"{p}{name}.qweight", q)
            put(f"{p}{name}.wscale", s)
            put(f"{p}{name}.bias", b.contiguous())
    return out


def synthetic(cfg: ModelConfig, seed: int = 0, device: str | torch.device = "cuda") -> dict[str, torch.Tensor]:
    """Random-init model converted to the engine format, generated on `device`."""
    if cfg.arch == "pixai":
        return convert_pixai(pixai_random_raw(cfg, seed, device), cfg, device)
    return convert(random_raw(cfg, seed, device), cfg, device)


# ---------------------------------------------------------------- PixAI Tagger v1.0


def window_order(grid: int, window: int) -> torch.Tensor:
    """Position i of the window-ordered token sequence -> its row-major grid index: windows row-major, the
    window's patches row-major inside (foidfinder/backends/cuda/reference.py:21-24)."""
    nw = grid // window
    wr, wc, r, c = torch.meshgrid(*(torch.arange(n) for n in (nw, nw, window, window)), indexing="ij")
    return ((wr * window + r) * grid + wc * window + c).reshape(-1)


def axial_rope(end: int, scale: float, head_dim: int = 64) -> tuple[torch.Tensor, torch.Tensor]:
    """PixAI's axial 2-D RoPE (reference.py:27-34): for position t of an end x end grid, the head_dim/4
    frequencies times x = (t % end) * scale, then times y = (t // end) * scale. cos/sin [end^2, head_dim/2] f32."""
    freqs = 1.0 / (10000.0 ** (torch.arange(0, head_dim, 4)[: head_dim // 4].float() / head_dim))
    t = torch.arange(end * end, dtype=torch.float32)
    tx = (t % end) * scale
    ty = torch.div(t, end, rounding_mode="floor") * scale
    ang = torch.cat([torch.outer(tx, freqs), torch.outer(ty, freqs)], dim=-1)
    return torch.cos(ang), torch.sin(ang)


def pixai_random_raw(cfg: ModelConfig, seed: int = 0, device: str | torch.device = "cpu",
                     pre_grid: int | None = None) -> dict[str, torch.Tensor]:
    """Seeded random-init weights under the official PixAI checkpoint's names and shapes (the tensors
    reference.py:68-98 reads). Linear weights, biases and embeddings ~ N(0, 0.02), LayerNorm weights
    1 + N(0, 0.02); the pool's learned query ~ N(0, 1) so its softmax is not uniform. pre_grid: the
    pretraining grid of pos_embed (24 for the real checkpoint; it must divide the grid)."""
    g = torch.Generator(device=device).manual_seed(seed)
    D, H, G, p = cfg.dim, cfg.mlp_hidden, cfg.grid, cfg.patch
    pre = pre_grid or (24 if G % 24 == 0 else G)

    def n(*shape, std=0.02):
        return torch.randn(*shape, generator=g, device=device) * std

    raw = {
        "patch_embed.proj.weight": n(D, 3, p, p),
        "pos_embed": n(1, 1 + pre * pre, D),
        "ln_pre.weight": 1.0 + n(D),
        "ln_pre.bias": n(D),
        "head_pool.norm.weight": 1.0 + n(D),
        "head_pool.norm.bias": n(D),
        "head_pool.pos_embed": n(cfg.patches, D),
        "head_pool.q": n(1, 1, D, std=1.0),
        "head_pool.kv.weight": n(2 * D, D),
        "head_pool.kv.bias": n(2 * D),
        "head_pool.proj.weight": n(D, D),
        "head_pool.proj.bias": n(D),
        "head.weight": n(cfg.num_tags, D),
        "head.bias": n(cfg.num_tags),
    }
    for i in range(cfg.depth):
        b = f"blocks.{i}."
        raw.update({
            b + "norm1.weight": 1.0 + n(D), b + "norm1.bias": n(D),
            b + "attn.qkv.weight": n(3 * D, D), b + "attn.qkv.bias": n(3 * D),
            b + "attn.proj.weight": n(D, D), b + "attn.proj.bias": n(D),
            b + "norm2.weight": 1.0 + n(D), b + "norm2.bias": n(D),
            b + "mlp.fc1.weight": n(H, D), b + "mlp.fc1.bias": n(H),
            b + "mlp.fc2.weight": n(D, H), b + "mlp.fc2.bias": n(D),
        })
    return raw


# Quantised block linears of the PixAI checkpoint -> which Hadamard block rotates their input (engine.py:45:
# H1024 for the dim-wide inputs, H128 for the hidden; ModelConfig.rot_block_dim / rot_block_hidden).
PIXAI_QUANTIZED = {"attn.qkv": "dim", "attn.proj": "dim", "mlp.fc1": "dim", "mlp.fc2": "hidden"}
PIXAI_INT8_FORMAT = "foidfinder-pixai-int8-v1"  # the reference's `foidfinder convert` output (engine.py:46)


def is_pixai_int8(raw: dict) -> bool:
    """True for the reference's converted checkpoint (PixAICuda.__init__'s test, engine.py:71)."""
    return "blocks.0.attn.qkv.qweight" in raw


def pixai_convert_checkpoint(raw: dict[str, torch.Tensor], cfg: ModelConfig) -> dict[str, torch.Tensor]:
    """Official fp32 PixAI state dict -> the reference's int8 checkpoint (convert_checkpoint,
    foidfinder/backends/cuda/engine.py:49-62): every block linear becomes `.qweight` (int8 codes of
    W · blockdiag(H) computed as one float32 matmul on the tensor's device, per-output-channel scale),
    `.wscale` (f32) and `.bias` (f32); every other tensor is passed through. Same tensor names, same codes."""
    out = {k: v for k, v in raw.items() if not any(f".{n}." in k for n in PIXAI_QUANTIZED)}
    for i in range(cfg.depth):
        for name, which in PIXAI_QUANTIZED.items():
            block = cfg.rot_block_dim if which == "dim" else cfg.rot_block_hidden
            p = f"blocks.{i}.{name}"
            out[p + ".qweight"], out[p + ".wscale"] = quantize_rows_int8(rotate_rows(raw[p + ".weight"].float(), block))
            out[p + ".bias"] = raw[p + ".bias"].float().contiguous()
    return out


def convert_pixai(raw: dict[str, torch.Tensor], cfg: ModelConfig,
                  device: str | torch.device | None = None) -> dict[str, torch.Tensor]:
    """Official PixAI fp32 checkpoint, or the reference's int8 checkpoint (`foidfinder convert`, format
    foidfinder-pixai-int8-v1), -> the engine format. The fp32 form is first quantised exactly as
    `convert_checkpoint` does (`pixai_convert_checkpoint`), so both sources give identical engine weights.

    From the int8 checkpoint: `.qweight` codes are used unchanged. The attention scale 1/sqrt(64) of
    F.scaled_dot_product_attention (reference.py:125), which the reference applies in its QKV epilogue
    (engine.py:26), is folded into the q rows' `.wscale` and `.bias`: a power of two, so the product equals
    the reference's scaled output. The hidden is padded to mlp_hidden_pad (4736 -> 4864) with zero fc1
    rows (zero codes and bias) and zero fc2 columns (one extra all-zero H128 block), so fc1 runs on
    256-wide tiles; the padding stays exactly zero through GELU and the H128 rotation.
    The stem and tables follow PixAITorch.__init__ (reference.py:70-98): patch weight in (kh, kw, c)
    column order, the pretraining position embedding tiled over the grid and put in window order, window
    and global RoPE tables (the global one at positions scaled by window / grid, window-ordered), stored
    angle-major [32, n]; the pool's position embedding in window order and its query carrying the 1/8
    scale. The patch embedding's bias, if the checkpoint has one, is not used — the reference's stem has
    none (reference.py:112)."""
    if not is_pixai_int8(raw):
        raw = pixai_convert_checkpoint(raw, cfg)
    dev = torch.device(device) if device is not None else raw["pos_embed"].device
    D, G, L, win, H, Hp = cfg.dim, cfg.grid, cfg.patches, cfg.window, cfg.mlp_hidden, cfg.mlp_hidden_pad
    src = raw["pos_embed"].device
    perm = window_order(G, win).to(src)
    out: dict[str, torch.Tensor] = {}

    def put(name: str, t: torch.Tensor) -> None:
        out[name] = t.to(dev).contiguous()

    pw = torch.zeros(D, cfg.k_pad, device=src)
    pw[:, : cfg.k_patch] = raw["patch_embed.proj.weight"].float().permute(0, 2, 3, 1).reshape(D, -1)
    put("patch_w", pw.half())
    pos = raw["pos_embed"].float()[0, 1:]
    pre = math.isqrt(pos.shape[0])
    put("pos_bias", pos.reshape(pre, pre, D).repeat(G // pre, G // pre, 1).reshape(L, D)[perm])
    put("ln_pre.weight", raw["ln_pre.weight"].float())
    put("ln_pre.bias", raw["ln_pre.bias"].float())
    cw, sw = axial_rope(win, 1.0, cfg.head_dim)
    cg, sg = axial_rope(G, win / G, cfg.head_dim)
    put("rope_cos", cw.t())
    put("rope_sin", sw.t())
    put("rope_cos_global", cg[perm.cpu()].t())
    put("rope_sin_global", sg[perm.cpu()].t())
    scale = cfg.head_dim**-0.5
    put("pool.norm.weight", raw["head_pool.norm.weight"].float())
    put("pool.norm.bias", raw["head_pool.norm.bias"].float())
    put("pool.pos", raw["head_pool.pos_embed"].float()[perm].half())
    put("pool.q", raw["head_pool.q"].float().reshape(D) * scale)
    put("pool.kv.weight", raw["head_pool.kv.weight"].half())
    put("pool.kv.bias", raw["head_pool.kv.bias"].float())
    put("pool.proj.weight", raw["head_pool.proj.weight"].half())
    put("pool.proj.bias", raw["head_pool.proj.bias"].float())
    hw = torch.zeros(cfg.num_tags_pad, D, device=src)
    hw[: cfg.num_tags] = raw["head.weight"].float()
    hb = torch.zeros(cfg.num_tags_pad, device=src)
    hb[: cfg.num_tags] = raw["head.bias"].float()
    put("head.weight", hw.half())
    put("head.bias", hb)
    pad_scale = torch.tensor(1e-12 / 127.0)  # what quantize_rows_int8 gives an all-zero row
    for i in range(cfg.depth):
        p = f"blocks.{i}."
        for n in ("norm1", "norm2"):
            put(p + n + ".weight", raw[p + n + ".weight"].float())
            put(p + n + ".bias", raw[p + n + ".bias"].float())

        def q(name: str):
            return (raw[f"{p}{name}.qweight"], raw[f"{p}{name}.wscale"].float().clone(),
                    raw[f"{p}{name}.bias"].float().clone())

        qw, qs, qb = q("attn.qkv")
        qs[:D] *= scale
        qb[:D] *= scale
        f1w, f1s, f1b = q("mlp.fc1")
        f1w = torch.nn.functional.pad(f1w, (0, 0, 0, Hp - H))
        f1s = torch.cat([f1s, pad_scale.to(f1s).expand(Hp - H)])
        f1b = torch.nn.functional.pad(f1b, (0, Hp - H))
        f2w, f2s, f2b = q("mlp.fc2")
        f2w = torch.nn.functional.pad(f2w, (0, Hp - H))
        for name, (w_, s_, b_) in {"qkv": (qw, qs, qb), "proj": q("attn.proj"), "fc1": (f1w, f1s, f1b),
                                   "fc2": (f2w, f2s, f2b)}.items():
            put(f"{p}{name}.qweight", w_.to(torch.int8))
            put(f"{p}{name}.wscale", s_)
            put(f"{p}{name}.bias", b_)
    return out


def from_folded(folded: dict, cfg: ModelConfig, device: str | torch.device = "cpu") -> dict[str, torch.Tensor]:
    """The folded checkpoint foidfinder/haruka.py:fold writes (`patch_b` [patches, dim] with the position
    embedding added, `cls` [1, dim] = class token + pos[0]; blocks in the same names as this module's raw
    layout) -> the raw layout `convert` takes. Pool-head tensors (`pool.*`) are passed through."""
    t = {k: torch.as_tensor(v).float().to(device) for k, v in folded.items()}
    if "pos_embed" in t:
        return t
    D = cfg.dim
    raw = dict(t)
    raw["pos_embed"] = torch.cat([torch.zeros(1, D, device=device), t["patch_b"].reshape(cfg.patches, D)])
    raw["patch_b"] = torch.zeros(D, device=device)
    raw["cls_token"] = t["cls"].reshape(D)
    del raw["cls"]
    return raw
