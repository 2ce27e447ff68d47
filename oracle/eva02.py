"""Oracle EVA02 tagger forwards on the CPU — test infrastructure only.

Restates, in plain PyTorch:
- the EVA02 block of foidfinder/backends/mlx/haruka.py:74-102 (pre-LN, fused qkv with the attention
  scale folded into q, 2-D RoPE on q/k, SDPA with scale 1, SwiGLU + hidden LayerNorm, eps 1e-6);
- the RoPE tables of mlx/haruka.py:22-33 and the pair rotation of mlx/kernels.py:12-29;
- the patch embedding over (kh, kw, c)-ordered pixels (reference.py:103-107, mlx/haruka.py:78-79) with
  the class token first;
- the int8 pipeline of foidfinder/backends/cuda/engine.py:1-10 and :142-161: per-token Hadamard-rotated
  int8 activations before every block linear, exact int32 accumulation, per-channel dequantisation,
  and fp16 storage of the residual stream and of every inter-kernel activation (engine.py:96-106).

`forward_fp32` runs the unquantised folded weights; `forward_int8` consumes the converted checkpoint
(the same int8 tensors the GPU engine reads) and rounds to fp16 exactly where the kernels store fp16.
"""

from __future__ import annotations

import numpy as np
import torch

from . import quant as Q


def rope_tables(grid: int, ref: int, head_dim: int = 64) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-pair cos/sin [1 + grid^2, head_dim/2] (mlx/haruka.py:22-33: ang repeated per pair; row 0 is
    the class token's identity rotation)."""
    bands = 1.0 / (10000.0 ** (np.arange(head_dim // 4, dtype=np.float32) / (head_dim // 4)))
    t = np.arange(grid, dtype=np.float32) / grid * ref
    ty, tx = np.meshgrid(t, t, indexing="ij")
    ang = np.concatenate([ty.reshape(-1, 1) * bands, tx.reshape(-1, 1) * bands], axis=1)
    cos = np.concatenate([np.ones((1, head_dim // 2), np.float32), np.cos(ang)])
    sin = np.concatenate([np.zeros((1, head_dim // 2), np.float32), np.sin(ang)])
    return torch.from_numpy(cos.astype(np.float32)), torch.from_numpy(sin.astype(np.float32))


def patchify(images: torch.Tensor, patch: int, mean, std) -> torch.Tensor:
    """uint8 [B, S, S, 3] -> normalised f32 patches [B, G*G, p*p*3] in (kh, kw, c) order: u * f32(1/255) - mean
    rounded once to f32 (exact in f64 first, as a fused multiply-add), then times f32(1/std)."""
    B, S = images.shape[:2]
    G = S // patch
    m = torch.tensor(mean, dtype=torch.float32, device=images.device).double()
    x = (images.double() * float(np.float32(1.0 / 255.0)) - m).float()
    x = x * (1.0 / torch.tensor(std, dtype=torch.float32, device=images.device))
    x = x.view(B, G, patch, G, patch, 3).permute(0, 1, 3, 2, 4, 5)
    return x.reshape(B, G * G, patch * patch * 3)


def _attention(qkv: torch.Tensor, B: int, T: int, heads: int) -> torch.Tensor:
    """softmax(q k^T) v per head (scale already in q), f32 math, qkv [B*T, 3*dim] -> [B*T, dim]."""
    dim = heads * 64
    q, k, v = qkv.float().view(B, T, 3, heads, 64).permute(2, 0, 3, 1, 4)
    o = torch.softmax(q @ k.transpose(-1, -2), dim=-1) @ v
    return o.transpose(1, 2).reshape(B * T, dim)


def _rope_qk(qkv: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, T: int, dim: int) -> torch.Tensor:
    pos = torch.arange(qkv.shape[0]) % T
    return Q.apply_rope_pairs(qkv, cos, sin, pos, 2 * dim)


def forward_fp32(raw: dict[str, torch.Tensor], cfg, images: torch.Tensor) -> torch.Tensor:
    """fp32 EVA02 forward on the folded (unquantised) weights -> logits [B, num_tags], on
    the images' device. Written with the fused torch ops the reference's PyTorch forward uses
    (F.layer_norm, F.linear, F.scaled_dot_product_attention; reference.py:114-131), so that timing it on the
    CPU measures what the reference's own CPU path costs."""
    import torch.nn.functional as F

    B, T, D, H = images.shape[0], cfg.tokens, cfg.dim, cfg.heads
    eps = cfg.ln_eps
    raw = {k: v.to(images.device).float() for k, v in raw.items()}
    x = F.linear(patchify(images, cfg.patch, cfg.mean, cfg.std), raw["patch_w"], raw["patch_b"])
    x = x + raw["pos_embed"][1:]
    cls = (raw["cls_token"] + raw["pos_embed"][0]).expand(B, 1, D)
    x = torch.cat([cls, x], dim=1).reshape(B * T, D)
    cos, sin = rope_tables(cfg.grid, cfg.rope_ref_grid, cfg.head_dim)
    for i in range(cfg.depth):
        p = f"blocks.{i}."
        h = F.layer_norm(x, (D,), raw[p + "norm1.weight"], raw[p + "norm1.bias"], eps)
        qkv = _rope_qk(F.linear(h, raw[p + "qkv.weight"], raw[p + "qkv.bias"]), cos, sin, T, D)
        q, k, v = qkv.view(B, T, 3, H, D // H).permute(2, 0, 3, 1, 4)
        o = F.scaled_dot_product_attention(q, k, v, scale=1.0).transpose(1, 2).reshape(B * T, D)
        x = x + F.linear(o, raw[p + "proj.weight"], raw[p + "proj.bias"])
        h = F.layer_norm(x, (D,), raw[p + "norm2.weight"], raw[p + "norm2.bias"], eps)
        gu = F.linear(h, raw[p + "fc1.weight"], raw[p + "fc1.bias"])
        hid = F.silu(gu[:, : cfg.mlp_hidden]) * gu[:, cfg.mlp_hidden :]
        hid = F.layer_norm(hid, (cfg.mlp_hidden,), raw[p + "mlp_norm.weight"], raw[p + "mlp_norm.bias"], eps)
        x = x + F.linear(hid, raw[p + "fc2.weight"], raw[p + "fc2.bias"])
    if cfg.head == "tree":
        xf = F.layer_norm(x, (D,), raw["norm.weight"], raw["norm.bias"], eps).view(B, T, D)
        feat = tree_pool(xf, raw, cfg, half=False)
    else:
        feat = F.layer_norm(x.view(B, T, D)[:, 0], (D,), raw["norm.weight"], raw["norm.bias"], eps)
    return F.linear(feat, raw["head.weight"], raw["head.bias"])


def tree_pool(x: torch.Tensor, w: dict, cfg, half: bool, eps: float | None = None) -> torch.Tensor:
    """Haruka tree attention pool (foidfinder/backends/mlx/haruka.py:104-136; the model card's MHAttnPool,
    tests/test_haruka.py:73-122) on final-normed tokens x [B, T, D] -> leaf features [B, leaves * leaf_dim].

    w holds the folded pool weights (`pool.*`, haruka.py:fold:66-80: key rows of `pool.kv` carry the
    1/sqrt(pool head dim) scale). With half=True the fp16 storage points of the GPU engine are applied
    (pool-normed tokens, key/value, leaf features); everything else is f32. The LayerNorm eps is the
    backbone's (1e-6, as mlx/haruka.py:19 uses for every norm) unless given: the model card's pool
    LayerNorms use torch's default 1e-5."""
    B, T, D = x.shape
    Hp, C, Qn, L = cfg.pool_heads, cfg.coarse_queries, cfg.leaf_queries, cfg.leaf_dim
    hd, eps = D // Hp, cfg.ln_eps if eps is None else eps
    f = (lambda t: t.half().float()) if half else (lambda t: t)
    g = lambda k: w[k].float()  # noqa: E731
    xn = f(Q.layer_norm(x.reshape(B * T, D).float(), g("pool.norm.weight"), g("pool.norm.bias"), eps))
    kv = f(xn @ g("pool.kv.weight").t() + g("pool.kv.bias")).view(B, T, 2, Hp, hd)
    k, v = kv[:, :, 0].transpose(1, 2), kv[:, :, 1].transpose(1, 2)  # [B, Hp, T, hd]

    def slot_attend(q: torch.Tensor, bias: torch.Tensor):  # q [B, M, D] -> attn [B, Hp, M, T], z [B, M, D]
        qh = q.view(B, -1, Hp, hd).transpose(1, 2)
        logits = qh @ k.transpose(-1, -2)
        attn = torch.softmax(logits, dim=2) * torch.sigmoid(logits + bias.view(1, 1, -1, 1))
        return attn, (attn @ v).transpose(1, 2).reshape(B, -1, D)

    _, z = slot_attend(g("pool.q_coarse").expand(B, C, D), g("pool.q_coarse_bias"))
    z_coarse = Q.layer_norm(z, g("pool.trunk_norm.weight"), g("pool.trunk_norm.bias"), eps)
    z_parent = z_coarse.repeat_interleave(Qn // C, dim=1)
    q_leaf = Q.layer_norm(z_parent + g("pool.q_child"), g("pool.child_q_norm.weight"), g("pool.child_q_norm.bias"), eps)
    attn, z_child = slot_attend(q_leaf, g("pool.q_child_bias"))
    z_tree = Q.layer_norm(z_parent + z_child, g("pool.leaf_norm.weight"), g("pool.leaf_norm.bias"), eps)
    mass = attn.sum(-1).mean(1)[..., None]  # [B, leaves, 1]
    z_tree = z_tree * (mass / (mass + 4.0))
    leaf = torch.einsum("bqd,qdf->bqf", z_tree, g("pool.leaf.weight")) + g("pool.leaf.bias")
    return f(leaf.reshape(B, Qn * L))


def _residual(x: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
    """fp16 residual stream: x + fp16(y), rounded to fp16 (the reference stages y as fp16 and adds with
    __hadd2, foidfinder/backends/cuda/csrc/gemm.cuh:153-169)."""
    return (x.float() + y.half().float()).half()


def _lin(a8: torch.Tensor, rs: torch.Tensor, conv: dict, name: str) -> torch.Tensor:
    acc = Q.gemm_s8_acc(a8, conv[name + ".qweight"])
    return Q.dequant(acc, rs, conv[name + ".wscale"], conv[name + ".bias"])


def forward_int8(
    conv: dict[str, torch.Tensor], cfg, images: torch.Tensor, trace: list | None = None, rot=None
) -> torch.Tensor:
    """The GPU engine's arithmetic, from the converted checkpoint -> logits [B, num_tags], on the images'
    device (the CPU, or a GPU to check full-size models quickly).

    fp16 rounding points match the kernels: patches, x after the stem / each residual add, qkv, the
    attention output, the SwiGLU output h and the final-normed class tokens. If `trace` is a list it
    receives one dict of every stage's inputs and outputs per block, then a final dict with the stem
    output, the normed class tokens and the logits (for teacher-forced kernel comparisons). `rot`
    replaces the activation quantiser (default `quant.rot_q8`)."""
    rot_q8 = rot or Q.rot_q8
    conv = {k: v.to(images.device) for k, v in conv.items()}
    B, T, D, H, Hp = images.shape[0], cfg.tokens, cfg.dim, cfg.heads, cfg.mlp_hidden_pad
    eps = cfg.ln_eps
    patches = patchify(images, cfg.patch, cfg.mean, cfg.std).half().float()
    pw = conv["patch_w"].float()[:, : cfg.k_patch]
    stem = patches @ pw.t() + conv["pos_bias"].float()
    x = torch.empty(B, T, D, dtype=torch.float16, device=images.device)
    x[:, 1:] = stem.half()
    x[:, 0] = conv["cls_row"]
    x = x.reshape(B * T, D)
    cos, sin = conv["rope_cos"].float().t(), conv["rope_sin"].float().t()  # stored angle-major [32, tokens]
    x_stem = x
    for i in range(cfg.depth):
        p = f"blocks.{i}."
        x_in = x
        a8, rs = rot_q8(x, conv[p + "norm1.weight"], conv[p + "norm1.bias"], block=cfg.rot_block_dim, eps=eps)
        qkv = _rope_qk(_lin(a8, rs, conv, p + "qkv"), cos, sin, T, D).half()
        o = _attention(qkv, B, T, H).half()
        a8o, rso = rot_q8(o, None, None, block=cfg.rot_block_dim)
        x = _residual(x, _lin(a8o, rso, conv, p + "proj"))
        a8m, rsm = rot_q8(x, conv[p + "norm2.weight"], conv[p + "norm2.bias"], block=cfg.rot_block_dim, eps=eps)
        gu = _lin(a8m, rsm, conv, p + "fc1").view(B * T, Hp // 64, 2, 64)
        h = Q.silu_mul(gu[:, :, 0], gu[:, :, 1]).reshape(B * T, Hp).half()
        a8h, rsh = rot_q8(
            h, conv[p + "mlp_norm.weight"], conv[p + "mlp_norm.bias"], block=cfg.rot_block_hidden, eps=eps,
            valid_cols=cfg.mlp_hidden,
        )
        x_mid = x
        x = _residual(x, _lin(a8h, rsh, conv, p + "fc2"))
        if trace is not None:
            trace.append(
                dict(x_in=x_in, a8=a8, rs=rs, qkv=qkv, o=o, a8o=a8o, rso=rso, x_attn=x_mid, a8m=a8m, rsm=rsm, h=h,
                     a8h=a8h, rsh=rsh, x_out=x)
            )
    if cfg.head == "tree":
        xf = Q.layer_norm(x.float(), conv["norm.weight"], conv["norm.bias"], eps).half().float().view(B, T, D)
        xc = tree_pool(xf, conv, cfg, half=True).half()
    else:
        xc = Q.layer_norm(x.view(B, T, D)[:, 0], conv["norm.weight"], conv["norm.bias"], eps).half()
    logits = xc.float() @ conv["head.weight"].float()[: cfg.num_tags].t() + conv["head.bias"][: cfg.num_tags]
    if trace is not None:
        trace.append(dict(x_stem=x_stem, patches=patches.half(), x_final=x, cls=xc, logits=logits))
    return logits
