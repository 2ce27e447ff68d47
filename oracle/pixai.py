"""Oracle restatement of the reference's PixAI layout helpers (CPU, torch) — test infrastructure only.

- `window_perm`  foidfinder/backends/cuda/reference.py:21-24 (window order -> row-major grid index)
- `axial_rope`   reference.py:27-34 (x bands then y bands, fp32)
- `apply_rope`   reference.py:37-41 (interleaved pairs, fp32, cast back)
- `gelu_tanh`    foidfinder/backends/cuda/csrc/common.cuh:55-56 (the fc1 epilogue's tanh GELU)
- `forward_fp32` reference.py:109-140 (PixAITorch.forward + pool_head, f32, official checkpoint names)
- `forward_int8` foidfinder/backends/cuda/engine.py:142-161 (PixAICuda._forward: int8 blocks, fp16 storage)
- `reference_engine_forward` engine.py:142-161 itself: the reference's launch sequence through the
                 reference's own compiled kernels (torch.ops.foidfinder), with its fp16 torch stem and pool
                 head (reference.py:103-107, :133-140) — the reference engine as a second, GPU checker
The forwards run on the device of their inputs (the CPU, or a GPU to check full-size models quickly).
- `rgb_on_white` foidfinder/image.py:41-48 (transparency composited onto white)
- `preprocess`   foidfinder/backends/cuda/preprocess.py:16-32 (float letterbox: /255, antialiased bilinear
                 F.interpolate, x * 2 - 1 to fp16 on a -1 canvas), run with torch on the CPU
"""

from __future__ import annotations

import torch

D = 64


def window_perm(grid: int, window: int) -> torch.Tensor:
    """Index i of the window-ordered sequence -> row-major grid index: windows row-major, then the
    window's patches row-major (reference.py:21-24 with grid 72, window 24)."""
    nw = grid // window
    wr, wc, r, c = torch.meshgrid(*(torch.arange(n) for n in (nw, nw, window, window)), indexing="ij")
    return ((wr * window + r) * grid + wc * window + c).reshape(-1)


def gelu_tanh(x: torch.Tensor) -> torch.Tensor:
    """0.5 x (1 + tanh(0.7978845608 (x + 0.044715 x^3))) in f32."""
    x = x.float()
    return 0.5 * x * (1.0 + torch.tanh(0.7978845608 * (x + 0.044715 * x * x * x)))


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



def rgb_on_white(image):
    """PIL image -> RGB with any transparency composited onto white (foidfinder/image.py:41-48)."""
    from PIL import Image

    if image.mode == "RGB":
        return image
    rgba = image.convert("RGBA")
    canvas = Image.new("RGBA", rgba.size, (255, 255, 255, 255))
    canvas.alpha_composite(rgba)
    return canvas.convert("RGB")


@torch.no_grad()
def preprocess(images: list, size: int = 1008) -> torch.Tensor:
    """PIL images -> [B, size, size, 3] fp16 normalised pixels, as preprocess.py:16-32 computes them (on the
    CPU here): pixels / 255 in f32, the longer side scaled to `size` with F.interpolate(mode="bilinear",
    align_corners=False, antialias=True) when the size changes, x * 2 - 1 rounded to fp16, centred on -1."""
    import numpy as np
    import torch.nn.functional as F

    out = torch.full((len(images), size, size, 3), -1.0, dtype=torch.half)
    for b, image in enumerate(images):
        x = torch.from_numpy(np.array(rgb_on_white(image))).permute(2, 0, 1)[None].float().div_(255.0)
        h, w = x.shape[-2:]
        r = min(size / h, size / w)
        nh, nw = int(h * r), int(w * r)
        if (nh, nw) != (h, w):
            x = F.interpolate(x, size=(nh, nw), mode="bilinear", align_corners=False, antialias=True)
        top, left = (size - nh) // 2, (size - nw) // 2
        out[b, top : top + nh, left : left + nw] = (x[0].permute(1, 2, 0) * 2.0 - 1.0).half()
    return out


# ---------------------------------------------------------------- whole model


def patch_rows(images: torch.Tensor, cfg) -> torch.Tensor:
    """uint8 [B, S, S, 3] -> normalised f32 patches [B, L, p*p*3] in window order, (kh, kw, c) columns
    (PixAITorch.patchify, reference.py:103-107, on the normalised pixels of preprocess.py:30)."""
    from . import eva02 as E

    return E.patchify(images, cfg.patch, cfg.mean, cfg.std)[:, window_perm(cfg.grid, cfg.window)]


def _window_tables(cfg) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """(window cos, sin) [window^2, 32] and (global cos, sin) [L, 32] in window order (reference.py:95-98)."""
    cw, sw = axial_rope(cfg.window, 1.0)
    cg, sg = axial_rope(cfg.grid, cfg.window / cfg.grid)
    perm = window_perm(cfg.grid, cfg.window)
    return cw, sw, cg[perm], sg[perm]


def _sdpa(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float) -> torch.Tensor:
    return torch.softmax((q @ k.transpose(-1, -2)) * scale, dim=-1) @ v


def forward_fp32(raw: dict[str, torch.Tensor], cfg, images: torch.Tensor) -> torch.Tensor:
    """PixAITorch.forward (reference.py:109-130) and pool_head (:132-140) in f32 on the official checkpoint
    layout, from uint8 images -> logits [B, num_tags], with the same torch calls (F.layer_norm, F.linear,
    F.scaled_dot_product_attention, erf F.gelu), so that its CPU time is the reference's."""
    import torch.nn.functional as F

    B, G, D, nh, L, win = images.shape[0], cfg.grid, cfg.dim, cfg.heads, cfg.patches, cfg.window
    nw, eps, dev = G // win, cfg.ln_eps, images.device
    g = lambda k: raw[k].to(dev).float()  # noqa: E731
    perm = window_perm(G, win).to(dev)
    pw = g("patch_embed.proj.weight").permute(0, 2, 3, 1).reshape(D, -1)
    pos = g("pos_embed")[0, 1:]
    pre = int(round(pos.shape[0] ** 0.5))
    pos = pos.reshape(pre, pre, D).repeat(G // pre, G // pre, 1).reshape(L, D)[perm]
    x = (patch_rows(images, cfg) @ pw.t() + pos).reshape(B * L, D)
    x = F.layer_norm(x, (D,), g("ln_pre.weight"), g("ln_pre.bias"), eps)
    cw, sw, cg, sg = (t.to(dev) for t in _window_tables(cfg))
    for i in range(cfg.depth):
        p = f"blocks.{i}."
        h = F.layer_norm(x, (D,), g(p + "norm1.weight"), g(p + "norm1.bias"), eps)
        qkv = F.linear(h, g(p + "attn.qkv.weight"), g(p + "attn.qkv.bias"))
        nb, n, cos, sin = (B, L, cg, sg) if cfg.is_global(i) else (B * nw * nw, win * win, cw, sw)
        q, k, v = qkv.view(nb, n, 3, nh, D // nh).permute(2, 0, 3, 1, 4)
        o = F.scaled_dot_product_attention(apply_rope(q, cos, sin), apply_rope(k, cos, sin), v)
        x = x + F.linear(o.transpose(1, 2).reshape(B * L, D), g(p + "attn.proj.weight"), g(p + "attn.proj.bias"))
        h = F.layer_norm(x, (D,), g(p + "norm2.weight"), g(p + "norm2.bias"), eps)
        h = F.gelu(F.linear(h, g(p + "mlp.fc1.weight"), g(p + "mlp.fc1.bias")))
        x = x + F.linear(h, g(p + "mlp.fc2.weight"), g(p + "mlp.fc2.bias"))
    return pool_head_fp32(x.view(B, L, D), raw, cfg)


def pool_head_fp32(x: torch.Tensor, raw: dict[str, torch.Tensor], cfg) -> torch.Tensor:
    """PixAITorch.pool_head (reference.py:132-140) in f32: x [B, L, D] window-ordered -> logits."""
    import torch.nn.functional as F

    B, L, D = x.shape
    nh = cfg.heads
    g = lambda k: raw[k].to(x.device).float()  # noqa: E731
    h = F.layer_norm(x, (D,), g("head_pool.norm.weight"), g("head_pool.norm.bias"), cfg.ln_eps)
    h = h + g("head_pool.pos_embed")[window_perm(cfg.grid, cfg.window).to(x.device)]
    k, v = F.linear(h, g("head_pool.kv.weight"), g("head_pool.kv.bias")).view(B, L, 2, nh, D // nh).permute(2, 0, 3, 1, 4)
    q = g("head_pool.q").reshape(1, nh, 1, D // nh).expand(B, nh, 1, D // nh)
    o = F.scaled_dot_product_attention(q, k, v).reshape(B, D)
    o = F.linear(o, g("head_pool.proj.weight"), g("head_pool.proj.bias"))
    return F.linear(o, g("head.weight"), g("head.bias"))


def forward_int8(conv: dict[str, torch.Tensor], cfg, images: torch.Tensor, trace: list | None = None,
                 rot=None) -> torch.Tensor:
    """The GPU engine's PixAI arithmetic on the CPU, from the converted checkpoint -> logits [B, num_tags].

    PixAICuda._forward (foidfinder/backends/cuda/engine.py:142-161) step by step: fp16 stem (+ window-ordered
    position embedding), ln_pre to fp16, then per block LN1+H1024+q8 -> QKV GEMM + RoPE (window table, or
    the global one in the global blocks) -> attention per window / per image -> H1024+q8 -> proj + residual
    -> LN2+H1024+q8 -> fc1 + tanh GELU (csrc/common.cuh:56) -> H128+q8 -> fc2 + residual, and the pool head
    of reference.py:132-140 with fp16 storage between its steps. If `trace` is a list it receives one dict
    per block (every stage's inputs and outputs) and a final dict (stem, pool stages, logits). `rot`
    replaces the activation quantiser (default `quant.rot_q8`)."""
    from . import eva02 as E
    from . import quant as Q

    rot_q8 = rot or Q.rot_q8
    conv = {k: v.to(images.device) for k, v in conv.items()}
    B, L, D, nh, win = images.shape[0], cfg.patches, cfg.dim, cfg.heads, cfg.window
    M, eps = B * L, cfg.ln_eps
    patches = patch_rows(images, cfg).half()
    x = (patches.float() @ conv["patch_w"].float()[:, : cfg.k_patch].t() + conv["pos_bias"].float()).half()
    x_stem = x.reshape(M, D)
    x = Q.layer_norm(x_stem.float(), conv["ln_pre.weight"], conv["ln_pre.bias"], eps).half()
    x_pre = x
    tables = {
        False: (conv["rope_cos"].float().t(), conv["rope_sin"].float().t(), win * win),
        True: (conv["rope_cos_global"].float().t(), conv["rope_sin_global"].float().t(), L),
    }

    def lin(a8, rs, name):
        return Q.dequant(Q.gemm_s8_acc(a8, conv[name + ".qweight"]), rs, conv[name + ".wscale"], conv[name + ".bias"])

    for i in range(cfg.depth):
        p = f"blocks.{i}."
        x_in = x
        cos, sin, n = tables[cfg.is_global(i)]
        a8, rs = rot_q8(x, conv[p + "norm1.weight"], conv[p + "norm1.bias"], block=cfg.rot_block_dim, eps=eps)
        qkv = Q.apply_rope_pairs(lin(a8, rs, p + "qkv"), cos, sin, torch.arange(M, device=x.device) % n, 2 * D).half()
        o = E._attention(qkv, M // n, n, nh).half()
        a8o, rso = rot_q8(o, None, None, block=cfg.rot_block_dim)
        x = E._residual(x, lin(a8o, rso, p + "proj"))
        x_attn = x
        a8m, rsm = rot_q8(x, conv[p + "norm2.weight"], conv[p + "norm2.bias"], block=cfg.rot_block_dim, eps=eps)
        h = gelu_tanh(lin(a8m, rsm, p + "fc1")).half()
        a8h, rsh = rot_q8(h, None, None, block=cfg.rot_block_hidden)
        x = E._residual(x, lin(a8h, rsh, p + "fc2"))
        if trace is not None:
            trace.append(dict(x_in=x_in, a8=a8, rs=rs, qkv=qkv, o=o, a8o=a8o, rso=rso, x_attn=x_attn, a8m=a8m, rsm=rsm,
                              h=h, a8h=a8h, rsh=rsh, x_out=x, seq=n))
    xn = (Q.layer_norm(x.float(), conv["pool.norm.weight"], conv["pool.norm.bias"], eps).half().view(B, L, D)
          + conv["pool.pos"]).view(M, D)
    kv = (xn.float() @ conv["pool.kv.weight"].float().t() + conv["pool.kv.bias"]).half()
    k = kv[:, :D].float().view(B, L, nh, D // nh).permute(0, 2, 1, 3)
    v = kv[:, D:].float().view(B, L, nh, D // nh).permute(0, 2, 1, 3)
    q = conv["pool.q"].float().view(1, nh, 1, D // nh)
    att = _sdpa(q, k, v, 1.0).reshape(B, D).half()
    z = (att.float() @ conv["pool.proj.weight"].float().t() + conv["pool.proj.bias"]).half()
    logits = z.float() @ conv["head.weight"].float()[: cfg.num_tags].t() + conv["head.bias"][: cfg.num_tags]
    if trace is not None:
        trace.append(dict(patches=patches.reshape(M, -1), x_stem=x_stem, x_pre=x_pre, x_final=x, xn=xn, kv=kv,
                          att=att, z=z, logits=logits))
    return logits


Q_SCALE_REF = 0.125 * 1.4426950408889634  # engine.py:26: 1/sqrt(64) * log2(e), applied by the QKV epilogue


@torch.no_grad()
def reference_engine_forward(k, ck: dict[str, torch.Tensor], cfg, pixels: torch.Tensor, stages: int = 3) -> torch.Tensor:
    """PixAICuda._forward (foidfinder/backends/cuda/engine.py:142-161) on the reference's int8 checkpoint `ck`
    (convert_checkpoint's output, official names) through the reference's own kernels `k` (its
    torch.ops.foidfinder namespace: gemm_s8, rot_q8_1024, rot_q8_h128, attention), from normalised fp16
    pixels [B, S, S, 3] on a GPU -> logits [B, num_tags] f32. The stem and the pool head are the reference's
    fp16 torch code (PixAITorch with dtype fp16: patchify + matmul + position, F.layer_norm ln_pre,
    reference.py:103-107, :114-116, pool_head :133-140); buffers as _buffers (engine.py:96-106); `stages`
    is the GEMM pipeline depth _autotune would pick (it changes speed, not results)."""
    import torch.nn.functional as F

    dev = pixels.device
    B, G, P, C, nh, win = pixels.shape[0], cfg.grid, cfg.patch, cfg.dim, cfg.heads, cfg.window
    L, nw, HID, eps = cfg.patches, G // win, cfg.mlp_hidden, cfg.ln_eps
    T = B * L

    def h16(t):
        return t.to(dev, torch.float16).contiguous()

    def f32(t):
        return t.to(dev, torch.float32).contiguous()

    perm = window_perm(G, win).to(dev)
    patch_w = h16(ck["patch_embed.proj.weight"].permute(0, 2, 3, 1).reshape(C, -1))
    pos = ck["pos_embed"][0, 1:]
    pre = int(round(pos.shape[0] ** 0.5))
    pos = h16(pos.reshape(pre, pre, C).repeat(G // pre, G // pre, 1).reshape(L, C).to(dev)[perm])
    cw, sw = (f32(t) for t in axial_rope(win, 1.0))
    cg, sg = axial_rope(G, win / G)
    cg, sg = f32(cg.to(dev)[perm]), f32(sg.to(dev)[perm])
    x = torch.empty(T, C, device=dev, dtype=torch.half)
    a8 = torch.empty(T, C, device=dev, dtype=torch.int8)
    rs = torch.empty(T, device=dev)
    qkv = torch.empty(T, 3 * C, device=dev, dtype=torch.half)
    o16 = torch.empty(T, C, device=dev, dtype=torch.half)
    hh = torch.empty(T, HID, device=dev, dtype=torch.half)
    h8 = torch.empty(T, HID, device=dev, dtype=torch.int8)
    patches = pixels.to(torch.float16).view(B, nw, win, P, nw, win, P, 3).permute(0, 1, 4, 2, 5, 3, 6, 7)
    torch.matmul(patches.reshape(T, P * P * 3), patch_w.t(), out=x)
    x.view(B, L, C).add_(pos)
    x.copy_(F.layer_norm(x, (C,), h16(ck["ln_pre.weight"]), h16(ck["ln_pre.bias"]), eps))

    def lin(p):
        return ck[p + ".qweight"].to(dev), f32(ck[p + ".wscale"]), f32(ck[p + ".bias"])

    for i in range(cfg.depth):
        b = f"blocks.{i}."
        seq, (cos, sin) = (L, (cg, sg)) if cfg.is_global(i) else (win * win, (cw, sw))
        k.rot_q8_1024(x, f32(ck[b + "norm1.weight"]), f32(ck[b + "norm1.bias"]), a8, rs)
        w, s, bb = lin(b + "attn.qkv")
        k.gemm_s8(a8, w, rs, s, bb, qkv, 0, stages, cos, sin, Q_SCALE_REF)
        k.attention(qkv, o16, seq)
        k.rot_q8_1024(o16, None, None, a8, rs)
        w, s, bb = lin(b + "attn.proj")
        k.gemm_s8(a8, w, rs, s, bb, x, 1, stages, None, None, Q_SCALE_REF)
        k.rot_q8_1024(x, f32(ck[b + "norm2.weight"]), f32(ck[b + "norm2.bias"]), a8, rs)
        w, s, bb = lin(b + "mlp.fc1")
        k.gemm_s8(a8, w, rs, s, bb, hh, 2, stages, None, None, Q_SCALE_REF)
        k.rot_q8_h128(hh, h8, rs)
        w, s, bb = lin(b + "mlp.fc2")
        k.gemm_s8(h8, w, rs, s, bb, x, 1, stages, None, None, Q_SCALE_REF)
    xv = x.view(B, L, C)
    h = F.layer_norm(xv, (C,), h16(ck["head_pool.norm.weight"]), h16(ck["head_pool.norm.bias"]), eps)
    h = h + h16(ck["head_pool.pos_embed"].to(dev)[perm])
    kk, vv = F.linear(h, h16(ck["head_pool.kv.weight"]), h16(ck["head_pool.kv.bias"])).view(
        B, L, 2, nh, C // nh).permute(2, 0, 3, 1, 4)
    q = h16(ck["head_pool.q"]).view(1, nh, 1, C // nh).expand(B, nh, 1, C // nh)
    o = F.scaled_dot_product_attention(q, kk, vv).reshape(B, C)
    o = F.linear(o, h16(ck["head_pool.proj.weight"]), h16(ck["head_pool.proj.bias"]))
    return F.linear(o, h16(ck["head.weight"]), h16(ck["head.bias"])).float()
