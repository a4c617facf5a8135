"""CPU fp32 oracle of the SDXL UNet2DConditionModel forward — TEST INFRASTRUCTURE ONLY.

This module is the checker for the B200 kernels, never the thing measured or shipped: only
`tests/`, `__graft_entry__.smoke()` and the `cpu_baseline` / `--impl reference` legs of
`bench.py` import it.

It restates, in plain PyTorch fp32 ops, the UNet that the reference orchestrates in
`src/infer/unet.cu` (structure `src/infer/unet.cuh:21-36`):
  * time embedding: sinusoidal(320, flip_sin_to_cos, shift 0) -> linear_1 + SiLU -> linear_2
    (`unet.cu:980-993`, `src/kernels/timeembed.cuh:13-28`);
  * add embedding: [text_embeds(1280) | 6 x sinusoidal(256) of time_ids] -> linear_1 + SiLU ->
    linear_2, added to temb (`unet.cu:1005-1030`);
  * ResnetBlock2D (`unet.cu:528-663`): GN(32, 1e-5)+SiLU -> conv1 -> +time_emb_proj(SiLU(temb))
    -> GN+SiLU -> conv2 -> + (x | conv_shortcut(x));
  * Transformer2D (`unet.cu:800-858`): GN(32, 1e-6) -> proj_in -> L x BasicTransformerBlock ->
    proj_out -> + residual; BasicTransformerBlock (`unet.cu:667-797`): LN -> self-attn -> +res;
    LN -> cross-attn(ctx) -> +res; LN -> GEGLU FF -> +res; head_dim 64, scale 1/8;
  * Downsample2D = conv3x3 stride 2 pad 1; Upsample2D = nearest 2x + conv3x3 (`unet.cu:861-881`);
  * block order and the skip stack (`unet.cu:1071-1290`).
The SDXL architecture semantics come from diffusers' UNet2DConditionModel, whose source is not
part of the reference tree (it is the reference's golden-dump dependency,
`scripts/dollma_dump_unet_golden.py`); this file is written from the architecture as the
reference's orchestration documents it, not from diffusers' code.

Parity pin: the reference's golden files (`unet_io.safetensors`, produced by diffusers with
pretrained weights) are not in the reference checkout, so this oracle is pinned to the
reference's own per-op definitions (see tests/test_oracle_*.py); whole-UNet parity against the
reference's goldens is unpinned.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch
import torch.nn.functional as F


@dataclass
class UNetConfig:
    """SDXL UNet hyper-parameters (`unet.cuh:21-36`).  `depths` may be reduced for tests."""

    channels: tuple = (320, 640, 1280)
    depths: tuple = (0, 2, 10)          # transformer layers per Transformer2D at each level
    mid_depth: int = 10
    ctx_dim: int = 2048
    ctx_tokens: int = 77
    head_dim: int = 64
    groups: int = 32
    temb_dim: int = 1280
    time_proj_dim: int = 320
    add_time_dim: int = 256
    text_embed_dim: int = 1280
    in_channels: int = 4
    out_channels: int = 4

    @property
    def add_in_dim(self) -> int:
        return self.text_embed_dim + 6 * self.add_time_dim  # 2816


SDXL = UNetConfig()


# ---------------------------------------------------------------------------- storage rounding

_FP16_STORAGE = [False]


class fp16_storage:
    """Context manager: while active, the oracle rounds every activation it would hand to the
    next layer to fp16 (then computes on in fp32), at the points where an fp16-storage
    implementation writes its tensors: normalised inputs of a convolution / linear, each
    convolution or linear output after its bias / residual, attention outputs, GEGLU outputs.
    The reference stores fp16 at these points too (and at more), so the difference between this
    variant and the plain fp32 oracle is the error that fp16 storage alone costs."""

    def __enter__(self):
        _FP16_STORAGE[0] = True
        return self

    def __exit__(self, *exc):
        _FP16_STORAGE[0] = False
        return False


def _st(t: torch.Tensor) -> torch.Tensor:
    return t.half().float() if _FP16_STORAGE[0] else t


# ---------------------------------------------------------------------------- primitives

def timestep_embedding(t: torch.Tensor, dim: int, max_period: float = 10000.0) -> torch.Tensor:
    """Sinusoidal embedding, flip_sin_to_cos=True, shift 0: [cos(t f_i) | sin(t f_i)],
    f_i = max_period^(-i/half) (`src/kernels/timeembed.cuh:13-28`).  t: [n] -> [n, dim]."""
    half = dim // 2
    exponent = -math.log(max_period) * torch.arange(half, dtype=torch.float32) / half
    freqs = torch.exp(exponent)
    args = t.float()[:, None] * freqs[None, :]
    return torch.cat([torch.cos(args), torch.sin(args)], dim=-1)


def linear(x, sd, name, bias=True):
    w = sd[name + ".weight"].float()
    b = sd[name + ".bias"].float() if bias else None
    return F.linear(x, w, b)


def group_norm(x, sd, name, groups, eps):
    return F.group_norm(x, groups, sd[name + ".weight"].float(), sd[name + ".bias"].float(), eps)


def conv(x, sd, name, stride=1, padding=1):
    return F.conv2d(x, sd[name + ".weight"].float(), sd[name + ".bias"].float(), stride=stride,
                    padding=padding)


def layer_norm(x, sd, name, eps=1e-5):
    C = x.shape[-1]
    return F.layer_norm(x, (C,), sd[name + ".weight"].float(), sd[name + ".bias"].float(), eps)


def attention(q, k, v, heads):
    """softmax(q k^T / sqrt(64)) v over [B, S, heads*64] (`unet.cu:677-797`)."""
    B, Sq, C = q.shape
    Sk = k.shape[1]
    dh = C // heads
    q = q.view(B, Sq, heads, dh).transpose(1, 2)
    k = k.view(B, Sk, heads, dh).transpose(1, 2)
    v = v.view(B, Sk, heads, dh).transpose(1, 2)
    s = (q @ k.transpose(-1, -2)) * (1.0 / math.sqrt(dh))
    p = torch.softmax(s, dim=-1)
    o = p @ v
    return o.transpose(1, 2).reshape(B, Sq, C)


# ---------------------------------------------------------------------------- blocks

def resnet_block(x, temb_silu, sd, prefix, cfg: UNetConfig):
    """`unet.cu:537-663`."""
    h = _st(F.silu(group_norm(x, sd, prefix + "norm1", cfg.groups, 1e-5)))
    h = conv(h, sd, prefix + "conv1")
    h = _st(h + linear(temb_silu, sd, prefix + "time_emb_proj")[:, :, None, None])
    h = _st(F.silu(group_norm(h, sd, prefix + "norm2", cfg.groups, 1e-5)))
    h = conv(h, sd, prefix + "conv2")
    if (prefix + "conv_shortcut.weight") in sd:
        x = conv(x, sd, prefix + "conv_shortcut", padding=0)
    return _st(x + h)


def transformer_block(x, ctx, sd, p, heads):
    """`unet.cu:677-797`: x [B, S, C]."""
    n = layer_norm(x, sd, p + "norm1")
    q = _st(linear(n, sd, p + "attn1.to_q", bias=False))
    k = _st(linear(n, sd, p + "attn1.to_k", bias=False))
    v = _st(linear(n, sd, p + "attn1.to_v", bias=False))
    x = _st(x + linear(_st(attention(q, k, v, heads)), sd, p + "attn1.to_out.0"))
    n = layer_norm(x, sd, p + "norm2")
    q = _st(linear(n, sd, p + "attn2.to_q", bias=False))
    k = _st(linear(ctx, sd, p + "attn2.to_k", bias=False))
    v = _st(linear(ctx, sd, p + "attn2.to_v", bias=False))
    x = _st(x + linear(_st(attention(q, k, v, heads)), sd, p + "attn2.to_out.0"))
    n = layer_norm(x, sd, p + "norm3")
    h = linear(n, sd, p + "ff.net.0.proj")
    hid, gate = h.chunk(2, dim=-1)
    x = _st(x + linear(_st(hid * F.gelu(gate)), sd, p + "ff.net.2"))
    return x


def transformer2d(x, ctx, sd, prefix, layers, cfg: UNetConfig):
    """`unet.cu:810-858`: GN(eps 1e-6) -> proj_in -> blocks -> proj_out -> + residual."""
    B, C, H, W = x.shape
    heads = C // cfg.head_dim
    h = _st(group_norm(x, sd, prefix + "norm", cfg.groups, 1e-6))
    h = h.permute(0, 2, 3, 1).reshape(B, H * W, C)
    h = _st(linear(h, sd, prefix + "proj_in"))
    for l in range(layers):
        h = transformer_block(h, ctx, sd, f"{prefix}transformer_blocks.{l}.", heads)
    h = linear(h, sd, prefix + "proj_out")
    h = h.reshape(B, H, W, C).permute(0, 3, 1, 2)
    return _st(x + h)


def downsample(x, sd, prefix):
    return _st(conv(x, sd, prefix + "conv", stride=2, padding=1))


def upsample(x, sd, prefix):
    x = F.interpolate(x, scale_factor=2.0, mode="nearest")
    return _st(conv(x, sd, prefix + "conv"))


# ---------------------------------------------------------------------------- embeddings

def time_embeddings(sd, timestep: float, text_embeds, time_ids, cfg: UNetConfig):
    """temb [B, 1280] (`unet.cu:980-1030`); time_ids [6] shared by the batch."""
    B = text_embeds.shape[0]
    t = torch.full((B,), float(timestep))
    sin = timestep_embedding(t, cfg.time_proj_dim)
    temb = linear(F.silu(linear(sin, sd, "time_embedding.linear_1")), sd, "time_embedding.linear_2")
    tid = timestep_embedding(time_ids.float().reshape(-1), cfg.add_time_dim).reshape(1, -1)
    add_in = torch.cat([text_embeds.float(), tid.expand(B, -1)], dim=-1)
    aug = linear(F.silu(linear(add_in, sd, "add_embedding.linear_1")), sd, "add_embedding.linear_2")
    return temb + aug


# ---------------------------------------------------------------------------- UNet

def unet_forward(sd, latent, timestep, ehs, text_embeds, time_ids, cfg: UNetConfig = SDXL,
                 hook=None):
    """Full forward: latent [B,4,H,W], ehs [B,77,2048], text_embeds [B,1280], time_ids [6]
    -> noise_pred [B,4,H,W] (all fp32).  `hook(name, tensor)` sees the stage outputs named as
    the reference's stage hooks (`unet.cu` dbg_stat names)."""
    def tap(name, t):
        if hook is not None:
            hook(name, t)
        return t

    C0, C1, C2 = cfg.channels
    ctx = ehs.float()
    temb = tap("temb_final", time_embeddings(sd, timestep, text_embeds, time_ids, cfg))
    ts = F.silu(temb)
    x = tap("conv_in_out", _st(conv(latent.float(), sd, "conv_in")))
    skips = [x]
    # down 0
    for r in range(2):
        x = resnet_block(x, ts, sd, f"down_blocks.0.resnets.{r}.", cfg)
        skips.append(x)
    x = downsample(x, sd, "down_blocks.0.downsamplers.0.")
    skips.append(x)
    tap("down_block_0_out", x)
    # down 1, down 2
    for lvl, has_ds in ((1, True), (2, False)):
        for r in range(2):
            x = resnet_block(x, ts, sd, f"down_blocks.{lvl}.resnets.{r}.", cfg)
            if cfg.depths[lvl] > 0:
                x = transformer2d(x, ctx, sd, f"down_blocks.{lvl}.attentions.{r}.",
                                  cfg.depths[lvl], cfg)
            skips.append(x)
        if has_ds:
            x = downsample(x, sd, f"down_blocks.{lvl}.downsamplers.0.")
            skips.append(x)
        tap(f"down_block_{lvl}_out", x)
    # mid
    x = resnet_block(x, ts, sd, "mid_block.resnets.0.", cfg)
    x = transformer2d(x, ctx, sd, "mid_block.attentions.0.", cfg.mid_depth, cfg)
    x = resnet_block(x, ts, sd, "mid_block.resnets.1.", cfg)
    tap("mid_block_out", x)
    # up
    for u in range(3):
        lvl = 2 - u
        for r in range(3):
            x = torch.cat([x, skips.pop()], dim=1)
            x = resnet_block(x, ts, sd, f"up_blocks.{u}.resnets.{r}.", cfg)
            if cfg.depths[lvl] > 0:
                x = transformer2d(x, ctx, sd, f"up_blocks.{u}.attentions.{r}.", cfg.depths[lvl], cfg)
        if u < 2:
            x = upsample(x, sd, f"up_blocks.{u}.upsamplers.0.")
        tap(f"up_block_{u}_out", x)
    h = _st(F.silu(group_norm(x, sd, "conv_norm_out", cfg.groups, 1e-5)))
    out = conv(h, sd, "conv_out")
    return tap("noise_pred", out)


# ---------------------------------------------------------------------------- weights

def weight_shapes(cfg: UNetConfig = SDXL) -> dict:
    """name -> shape of every UNet tensor (diffusers state-dict keys, as `unet.cu` reads them)."""
    C0, C1, C2 = cfg.channels
    S = {}

    def lin(n, o, i, bias=True):
        S[n + ".weight"] = (o, i)
        if bias:
            S[n + ".bias"] = (o,)

    def cv(n, o, i, k=3):
        S[n + ".weight"] = (o, i, k, k)
        S[n + ".bias"] = (o,)

    def norm(n, c):
        S[n + ".weight"] = (c,)
        S[n + ".bias"] = (c,)

    def resnet(p, cin, cout):
        norm(p + "norm1", cin)
        cv(p + "conv1", cout, cin)
        lin(p + "time_emb_proj", cout, cfg.temb_dim)
        norm(p + "norm2", cout)
        cv(p + "conv2", cout, cout)
        if cin != cout:
            cv(p + "conv_shortcut", cout, cin, k=1)

    def t2d(p, c, layers):
        norm(p + "norm", c)
        lin(p + "proj_in", c, c)
        for l in range(layers):
            b = f"{p}transformer_blocks.{l}."
            norm(b + "norm1", c)
            norm(b + "norm2", c)
            norm(b + "norm3", c)
            for q in ("to_q", "to_k", "to_v"):
                lin(b + "attn1." + q, c, c, bias=False)
            lin(b + "attn1.to_out.0", c, c)
            lin(b + "attn2.to_q", c, c, bias=False)
            lin(b + "attn2.to_k", c, cfg.ctx_dim, bias=False)
            lin(b + "attn2.to_v", c, cfg.ctx_dim, bias=False)
            lin(b + "attn2.to_out.0", c, c)
            lin(b + "ff.net.0.proj", 8 * c, c)
            lin(b + "ff.net.2", c, 4 * c)
        lin(p + "proj_out", c, c)

    lin("time_embedding.linear_1", cfg.temb_dim, cfg.time_proj_dim)
    lin("time_embedding.linear_2", cfg.temb_dim, cfg.temb_dim)
    lin("add_embedding.linear_1", cfg.temb_dim, cfg.add_in_dim)
    lin("add_embedding.linear_2", cfg.temb_dim, cfg.temb_dim)
    cv("conv_in", C0, cfg.in_channels)
    chans = [C0, C1, C2]
    cin = C0
    for lvl in range(3):
        c = chans[lvl]
        for r in range(2):
            resnet(f"down_blocks.{lvl}.resnets.{r}.", cin if r == 0 else c, c)
            if cfg.depths[lvl] > 0:
                t2d(f"down_blocks.{lvl}.attentions.{r}.", c, cfg.depths[lvl])
        if lvl < 2:
            cv(f"down_blocks.{lvl}.downsamplers.0.conv", c, c)
        cin = c
    resnet("mid_block.resnets.0.", C2, C2)
    t2d("mid_block.attentions.0.", C2, cfg.mid_depth)
    resnet("mid_block.resnets.1.", C2, C2)
    # skip channels in pop order: per up block (u), per resnet (r)
    skip_ch = [C0, C0, C0, C0, C1, C1, C1, C2, C2]  # push order
    cur = C2
    for u in range(3):
        lvl = 2 - u
        c = chans[lvl]
        for r in range(3):
            sk = skip_ch.pop()
            resnet(f"up_blocks.{u}.resnets.{r}.", cur + sk, c)
            cur = c
            if cfg.depths[lvl] > 0:
                t2d(f"up_blocks.{u}.attentions.{r}.", c, cfg.depths[lvl])
        if u < 2:
            cv(f"up_blocks.{u}.upsamplers.0.conv", c, c)
    norm("conv_norm_out", C0)
    cv("conv_out", cfg.out_channels, C0)
    return S


def init_weights(cfg: UNetConfig = SDXL, seed: int = 7, device="cpu", dtype=torch.float16):
    """Random-init weights of the named architecture: Linear weights N(0, 0.02), conv weights and
    biases Kaiming-uniform U(-1/sqrt(fan_in), +1/sqrt(fan_in)) (PyTorch's default), Linear
    biases N(0, 0.02), norm gammas 1 + N(0, 0.05), betas N(0, 0.05).  Deterministic in `seed`
    (names are visited in sorted order with one generator)."""
    g = torch.Generator(device=device).manual_seed(seed)
    sd = {}
    for name, shape in sorted(weight_shapes(cfg).items()):
        parts = name.rsplit(".", 1)
        base, kind = parts[0], parts[1]
        is_norm = base.endswith(("norm", "norm1", "norm2", "norm3", "conv_norm_out")) and len(shape) == 1
        if len(shape) == 4 or (kind == "bias" and _is_conv(base, cfg)):
            fan_in = _conv_fan_in(base, shape, cfg)
            bound = 1.0 / math.sqrt(fan_in)
            t = (torch.rand(shape, generator=g, device=device) * 2 - 1) * bound
        elif is_norm:
            if kind == "weight":
                t = 1.0 + 0.05 * torch.randn(shape, generator=g, device=device)
            else:
                t = 0.05 * torch.randn(shape, generator=g, device=device)
        else:
            t = 0.02 * torch.randn(shape, generator=g, device=device)
        sd[name] = t.to(dtype)
    return sd


_CONV_SUFFIXES = ("conv1", "conv2", "conv_shortcut", "conv_in", "conv_out", "downsamplers.0.conv",
                  "upsamplers.0.conv")


def _is_conv(base: str, cfg) -> bool:
    return base.endswith(_CONV_SUFFIXES)


def _conv_fan_in(base, shape, cfg):
    if len(shape) == 4:
        return shape[1] * shape[2] * shape[3]
    w = weight_shapes(cfg)[base + ".weight"]
    return w[1] * w[2] * w[3]


def make_inputs(B: int = 2, H: int = 128, W: int = 128, seed: int = 6, cfg: UNetConfig = SDXL):
    """Seeded synthetic inputs of the UNet step: latent [B,4,H,W] ~ N(0,1) (cond and uncond
    share it), ehs [B,77,2048] ~ N(0,1), text_embeds [B,1280] ~ N(0,1), time_ids
    [1024,1024,0,0,1024,1024] (as the reference's golden dump,
    `scripts/dollma_dump_unet_golden.py:141`).  All fp16."""
    g = torch.Generator().manual_seed(seed)
    lat = torch.randn(1, cfg.in_channels, H, W, generator=g).expand(B, -1, -1, -1).contiguous()
    ehs = torch.randn(B, cfg.ctx_tokens, cfg.ctx_dim, generator=g)
    te = torch.randn(B, cfg.text_embed_dim, generator=g)
    tid = torch.tensor([1024.0, 1024.0, 0.0, 0.0, 1024.0, 1024.0])
    return lat.half(), ehs.half(), te.half(), tid.half()


def unet_flops(B: int, H: int, W: int, cfg: UNetConfig = SDXL) -> float:
    """Algorithmic FLOPs (2 per MAC) of one forward: convs, linears and attention matmuls."""
    C0, C1, C2 = cfg.channels
    fl = 0.0

    def conv_f(cin, cout, h, w, k=3):
        return 2.0 * B * h * w * cin * cout * k * k

    def t2d_f(c, h, w, layers):
        S = h * w
        f = 2 * (2.0 * B * S * c * c)  # proj in/out
        per = 0.0
        per += 4 * 2.0 * B * S * c * c                 # self q,k,v,o
        per += 2 * 2.0 * B * S * S * c                 # self QK^T and PV
        per += 2 * 2.0 * B * S * c * c                 # cross q, o
        per += 2 * 2.0 * B * cfg.ctx_tokens * cfg.ctx_dim * c  # cross k, v
        per += 2 * 2.0 * B * S * cfg.ctx_tokens * c    # cross QK^T, PV
        per += 2.0 * B * S * c * 8 * c + 2.0 * B * S * 4 * c * c  # GEGLU proj + out
        return f + layers * per

    def res_f(cin, cout, h, w):
        f = conv_f(cin, cout, h, w) + conv_f(cout, cout, h, w)
        if cin != cout:
            f += conv_f(cin, cout, h, w, 1)
        return f

    h, w = H, W
    fl += conv_f(cfg.in_channels, C0, h, w)
    chans = [C0, C1, C2]
    cin = C0
    for lvl in range(3):
        c = chans[lvl]
        for r in range(2):
            fl += res_f(cin if r == 0 else c, c, h, w)
            if cfg.depths[lvl]:
                fl += t2d_f(c, h, w, cfg.depths[lvl])
        if lvl < 2:
            fl += conv_f(c, c, h // 2, w // 2)
            h, w = h // 2, w // 2
        cin = c
    fl += 2 * res_f(C2, C2, h, w) + t2d_f(C2, h, w, cfg.mid_depth)
    skip_ch = [C0, C0, C0, C0, C1, C1, C1, C2, C2]
    cur = C2
    for u in range(3):
        lvl = 2 - u
        c = chans[lvl]
        for r in range(3):
            fl += res_f(cur + skip_ch.pop(), c, h, w)
            cur = c
            if cfg.depths[lvl]:
                fl += t2d_f(c, h, w, cfg.depths[lvl])
        if u < 2:
            h, w = h * 2, w * 2
            fl += conv_f(c, c, h, w)
    fl += conv_f(C0, cfg.out_channels, h, w)
    return fl
