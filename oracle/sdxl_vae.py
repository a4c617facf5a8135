"""CPU fp32 oracle of the SDXL AutoencoderKL decoder — TEST INFRASTRUCTURE ONLY.

The checker of the B200 VAE path; imported by tests/, smoke() and bench.py's baseline legs only.
Restates, in plain PyTorch fp32, the decoder the reference orchestrates in
src/kernels/vae_decode.cu (structure vae_decode.cuh:19-33):
  post_quant_conv (1x1, 4->4) -> conv_in (3x3, 4->512)
  mid: ResnetBlock(512) -> AttnBlock(512: GN -> q,k,v Linear -> single-head attention over
       H*W tokens, scale 1/sqrt(512) -> to_out -> + residual, vae_decode.cu:660-691) -> Resnet
  up_blocks[0..3]: 3 ResnetBlocks each (512, 512, 512->256, 256->128), nearest-2x + 3x3 conv
       upsamplers after blocks 0..2
  conv_norm_out (GN 32) -> SiLU -> conv_out (3x3, 128->3)
ResnetBlock (vae_decode.cu:575-658): GN(32, eps 1e-6)+SiLU -> conv1 -> GN+SiLU -> conv2 ->
+ (x | conv_shortcut(x)); no time embedding.  All GroupNorms use eps 1e-6 (vae_decode.cu:579,
621, 665, 704).  Keys follow the diffusers state dict the reference reads (decoder.*,
post_quant_conv.*).
Parity to the reference's golden files (dollma_dump_vae_golden.py outputs, not in the checkout)
is unpinned; this restatement is checked against per-op PyTorch definitions.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

CH = (128, 256, 512, 512)   # block_out_channels; up path runs them reversed
LATENT_C = 4
GROUPS = 32
EPS = 1e-6


_FP16_STORAGE = [False]


class fp16_storage:
    """Context manager: while active, the oracle rounds to fp16 every tensor that an fp16-storage
    decoder writes — the normalised input of every convolution, the mid attention's q / k / v and
    output, and the residual stream up to up_blocks[1] (after it the reference, and this
    library, carry fp32, vae_decode.cu:9-20) — and computes on in fp32.  Its difference from the
    plain fp32 oracle is the error fp16 storage alone costs."""

    def __enter__(self):
        _FP16_STORAGE[0] = True
        return self

    def __exit__(self, *exc):
        _FP16_STORAGE[0] = False
        return False


def _st(t, on=True):
    return t.half().float() if (_FP16_STORAGE[0] and on) else t


def _operand(t, carry16):
    """A GEMM operand: fp16 as stored, or, for an fp32 carry, fp16(t / 64) * 64 (how an fp32
    carry enters an fp16 GEMM without leaving the fp16 range)."""
    if not _FP16_STORAGE[0]:
        return t
    return t.half().float() if carry16 else (t / 64.0).half().float() * 64.0


def _conv(x, sd, name, padding=1):
    return F.conv2d(x, sd[name + ".weight"].float(), sd[name + ".bias"].float(), padding=padding)


def _gn(x, sd, name):
    return F.group_norm(x, GROUPS, sd[name + ".weight"].float(), sd[name + ".bias"].float(), EPS)


def resnet(x, sd, p, carry16=False, in16=None):
    """carry16: this block's outputs are stored fp16 (else fp32 carries); in16: its input is
    fp16 (defaults to carry16)."""
    in16 = carry16 if in16 is None else in16
    h = _conv(_st(F.silu(_gn(x, sd, p + "norm1"))), sd, p + "conv1")
    h = _st(h, carry16)
    h = _conv(_st(F.silu(_gn(h, sd, p + "norm2"))), sd, p + "conv2")
    if (p + "conv_shortcut.weight") in sd:
        x = _conv(_operand(x, in16), sd, p + "conv_shortcut", padding=0)
    return _st(x + h, carry16)


def mid_attention(q, k, v):
    """Single-head softmax(q k^T / sqrt(C)) v over [B, S, C] (vae_decode.cu:660-691)."""
    s = (q @ k.transpose(1, 2)) * (1.0 / math.sqrt(q.shape[-1]))
    return torch.softmax(s, dim=-1) @ v


def attn_block(x, sd, p):
    B, C, H, W = x.shape
    h = _st(_gn(x, sd, p + "group_norm")).permute(0, 2, 3, 1).reshape(B, H * W, C)
    lin = lambda t, n: F.linear(t, sd[p + n + ".weight"].float(), sd[p + n + ".bias"].float())
    q, k, v = _st(lin(h, "to_q")), _st(lin(h, "to_k")), _st(lin(h, "to_v"))
    o = _st(mid_attention(q, k, v))
    o = lin(o, "to_out.0").reshape(B, H, W, C).permute(0, 3, 1, 2)
    return _st(x + o)


def vae_decode(sd, latent, hook=None):
    """latent [B,4,h,w] (already divided by the scaling factor) -> image [B,3,8h,8w], fp32."""
    def tap(n, t):
        if hook is not None:
            hook(n, t)
        return t

    x = _st(_conv(latent.float(), sd, "post_quant_conv", padding=0))
    x = _st(_conv(x, sd, "decoder.conv_in"))
    x = resnet(x, sd, "decoder.mid_block.resnets.0.", True)
    x = attn_block(x, sd, "decoder.mid_block.attentions.0.")
    x = resnet(x, sd, "decoder.mid_block.resnets.1.", True)
    tap("mid_block_out", x)
    for u in range(4):
        for r in range(3):
            x = resnet(x, sd, f"decoder.up_blocks.{u}.resnets.{r}.", u < 2, u < 2 or (u == 2 and r == 0))
        if u < 3:
            x = F.interpolate(x, scale_factor=2.0, mode="nearest")
            x = _conv(_operand(x, u < 2), sd, f"decoder.up_blocks.{u}.upsamplers.0.conv")
            x = _st(x, u < 2)
        tap(f"up_block_{u}_out", x)
    x = _st(F.silu(_gn(x, sd, "decoder.conv_norm_out")))
    return tap("image", _conv(x, sd, "decoder.conv_out"))


def weight_shapes() -> dict:
    S = {}

    def cv(n, o, i, k=3):
        S[n + ".weight"] = (o, i, k, k)
        S[n + ".bias"] = (o,)

    def nrm(n, c):
        S[n + ".weight"] = (c,)
        S[n + ".bias"] = (c,)

    def res(p, cin, cout):
        nrm(p + "norm1", cin)
        cv(p + "conv1", cout, cin)
        nrm(p + "norm2", cout)
        cv(p + "conv2", cout, cout)
        if cin != cout:
            cv(p + "conv_shortcut", cout, cin, 1)

    cv("post_quant_conv", LATENT_C, LATENT_C, 1)
    top = CH[-1]
    cv("decoder.conv_in", top, LATENT_C)
    res("decoder.mid_block.resnets.0.", top, top)
    p = "decoder.mid_block.attentions.0."
    nrm(p + "group_norm", top)
    for n in ("to_q", "to_k", "to_v", "to_out.0"):
        S[p + n + ".weight"] = (top, top)
        S[p + n + ".bias"] = (top,)
    res("decoder.mid_block.resnets.1.", top, top)
    rev = list(reversed(CH))  # 512, 512, 256, 128
    cin = top
    for u in range(4):
        c = rev[u]
        for r in range(3):
            res(f"decoder.up_blocks.{u}.resnets.{r}.", cin if r == 0 else c, c)
        cin = c
        if u < 3:
            cv(f"decoder.up_blocks.{u}.upsamplers.0.conv", c, c)
    nrm("decoder.conv_norm_out", CH[0])
    cv("decoder.conv_out", 3, CH[0])
    return S


def init_weights(seed: int = 9, device="cpu", dtype=torch.float16):
    """Random init: conv weights / biases Kaiming-uniform U(+-1/sqrt(fan_in)), Linear weights
    N(0, 0.02), Linear biases N(0, 0.02), norm gammas 1 + N(0, 0.05), betas N(0, 0.05)."""
    g = torch.Generator(device=device).manual_seed(seed)
    shapes = weight_shapes()
    sd = {}
    for name, shape in sorted(shapes.items()):
        base, kind = name.rsplit(".", 1)
        wshape = shapes.get(base + ".weight")
        if wshape is not None and len(wshape) == 4:
            bound = 1.0 / math.sqrt(wshape[1] * wshape[2] * wshape[3])
            t = (torch.rand(shape, generator=g, device=device) * 2 - 1) * bound
        elif len(shape) == 1 and base.rsplit(".", 1)[-1] in ("norm1", "norm2", "group_norm",
                                                              "conv_norm_out"):
            t = (1.0 if kind == "weight" else 0.0) + 0.05 * torch.randn(shape, generator=g,
                                                                        device=device)
        else:
            t = 0.02 * torch.randn(shape, generator=g, device=device)
        sd[name] = t.to(dtype)
    return sd


def vae_flops(B: int, h: int, w: int) -> float:
    """Algorithmic FLOPs (2 per MAC) of one decode of [B,4,h,w]."""
    fl = 0.0

    def conv(cin, cout, hh, ww, k=3):
        return 2.0 * B * hh * ww * cin * cout * k * k

    def res(cin, cout, hh, ww):
        f = conv(cin, cout, hh, ww) + conv(cout, cout, hh, ww)
        return f + (conv(cin, cout, hh, ww, 1) if cin != cout else 0.0)

    top = CH[-1]
    fl += conv(LATENT_C, LATENT_C, h, w, 1) + conv(LATENT_C, top, h, w)
    S = h * w
    fl += 2 * res(top, top, h, w) + 4 * 2.0 * B * S * top * top + 2 * 2.0 * B * S * S * top
    rev = list(reversed(CH))
    cin, hh, ww = top, h, w
    for u in range(4):
        c = rev[u]
        for r in range(3):
            fl += res(cin if r == 0 else c, c, hh, ww)
        cin = c
        if u < 3:
            hh, ww = hh * 2, ww * 2
            fl += conv(c, c, hh, ww)
    fl += conv(CH[0], 3, hh, ww)
    return fl
