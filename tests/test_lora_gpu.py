"""Runtime LoRA on the resident UNet weights against the CPU oracle, as the reference's
test_lora_runtime.cu checks it ([2] parity after apply, [3] bit-exact revert, [4] two LoRAs
stack): here through the forward, since the handle keeps its weights repacked and
LayerNorm-folded.

  * apply: the step's outputs match the oracle UNet run on W + h(scale * B @ A) (fp16 merged
    weights; the same SSIM / max-rel bars as the plain UNet parity test), and they moved far
    more than that tolerance away from the base outputs, so every merged key takes part;
  * stack: a second module set on top matches the oracle on W + d1 + d2 (two fp16 roundings);
  * clear: the step is bit-identical to the step before the first apply.
Every kind of prepared target is covered: packed 3x3 convs (conv_in with padded input channels,
conv_out with padded rows, resnet conv1 / conv2, samplers), the 1x1 shortcut stored after
conv2's columns, time_emb_proj rows in the concatenated projection, q / k / v inside the
q|k|v matrix with the LayerNorm fold, cross-attention q (folded) and k / v in the concatenated
context projection, the GEGLU projection (row interleave + fold), and plain linears.
"""
import numpy as np
import pytest
import torch

from oracle.metrics import max_rel_err, ssim_uniform
from oracle.sdxl_unet import UNetConfig, init_weights, make_inputs, unet_forward

pytestmark = pytest.mark.gpu

CFG = UNetConfig(depths=(0, 1, 1), mid_depth=1)
TB = "down_blocks.1.attentions.0.transformer_blocks.0."
MB = "mid_block.attentions.0.transformer_blocks.0."
KEYS_1 = [
    "conv_in.weight", "conv_out.weight",
    "down_blocks.0.resnets.0.conv1.weight", "down_blocks.1.resnets.0.conv1.weight",
    "down_blocks.1.resnets.0.conv2.weight", "down_blocks.1.resnets.0.conv_shortcut.weight",
    "down_blocks.1.resnets.0.time_emb_proj.weight", "down_blocks.0.downsamplers.0.conv.weight",
    "up_blocks.1.upsamplers.0.conv.weight", "time_embedding.linear_1.weight",
    "add_embedding.linear_2.weight", "down_blocks.1.attentions.0.proj_in.weight",
    TB + "attn1.to_q.weight", TB + "attn1.to_k.weight", TB + "attn1.to_v.weight",
    TB + "attn1.to_out.0.weight", TB + "attn2.to_q.weight", TB + "attn2.to_k.weight",
    TB + "attn2.to_v.weight", TB + "ff.net.0.proj.weight", TB + "ff.net.2.weight",
    MB + "attn2.to_v.weight", MB + "ff.net.0.proj.weight",
]
KEYS_2 = [TB + "attn1.to_k.weight", "down_blocks.1.resnets.0.conv2.weight",
          "up_blocks.0.resnets.2.conv_shortcut.weight", MB + "attn1.to_q.weight"]


def _kohya(seed, keys, shapes, rank=4):
    """A synthetic kohya LoRA over `keys`: |delta| ~ 1/4 of a linear weight's spread."""
    r = np.random.default_rng(seed)
    lora = {}
    for k in keys:
        shp = shapes[k]
        name = "lora_unet_" + k[: -len(".weight")].replace(".", "_")
        lora[name + ".lora_down.weight"] = (0.1 * r.standard_normal((rank,) + tuple(shp[1:]))).astype(np.float16)
        lora[name + ".lora_up.weight"] = (0.025 * r.standard_normal((shp[0], rank) + (1,) * (len(shp) - 2))).astype(np.float16)
        lora[name + ".alpha"] = np.array(rank / 2.0, dtype=np.float32)
    return lora


def _merge(sd, mods):
    """Oracle merge: W = h(W + h(scale * (B @ A))) in fp32, per module in order."""
    out = dict(sd)
    for m in mods:
        w = out[m.base_key]
        d = (torch.from_numpy(m.b_fp16.astype(np.float32)) @ torch.from_numpy(m.a_fp16.astype(np.float32)))
        d = (m.scale * d).half().float().reshape(w.shape)
        out[m.base_key] = (w.float() + d).half()
    return out


def _oracle(sd, inputs):
    lat, ehs, te, tid = inputs
    with torch.no_grad():
        sdf = {k: v.float() for k, v in sd.items()}
        return unet_forward(sdf, lat, 500.0, ehs, te, tid, CFG)


def test_lora_apply_stack_clear():
    from dollama_b200.lora import load_lora_modules
    from dollama_b200.unet import SDXLUNet, weight_spec

    shapes = weight_spec(CFG.depths, CFG.mid_depth)
    sd = init_weights(CFG, seed=7)
    inputs = make_inputs(2, 64, 64, seed=6, cfg=CFG)
    net = SDXLUNet({k: v.cuda() for k, v in sd.items()}, depths=CFG.depths, mid_depth=CFG.mid_depth)
    dev = [t.cuda() for t in inputs]

    def step():
        y = net(dev[0], 500.0, dev[1], dev[2], dev[3]).clone()
        torch.cuda.synchronize()
        return y

    base = step()
    assert torch.equal(base, step())  # the step is deterministic, so the revert can be exact

    mods1, rep = load_lora_modules(shapes, _kohya(1, KEYS_1, shapes), strength=0.8)
    assert rep.modules == len(KEYS_1)
    net.apply_loras(mods1)
    got1 = step().float().cpu()
    sd1 = _merge(sd, mods1)
    ref1 = _oracle(sd1, inputs)
    s1, e1 = ssim_uniform(got1.numpy(), ref1.numpy()), max_rel_err(got1.numpy(), ref1.numpy())
    moved = max_rel_err(got1.numpy(), base.float().cpu().numpy())
    print(f"lora x1: SSIM {s1:.6f} max_rel {e1:.2e}; moved from base by {moved:.2e}")
    assert s1 >= 0.9999 and e1 < 1e-2
    assert moved > 10 * e1

    mods2, _ = load_lora_modules(shapes, _kohya(2, KEYS_2, shapes), strength=1.0)
    net.apply_loras(mods2)
    got2 = step().float().cpu()
    ref2 = _oracle(_merge(sd1, mods2), inputs)
    s2, e2 = ssim_uniform(got2.numpy(), ref2.numpy()), max_rel_err(got2.numpy(), ref2.numpy())
    print(f"lora x2: SSIM {s2:.6f} max_rel {e2:.2e}")
    assert s2 >= 0.9999 and e2 < 2e-2

    net.clear_loras()
    assert torch.equal(step(), base)
    # a second apply / clear cycle through the device-tensor entry
    m = mods1[0]
    net.apply_lora(m.base_key, torch.from_numpy(m.a_fp16).cuda(), torch.from_numpy(m.b_fp16).cuda(),
                   m.scale)
    assert not torch.equal(step(), base)
    net.clear_loras()
    assert torch.equal(step(), base)
    net.close()


def test_lora_rejects_bad_modules():
    from dollama_b200 import _lib as L
    from dollama_b200.lora import LoraModule
    from dollama_b200.unet import SDXLUNet, weight_spec

    shapes = weight_spec(CFG.depths, CFG.mid_depth)
    sd = init_weights(CFG, seed=3)
    net = SDXLUNet({k: v.cuda() for k, v in sd.items()}, depths=CFG.depths, mid_depth=CFG.mid_depth)
    out, inn = shapes[TB + "attn1.to_q.weight"]
    a = np.zeros((2, inn), np.float16)
    b = np.zeros((out, 2), np.float16)
    with pytest.raises(L.DlmError):
        net.apply_loras([LoraModule("no.such.weight", a, b, 2, inn, out)])
    with pytest.raises(L.DlmError):
        net.apply_loras([LoraModule(TB + "attn1.to_q.weight", np.zeros((2, inn - 1), np.float16), b, 2,
                                    inn - 1, out)])
    with pytest.raises(L.DlmError):  # a norm vector is not a matrix
        net.apply_loras([LoraModule(TB + "norm1.weight", a, b, 2, inn, out)])
    net.clear_loras()
    net.close()
