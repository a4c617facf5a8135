"""GPU tests of the reference-side C++ binding (include/dollama_b200_shim.hpp): a C++ program
(tests/shim/shim_driver.cpp) calls the library only through the reference's own function names
and types — SafeTensors, unet_weights_create / launch_unet_batched / unet_weight_device_ptr,
launch_vae_decode(const SafeTensors&, ...), NCHW launch_conv2d (tensor-core and direct shapes),
launch_group_norm[_silu], launch_attention — and its outputs are checked here: the model calls
bit-identical to the library's Python API on the same weights, the kernels against fp32 torch."""
import subprocess
import tempfile
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from tests.helpers import max_rel_err
from tests.shim.build_shim_driver import OUT as DRIVER

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not DRIVER.exists(), reason="shim driver not built")]


def _w(d, name, t):
    t.detach().cpu().contiguous().half().numpy().tofile(str(Path(d) / name))


def _r(d, name, shape):
    return torch.from_numpy(np.fromfile(str(Path(d) / name), dtype=np.float16)).reshape(shape)


def _run(cmd, d):
    r = subprocess.run([str(DRIVER), cmd, str(d)], capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stderr


def test_shim_unet_matches_python_api_bit_for_bit():
    from baseline.ref_gpu import write_safetensors
    from dollama_b200.unet import SDXLUNet
    from oracle.sdxl_unet import init_weights, make_inputs
    sd = init_weights(seed=7)
    lat, ehs, te, tid = make_inputs(2, 128, 128, seed=6)
    with tempfile.TemporaryDirectory() as d:
        write_safetensors(sd, str(Path(d) / "unet.safetensors"))
        g = torch.Generator().manual_seed(5)
        la = (torch.randn(4, 36, generator=g) * 0.1).half()
        lb = (torch.randn(320, 4, generator=g) * 0.1).half()
        for n, t in (("lat.bin", lat), ("ehs.bin", ehs), ("te.bin", te), ("tid.bin", tid),
                     ("lora_a.bin", la), ("lora_b.bin", lb)):
            _w(d, n, t)
        _run("unet", d)
        got = _r(d, "noise.bin", lat.shape)
        w = _r(d, "conv_in_weight.bin", sd["conv_in.weight"].shape)
        wl = _r(d, "conv_in_weight_lora.bin", sd["conv_in.weight"].shape)
        got_lora = _r(d, "noise_lora.bin", lat.shape)
        got_clear = _r(d, "noise_clear.bin", lat.shape)
    assert torch.equal(w, sd["conv_in.weight"])
    # the reference's merge: delta = fp16(scale * B @ A), W = fp16(W + delta)
    delta = (0.5 * (lb.float() @ la.float())).half().float()
    want = (sd["conv_in.weight"].float().reshape(320, 36) + delta).half().reshape(wl.shape)
    assert (wl.float() - want.float()).abs().max().item() <= 2 * 2 ** -10 * want.float().abs().max().item()
    assert torch.equal(got_clear, got) and not torch.equal(got_lora, got)
    net = SDXLUNet({k: v.cuda() for k, v in sd.items()})
    ref = net(lat.cuda(), 999.0, ehs.cuda(), te.cuda(), tid.cuda()).cpu()
    net.close()
    assert torch.equal(got, ref)


def test_shim_vae_per_call_decode_matches_python_api_bit_for_bit():
    from baseline.ref_gpu import write_safetensors
    from dollama_b200.vae import SDXLVAEDecoder
    from oracle.sdxl_vae import init_weights
    sd = init_weights(seed=9)
    lat = torch.randn(1, 4, 128, 128, generator=torch.Generator().manual_seed(8)).half()
    with tempfile.TemporaryDirectory() as d:
        write_safetensors(sd, str(Path(d) / "vae.safetensors"))
        _w(d, "lat.bin", lat)
        _run("vae", d)
        got = _r(d, "image.bin", (1, 3, 1024, 1024))
    dec = SDXLVAEDecoder({k: v.cuda() for k, v in sd.items()})
    ref = dec(lat.cuda()).cpu()
    dec.close()
    assert torch.equal(got, ref)


def test_shim_kernel_entries_match_fp32_torch():
    g = torch.Generator().manual_seed(21)
    cx = torch.randn(2, 64, 32, 32, generator=g).half()
    cw = (torch.randn(128, 64, 3, 3, generator=g) * 0.05).half()
    cb = (torch.randn(128, generator=g) * 0.1).half()
    dx = torch.randn(1, 3, 17, 19, generator=g).half()
    dw = (torch.randn(5, 3, 3, 3, generator=g) * 0.2).half()
    db = (torch.randn(5, generator=g) * 0.1).half()
    gx = (torch.randn(2, 320, 16, 16, generator=g) * 2 + 0.5).half()
    gg = (1 + 0.1 * torch.randn(320, generator=g)).half()
    gb = (0.1 * torch.randn(320, generator=g)).half()
    aq, ak, av = (torch.randn(1, 2, 256, 64, generator=g).half() for _ in range(3))
    with tempfile.TemporaryDirectory() as d:
        for n, t in (("cx.bin", cx), ("cw.bin", cw), ("cb.bin", cb), ("dx.bin", dx), ("dw.bin", dw),
                     ("db.bin", db), ("gx.bin", gx), ("gg.bin", gg), ("gb.bin", gb),
                     ("aq.bin", aq), ("ak.bin", ak), ("av.bin", av)):
            _w(d, n, t)
        _run("ops", d)
        conv = _r(d, "conv_out.bin", (2, 128, 32, 32))
        dconv = _r(d, "dconv_out.bin", (1, 5, 9, 10))
        gns = _r(d, "gn_silu_out.bin", gx.shape)
        gni = _r(d, "gn_inplace_out.bin", gx.shape)
        att = _r(d, "attn_out.bin", aq.shape)
    ref = F.conv2d(cx.float(), cw.float(), cb.float(), padding=1)
    assert max_rel_err(conv, ref) < 2e-3
    ref = F.conv2d(dx.float(), dw.float(), db.float(), stride=2, padding=1)
    assert max_rel_err(dconv, ref) < 1e-3
    gn = F.group_norm(gx.float(), 32, gg.float(), gb.float(), 1e-5)
    assert max_rel_err(gns, F.silu(gn.half().float())) < 2e-3
    gn6 = F.group_norm(gx.float(), 32, gg.float(), gb.float(), 1e-6)
    assert max_rel_err(gni, gn6) < 2e-3
    s = torch.softmax(aq.float() @ ak.float().transpose(-1, -2) * 0.125, dim=-1)
    assert max_rel_err(att, s @ av.float()) < 2e-3


def _seeded_normal(seed, n):
    """The reference's initial-noise generator (src/infer/diffusion.cu:76-140), restated in
    Python for the check: splitmix64-seeded xorshift128+ uniforms, Box-Muller pairs in double."""
    M = (1 << 64) - 1

    def mix(z):
        z = (z + 0x9E3779B97F4A7C15) & M
        z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & M
        z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & M
        return z ^ (z >> 31)

    a, b = mix(seed), mix((seed + 0x9E3779B97F4A7C15) & M)
    out, spare = [], None

    def uniform():
        nonlocal a, b
        s1, s0 = a, b
        a = s0
        s1 ^= (s1 << 23) & M
        b = s1 ^ s0 ^ (s1 >> 17) ^ (s0 >> 26)
        return float(((b + s0) & M) >> 11) * (1.0 / 9007199254740992.0)

    import math
    while len(out) < n:
        if spare is not None:
            out.append(spare)
            spare = None
            continue
        u1 = uniform()
        while u1 <= 1e-12:
            u1 = uniform()
        u2 = uniform()
        r = math.sqrt(-2.0 * math.log(u1))
        out.append(r * math.cos(2.0 * math.pi * u2))
        spare = r * math.sin(2.0 * math.pi * u2)
    return out


def test_shim_runner_txt2img_is_the_python_pipeline_bit_for_bit():
    """The reference's diffusion-runner plugin (IDiffusionRunner, include/dollama_b200_runner.hpp)
    through its own factory: the initial latent follows the reference's seeded generator, and the
    RGB8 image equals the Python pipeline's decode of the same latent and conditioning converted
    with the reference's rule."""
    from baseline.ref_gpu import write_safetensors
    from dollama_b200.pipeline import euler_schedule, generate
    from dollama_b200.unet import SDXLUNet
    from dollama_b200.vae import SDXLVAEDecoder
    from oracle.sdxl_unet import init_weights
    from oracle.sdxl_vae import init_weights as vae_init
    sd, sdv = init_weights(seed=7), vae_init(seed=9)
    g = torch.Generator().manual_seed(31)
    ce, ue = torch.randn(77, 2048, generator=g), torch.randn(77, 2048, generator=g)
    ct, ut = torch.randn(1280, generator=g), torch.randn(1280, generator=g)
    tid = torch.tensor([1024.0, 1024.0, 0.0, 0.0, 1024.0, 1024.0])
    with tempfile.TemporaryDirectory() as d:
        write_safetensors(sd, str(Path(d) / "unet.safetensors"))
        write_safetensors(sdv, str(Path(d) / "vae.safetensors"))
        for n, t in (("cond_ehs.f32", ce), ("uncond_ehs.f32", ue), ("cond_te.f32", ct),
                     ("uncond_te.f32", ut), ("tid.f32", tid)):
            t.numpy().astype(np.float32).tofile(str(Path(d) / n))
        _run("runner", d)
        rgb = np.fromfile(str(Path(d) / "rgb.bin"), dtype=np.uint8).reshape(1024, 1024, 3)
        lat0 = torch.from_numpy(np.fromfile(str(Path(d) / "lat0.bin"), dtype=np.float32))
    sig, _ = euler_schedule(4)
    want0 = torch.tensor(_seeded_normal(1234, 64), dtype=torch.float64) * sig[0]
    assert torch.equal(lat0[:64], want0.float())
    net = SDXLUNet({k: v.cuda() for k, v in sd.items()})
    vae = SDXLVAEDecoder({k: v.cuda() for k, v in sdv.items()})
    ehs = torch.stack([ce, ue]).half().cuda()
    te = torch.stack([ct, ut]).half().cuda()
    img = generate(net, vae, lat0.view(1, 4, 128, 128).cuda(), ehs, te, tid.half().cuda(), steps=4,
                   guidance=7.5)
    torch.cuda.synchronize()
    net.close()
    vae.close()
    x = img[0].float().cpu().numpy() * np.float32(0.5) + np.float32(0.5)
    q = np.floor(np.clip(x, 0.0, 1.0) * np.float32(255.0) + np.float32(0.5)).astype(np.int32)
    want = np.clip(q, 0, 255).astype(np.uint8).transpose(1, 2, 0)
    assert np.array_equal(rgb, want)
