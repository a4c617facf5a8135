"""SDXL txt2img denoising on the device: the reference's DiffusionPipeline::generate_txt2img loop
(src/infer/diffusion.cu:896-988, Euler scheduler src/infer/scheduler.hpp) without its per-step
host round trip.  Thin ctypes wrapper over dlm_sdxl_*; all compute runs in libdollama_b200.so."""
from __future__ import annotations

import ctypes

import torch

from . import _lib as L

VAE_SCALING = 0.13025   # the reference's default VAE scaling factor (src/infer/diffusion.cuh:28)


def euler_schedule(steps: int):
    """(sigmas [steps + 1], timesteps [steps]) of the SDXL Euler schedule."""
    sig = (ctypes.c_float * (steps + 1))()
    ts = (ctypes.c_float * steps)()
    L.call("dlm_sdxl_schedule", steps, sig, ts)
    return list(sig), list(ts)


def _s(stream=None):
    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def denoise(unet, init_latent, ehs, text_embeds, time_ids, steps=20, guidance=7.5, stream=None):
    """init_latent [1, 4, H, W] fp32 CUDA (randn * sigmas[0]); ehs [2, 77, 2048], text_embeds
    [2, 1280] (cond, uncond), time_ids [6] fp16 CUDA -> final latent [1, 4, H, W] fp32."""
    _, _, H, W = init_latent.shape
    out = torch.empty_like(init_latent)
    L.call("dlm_sdxl_denoise", unet._h, H, W, _p(init_latent), int(steps), float(guidance),
           _p(ehs), _p(text_embeds), _p(time_ids), _p(out), _s(stream))
    return out


def generate(unet, vae, init_latent, ehs, text_embeds, time_ids, steps=20, guidance=7.5,
             vae_scaling=VAE_SCALING, stream=None):
    """The denoising loop followed by the VAE decode: image [1, 3, 8H, 8W] fp16 CUDA."""
    _, _, H, W = init_latent.shape
    img = torch.empty(1, 3, 8 * H, 8 * W, dtype=torch.float16, device=init_latent.device)
    L.call("dlm_sdxl_generate", unet._h, vae._h, H, W, _p(init_latent), int(steps), float(guidance),
           _p(ehs), _p(text_embeds), _p(time_ids), float(vae_scaling), _p(img), _s(stream))
    return img
