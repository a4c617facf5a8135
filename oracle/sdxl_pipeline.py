"""CPU oracle of the SDXL txt2img denoising loop — TEST INFRASTRUCTURE ONLY.

Restates the reference's EulerDiscreteScheduler (src/infer/scheduler.hpp: scaled_linear betas
0.00085..0.012 over 1000 training steps, "leading" spacing with steps_offset 1, np.interp of the
training sigmas, scale_model_input :110-119, epsilon Euler step :126-140) and the CFG loop of
DiffusionPipeline::generate_txt2img (src/infer/diffusion.cu:896-976) around the fp32 UNet oracle.
"""
from __future__ import annotations

import numpy as np
import torch

from oracle.sdxl_unet import unet_forward


def euler_schedule(steps: int):
    n_train = 1000
    sqrt_beta = np.linspace(np.sqrt(0.00085), np.sqrt(0.012), n_train, dtype=np.float64)
    alphas_cumprod = np.cumprod(1.0 - sqrt_beta ** 2)
    train = np.sqrt((1.0 - alphas_cumprod) / alphas_cumprod)
    ratio = n_train // steps
    ts = (np.round(np.arange(steps, dtype=np.float64) * ratio) + 1.0)[::-1]
    sig = np.interp(ts, np.arange(n_train, dtype=np.float64), train)
    sigmas = np.concatenate([sig, [0.0]]).astype(np.float32)
    return sigmas, ts.astype(np.float32)


def scale_input(x: torch.Tensor, sigma: float) -> torch.Tensor:
    """scale_model_input (scheduler.hpp:110-119): fp32(double(x) / sqrt(sigma^2 + 1))."""
    return (x.double() * (1.0 / np.sqrt(float(sigma) ** 2 + 1.0))).float()


def euler_step(x: torch.Tensor, eps: torch.Tensor, sigma: float, sigma_next: float) -> torch.Tensor:
    """Epsilon Euler step (scheduler.hpp:126-140): fp32(double(x) + double(eps) * (sigma' - sigma))."""
    return (x.double() + eps.double() * (float(sigma_next) - float(sigma))).float()


def denoise(sd, cfg, init_latent, ehs, te, tid, steps, guidance):
    """init_latent [1, 4, H, W] fp32; ehs [2, 77, 2048], te [2, 1280] (cond, uncond), tid [6] ->
    final latent [1, 4, H, W] fp32 (UNet in fp32)."""
    sigmas, ts = euler_schedule(steps)
    x = init_latent.float()
    with torch.no_grad():
        for i in range(steps):
            xin = scale_input(x, sigmas[i]).expand(2, -1, -1, -1).contiguous()
            noise = unet_forward(sd, xin, float(ts[i]), ehs.float(), te.float(), tid.float(), cfg)
            e = noise[1] + guidance * (noise[0] - noise[1])
            x = euler_step(x, e, sigmas[i], sigmas[i + 1])
    return x.float()
