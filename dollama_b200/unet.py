"""Python host mirror of the reference's UNet handle API over the C ABI.

Mirrors `unet_weights_create` / `launch_unet_batched` / `unet_weights_destroy`
(reference src/infer/unet.cuh:90-146): the weights become device-resident once, and each
call runs one UNet step for a CFG batch.  All compute runs in `libdollama_b200.so`; this
module only marshals torch CUDA tensors' pointers.
"""
from __future__ import annotations

import ctypes
import math

import torch

from . import _lib as L


def _stream_ptr(stream=None):
    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


class SDXLUNet:
    """SDXL UNet2DConditionModel on the B200 kernels.

    `state_dict` maps diffusers key names to fp16 CUDA tensors (the reference's
    `w.get(...)` names).  `depths` / `mid_depth` default to SDXL (0, 2, 10) / 10.
    """

    def __init__(self, state_dict: dict, depths=(0, 2, 10), mid_depth: int = 10, stream=None):
        names = list(state_dict.keys())
        tens = [state_dict[n] for n in names]
        for n, t in zip(names, tens):
            if not (t.is_cuda and t.dtype == torch.float16 and t.is_contiguous()):
                raise ValueError(f"{n}: expected a contiguous fp16 CUDA tensor")
        n = len(names)
        c_names = (ctypes.c_char_p * n)(*[x.encode() for x in names])
        c_ptrs = (ctypes.c_void_p * n)(*[t.data_ptr() for t in tens])
        c_numel = (ctypes.c_int64 * n)(*[t.numel() for t in tens])
        c_depths = (ctypes.c_int * 3)(*depths)
        h = ctypes.c_void_p()
        L.call("dlm_unet_create", c_depths, int(mid_depth), n, c_names, c_ptrs, c_numel,
               ctypes.byref(h), _stream_ptr(stream))
        self._h = h
        self.depths = tuple(depths)
        self.mid_depth = mid_depth

    def forward(self, latent, timestep: float, ehs, text_embeds, time_ids, out=None, stream=None):
        """latent [B,4,H,W], ehs [B,77,2048], text_embeds [B,1280], time_ids [6] -> noise [B,4,H,W]."""
        B, _, H, W = latent.shape
        self._last_b = B
        if out is None:
            out = torch.empty_like(latent)
        for t in (latent, ehs, text_embeds, time_ids, out):
            if not (t.is_cuda and t.dtype == torch.float16 and t.is_contiguous()):
                raise ValueError("inputs must be contiguous fp16 CUDA tensors")
        L.call("dlm_unet_forward", self._h, B, H, W, ctypes.c_void_p(latent.data_ptr()),
               float(timestep), ctypes.c_void_p(ehs.data_ptr()),
               ctypes.c_void_p(text_embeds.data_ptr()), ctypes.c_void_p(time_ids.data_ptr()),
               ctypes.c_void_p(out.data_ptr()), _stream_ptr(stream))
        return out

    __call__ = forward

    def forward_host(self, latent, timestep: float, ehs, text_embeds, time_ids, out, stream=None):
        """The step on HOST tensors (pinned for full speed): copies in, runs, copies `out` back and
        returns after the result is on the host (the reference loop's per-step boundary)."""
        B, _, H, W = latent.shape
        self._last_b = B
        for t in (latent, ehs, text_embeds, time_ids, out):
            if t.is_cuda or t.dtype != torch.float16 or not t.is_contiguous():
                raise ValueError("forward_host takes contiguous fp16 host tensors")
        L.call("dlm_unet_forward_host", self._h, B, H, W, ctypes.c_void_p(latent.data_ptr()),
               float(timestep), ctypes.c_void_p(ehs.data_ptr()),
               ctypes.c_void_p(text_embeds.data_ptr()), ctypes.c_void_p(time_ids.data_ptr()),
               ctypes.c_void_p(out.data_ptr()), _stream_ptr(stream))
        return out

    OP_CLASSES = ("gemm", "attention", "groupnorm", "layernorm", "other")

    def time_ops(self, stream=None) -> dict:
        """Per op class: device ms, algorithmic FLOPs and launches of one eager step."""
        ms = (ctypes.c_double * 5)()
        fl = (ctypes.c_double * 5)()
        cnt = (ctypes.c_int * 5)()
        L.call("dlm_unet_time_ops", self._h, ms, fl, cnt, _stream_ptr(stream))
        return {k: {"ms": ms[i], "flops": fl[i], "launches": cnt[i]}
                for i, k in enumerate(self.OP_CLASSES)}

    def set_graph(self, enable: bool) -> None:
        L.call("dlm_unet_set_graph", self._h, 1 if enable else 0)

    def stage(self, name: str) -> torch.Tensor:
        """Copy of a stage output of the last forward, NCHW fp16 (the reference's stage hook)."""
        ptr = ctypes.c_void_p()
        C, H, W = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
        L.call("dlm_unet_stage", self._h, name.encode(), ctypes.byref(ptr), ctypes.byref(C),
               ctypes.byref(H), ctypes.byref(W))
        B = getattr(self, "_last_b", None)
        if B is None:
            raise RuntimeError("stage(): no forward has run yet")
        torch.cuda.synchronize()
        total = B * H.value * W.value * C.value  # B images of [H, W, C]
        out = torch.empty(total, dtype=torch.float16, device="cuda")
        L.call("dlm_memcpy", ctypes.c_void_p(out.data_ptr()), ptr, total * 2, _stream_ptr())
        torch.cuda.synchronize()
        return out.view(B, H.value, W.value, C.value).permute(0, 3, 1, 2)

    def apply_loras(self, modules, stream=None) -> None:
        """Merge LoRA modules (`dollama_b200.lora.LoraModule`, host fp16 A / B) into the resident
        weights: W += h(scale * B @ A) per module, in order (the reference's unet_apply_loras)."""
        from .lora import pack_modules
        arr, keep = pack_modules(modules)
        L.call("dlm_unet_apply_loras", self._h, arr, len(modules), _stream_ptr(stream))
        del keep

    def apply_lora(self, base_key: str, A, B, scale: float = 1.0, stream=None) -> None:
        """One module from fp16 CUDA tensors A [rank, in_flat] and B [out, rank]."""
        A, B = A.contiguous(), B.contiguous()
        L.call("dlm_unet_apply_lora", self._h, base_key.encode(), ctypes.c_void_p(A.data_ptr()),
               ctypes.c_void_p(B.data_ptr()), A.shape[0], A.shape[1], B.shape[0], float(scale),
               _stream_ptr(stream))

    def clear_loras(self, stream=None) -> None:
        """Revert every applied LoRA, bit-exact (the reference's unet_clear_loras)."""
        L.call("dlm_unet_clear_loras", self._h, _stream_ptr(stream))

    def info(self):
        a, w, n = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int()
        L.call("dlm_unet_info", self._h, ctypes.byref(a), ctypes.byref(w), ctypes.byref(n))
        return {"arena_bytes": a.value, "weight_bytes": w.value, "launches_per_step": n.value}

    def close(self):
        if getattr(self, "_h", None):
            L.lib().dlm_unet_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def weight_spec(depths=(0, 2, 10), mid_depth: int = 10) -> dict:
    """name -> shape of every tensor dlm_unet_create expects (from the C library)."""
    lib = L.lib()
    d = (ctypes.c_int * 3)(*depths)
    n = lib.dlm_unet_weight_count(d, int(mid_depth))
    out = {}
    buf = ctypes.create_string_buffer(256)
    shape = (ctypes.c_int64 * 4)()
    nd = ctypes.c_int()
    for i in range(n):
        L.call("dlm_unet_weight_info", d, int(mid_depth), i, buf, 256, shape, ctypes.byref(nd))
        out[buf.value.decode()] = tuple(shape[j] for j in range(nd.value))
    return out


_CONV_SUFFIXES = ("conv1", "conv2", "conv_shortcut", "conv_in", "conv_out", "downsamplers.0.conv",
                  "upsamplers.0.conv")


def random_weights(depths=(0, 2, 10), mid_depth: int = 10, seed: int = 7, device="cuda") -> dict:
    """Synthetic random-init weights of the named architecture, generated on `device`:
    conv weights / biases Kaiming-uniform U(+-1/sqrt(fan_in)), Linear weights and biases
    N(0, 0.02), norm gammas 1 + N(0, 0.05), betas N(0, 0.05) (fp16)."""
    g = torch.Generator(device=device).manual_seed(seed)
    spec = weight_spec(depths, mid_depth)
    sd = {}
    for name, shape in sorted(spec.items()):
        base, kind = name.rsplit(".", 1)
        if base.endswith(_CONV_SUFFIXES):
            w = spec[base + ".weight"]
            bound = 1.0 / math.sqrt(w[1] * w[2] * w[3])
            t = (torch.rand(shape, generator=g, device=device) * 2 - 1) * bound
        elif len(shape) == 1 and base.rsplit(".", 1)[-1] in ("norm", "norm1", "norm2", "norm3",
                                                              "conv_norm_out"):
            t = (1.0 if kind == "weight" else 0.0) + 0.05 * torch.randn(shape, generator=g,
                                                                        device=device)
        else:
            t = 0.02 * torch.randn(shape, generator=g, device=device)
        sd[name] = t.half()
    return sd
