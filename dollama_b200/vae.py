"""Python host mirror of the reference's VAE handle API over the C ABI.

Mirrors `vae_weights_create` / `launch_vae_decode(handle, d_latent, d_image_out)` /
`vae_weights_destroy` (reference src/kernels/vae_decode.cuh:66-75): the decoder weights become
device-resident once and each call decodes a latent batch to an fp16 image.  All compute runs in
`libdollama_b200.so`; this module only marshals torch CUDA tensors' pointers.
"""
from __future__ import annotations

import ctypes
import math

import torch

from . import _lib as L

STAGES = ("mid_block_out", "up_block_0_out", "up_block_1_out", "up_block_2_out", "up_block_3_out")


def _stream_ptr(stream=None):
    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


class SDXLVAEDecoder:
    """SDXL AutoencoderKL decoder on the B200 kernels.

    `state_dict` maps diffusers key names (decoder.*, post_quant_conv.*) to fp16 CUDA tensors.
    """

    def __init__(self, state_dict: dict, stream=None):
        names = list(state_dict.keys())
        tens = [state_dict[n] for n in names]
        for n, t in zip(names, tens):
            if not (t.is_cuda and t.dtype == torch.float16 and t.is_contiguous()):
                raise ValueError(f"{n}: expected a contiguous fp16 CUDA tensor")
        n = len(names)
        c_names = (ctypes.c_char_p * n)(*[x.encode() for x in names])
        c_ptrs = (ctypes.c_void_p * n)(*[t.data_ptr() for t in tens])
        c_numel = (ctypes.c_int64 * n)(*[t.numel() for t in tens])
        h = ctypes.c_void_p()
        L.call("dlm_vae_create", n, c_names, c_ptrs, c_numel, ctypes.byref(h), _stream_ptr(stream))
        self._h = h

    def decode(self, latent, out=None, stream=None):
        """latent [B,4,h,w] fp16 CUDA (already divided by the scaling factor) -> image [B,3,8h,8w]."""
        B, C, h, w = latent.shape
        if C != 4:
            raise ValueError("latent must have 4 channels")
        self._last_b = B
        if out is None:
            out = torch.empty(B, 3, 8 * h, 8 * w, dtype=torch.float16, device=latent.device)
        for t in (latent, out):
            if not (t.is_cuda and t.dtype == torch.float16 and t.is_contiguous()):
                raise ValueError("latent / image must be contiguous fp16 CUDA tensors")
        L.call("dlm_vae_decode", self._h, B, h, w, ctypes.c_void_p(latent.data_ptr()),
               ctypes.c_void_p(out.data_ptr()), _stream_ptr(stream))
        return out

    __call__ = decode

    def decode_host(self, latent, out, stream=None):
        """The decode on HOST tensors (pinned for full speed); returns once `out` is on the host."""
        B, _, h, w = latent.shape
        self._last_b = B
        for t in (latent, out):
            if t.is_cuda or t.dtype != torch.float16 or not t.is_contiguous():
                raise ValueError("decode_host takes contiguous fp16 host tensors")
        L.call("dlm_vae_decode_host", self._h, B, h, w, ctypes.c_void_p(latent.data_ptr()),
               ctypes.c_void_p(out.data_ptr()), _stream_ptr(stream))
        return out

    OP_CLASSES = ("gemm", "attention", "groupnorm", "layernorm", "other")

    def time_ops(self, stream=None) -> dict:
        """Per op class: device ms, algorithmic FLOPs and launches of one eager decode."""
        ms = (ctypes.c_double * 5)()
        fl = (ctypes.c_double * 5)()
        cnt = (ctypes.c_int * 5)()
        L.call("dlm_vae_time_ops", self._h, ms, fl, cnt, _stream_ptr(stream))
        return {k: {"ms": ms[i], "flops": fl[i], "launches": cnt[i]}
                for i, k in enumerate(self.OP_CLASSES)}

    def set_graph(self, enable: bool) -> None:
        L.call("dlm_vae_set_graph", self._h, 1 if enable else 0)

    def stage(self, name: str) -> torch.Tensor:
        """Copy of a stage output of the last decode as NCHW (fp16 or fp32, as computed)."""
        ptr = ctypes.c_void_p()
        dt, C, H, W = ctypes.c_int(), ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
        L.call("dlm_vae_stage", self._h, name.encode(), ctypes.byref(ptr), ctypes.byref(dt),
               ctypes.byref(C), ctypes.byref(H), ctypes.byref(W))
        B = getattr(self, "_last_b", None)
        if B is None:
            raise RuntimeError("stage(): no decode has run yet")
        dtype = torch.float32 if dt.value == 1 else torch.float16
        torch.cuda.synchronize()
        total = B * H.value * W.value * C.value
        out = torch.empty(total, dtype=dtype, device="cuda")
        L.call("dlm_memcpy", ctypes.c_void_p(out.data_ptr()), ptr, total * out.element_size(),
               _stream_ptr())
        torch.cuda.synchronize()
        return out.view(B, H.value, W.value, C.value).permute(0, 3, 1, 2)

    def info(self):
        a, w, n = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int()
        L.call("dlm_vae_info", self._h, ctypes.byref(a), ctypes.byref(w), ctypes.byref(n))
        return {"arena_bytes": a.value, "weight_bytes": w.value, "launches_per_decode": n.value}

    def close(self):
        if getattr(self, "_h", None):
            L.lib().dlm_vae_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def weight_spec() -> dict:
    """name -> shape of every tensor dlm_vae_create expects (from the C library)."""
    lib = L.lib()
    n = lib.dlm_vae_weight_count()
    out = {}
    buf = ctypes.create_string_buffer(256)
    shape = (ctypes.c_int64 * 4)()
    nd = ctypes.c_int()
    for i in range(n):
        L.call("dlm_vae_weight_info", i, buf, 256, shape, ctypes.byref(nd))
        out[buf.value.decode()] = tuple(shape[j] for j in range(nd.value))
    return out


_NORMS = ("norm1", "norm2", "group_norm", "conv_norm_out")


def random_weights(seed: int = 9, device="cuda") -> dict:
    """Synthetic random-init decoder weights, generated on `device`: conv weights / biases
    Kaiming-uniform U(+-1/sqrt(fan_in)), Linear weights and biases N(0, 0.02), norm gammas
    1 + N(0, 0.05), betas N(0, 0.05) (fp16)."""
    g = torch.Generator(device=device).manual_seed(seed)
    spec = weight_spec()
    sd = {}
    for name, shape in sorted(spec.items()):
        base, kind = name.rsplit(".", 1)
        wshape = spec.get(base + ".weight")
        if wshape is not None and len(wshape) == 4:
            bound = 1.0 / math.sqrt(wshape[1] * wshape[2] * wshape[3])
            t = (torch.rand(shape, generator=g, device=device) * 2 - 1) * bound
        elif len(shape) == 1 and base.rsplit(".", 1)[-1] in _NORMS:
            t = (1.0 if kind == "weight" else 0.0) + 0.05 * torch.randn(shape, generator=g,
                                                                        device=device)
        else:
            t = 0.02 * torch.randn(shape, generator=g, device=device)
        sd[name] = t.half()
    return sd
