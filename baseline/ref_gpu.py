"""ctypes view of baseline/_ref_gpu/libref_sdxl_gpu.so: the reference's own CUDA SDXL UNet and
VAE decoder, unchanged, recompiled for sm_100a (built by baseline/build_ref_gpu.py).

A comparator and the whole-model pin of the CPU oracle — used by the tests and by bench.py's
comparator leg, never by dollama_b200/.  The reference launches on the default stream, takes
fp16 device pointers in its NCHW layout, and fixes the UNet latent at 128x128 and the VAE
latent at [1, 4, 128, 128] (src/infer/unet.cu:1044-1074, src/kernels/vae_decode.cuh:19-47).
"""
from __future__ import annotations

import ctypes
import os
import tempfile
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "_ref_gpu" / "libref_sdxl_gpu.so"
_lib = None


def available() -> bool:
    return LIB_PATH.exists()


def lib():
    global _lib
    if _lib is None:
        L = ctypes.CDLL(str(LIB_PATH))
        L.ref_last_error.restype = ctypes.c_char_p
        L.ref_unet_open.argtypes = [ctypes.c_char_p, ctypes.POINTER(ctypes.c_void_p)]
        L.ref_unet_close.argtypes = [ctypes.c_void_p]
        L.ref_unet_close.restype = None
        fwd = [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_float, ctypes.c_void_p,
               ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int]
        L.ref_unet_forward.argtypes = fwd
        L.ref_unet_launch.argtypes = fwd
        L.ref_unet_capture_stages.argtypes = [ctypes.c_int]
        L.ref_unet_capture_stages.restype = None
        L.ref_unet_stage.argtypes = [ctypes.c_char_p, ctypes.c_void_p, ctypes.c_size_t]
        L.ref_unet_stage.restype = ctypes.c_size_t
        L.ref_vae_open.argtypes = [ctypes.c_char_p, ctypes.POINTER(ctypes.c_void_p)]
        L.ref_vae_close.argtypes = [ctypes.c_void_p]
        L.ref_vae_close.restype = None
        L.ref_vae_decode.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
        _lib = L
    return _lib


def _check(rc):
    if rc != 0:
        raise RuntimeError(f"reference GPU call failed ({rc}): {lib().ref_last_error().decode()}")


def write_safetensors(sd: dict, path: str) -> None:
    """fp16 host tensors keyed by diffusers names -> a .safetensors file the reference reads."""
    from safetensors.torch import save_file
    save_file({k: v.contiguous() for k, v in sd.items()}, path)


class RefUNet:
    """The reference's resident-weight UNet handle (unet_weights_create over a SafeTensors file).
    The reference keeps borrowing the file's bytes, so the handle owns its SafeTensors."""

    def __init__(self, sd_host: dict):
        fd, self._path = tempfile.mkstemp(suffix=".safetensors")
        os.close(fd)
        write_safetensors(sd_host, self._path)
        h = ctypes.c_void_p()
        _check(lib().ref_unet_open(self._path.encode(), ctypes.byref(h)))
        self._h = h

    def forward(self, latent, timestep, ehs, te, tid, out, attn_fast=False, epilogue=False, sync=True):
        f = lib().ref_unet_forward if sync else lib().ref_unet_launch
        _check(f(self._h, latent.shape[0], latent.data_ptr(), float(timestep), ehs.data_ptr(),
                 te.data_ptr(), tid.data_ptr(), out.data_ptr(), int(attn_fast), int(epilogue)))
        return out

    @staticmethod
    def capture_stages(on: bool) -> None:
        lib().ref_unet_capture_stages(1 if on else 0)

    @staticmethod
    def stage(name: str):
        import torch
        n = lib().ref_unet_stage(name.encode(), None, 0)
        if n == 0:
            return None
        t = torch.empty(n, dtype=torch.float16)
        lib().ref_unet_stage(name.encode(), ctypes.c_void_p(t.data_ptr()), n)
        return t

    def close(self):
        if getattr(self, "_h", None):
            lib().ref_unet_close(self._h)
            self._h = None
        if getattr(self, "_path", None):
            os.unlink(self._path)
            self._path = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class RefVAE:
    """The reference's resident-weight VAE decoder handle (vae_weights_create)."""

    def __init__(self, sd_host: dict):
        fd, self._path = tempfile.mkstemp(suffix=".safetensors")
        os.close(fd)
        write_safetensors(sd_host, self._path)
        h = ctypes.c_void_p()
        _check(lib().ref_vae_open(self._path.encode(), ctypes.byref(h)))
        self._h = h

    def decode(self, latent, image):
        _check(lib().ref_vae_decode(self._h, latent.data_ptr(), image.data_ptr()))
        return image

    def close(self):
        if getattr(self, "_h", None):
            lib().ref_vae_close(self._h)
            self._h = None
        if getattr(self, "_path", None):
            os.unlink(self._path)
            self._path = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
