"""ctypes binding of ``libdollama_b200.so`` (the C ABI declared in ``include/dollama_b200.h``).

The library is the product: there is no CPU or PyTorch fallback.  ``lib()`` raises if the
shared library is missing or fails to load, so a caller never silently runs other code.
"""
from __future__ import annotations

import ctypes
import os
import re
from pathlib import Path

_PKG = Path(__file__).resolve().parent
LIB_PATH = _PKG / "libdollama_b200.so"
HEADER = _PKG.parent / "include" / "dollama_b200.h"

_lib = None

c_int = ctypes.c_int
c_uint = ctypes.c_uint
c_float = ctypes.c_float
c_void_p = ctypes.c_void_p
c_char_p = ctypes.c_char_p
c_size_t = ctypes.c_size_t

# name -> (restype, [argtypes]); every entry point the header declares.
_SIGS = {
    "dlm_last_error": (c_char_p, []),
    "dlm_version": (c_char_p, []),
    "dlm_get_device_status": (c_int, [ctypes.POINTER(c_int), c_int, c_void_p]),
    "dlm_memcpy": (c_int, [c_void_p, c_void_p, c_size_t, c_void_p]),
    "dlm_launch_gemm_fp16": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_float,
                                     c_float, c_int, c_int, c_void_p]),
    "dlm_gemm_fp16_ex": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_int, c_int, c_int, c_int,
                                 c_uint, c_void_p, c_void_p, c_int, c_void_p, c_int, c_void_p]),
    "dlm_gemm_set_tile_mode": (c_int, [c_int]),
    "dlm_gemm_fp16_batched": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int,
                                      ctypes.c_longlong, ctypes.c_longlong, ctypes.c_longlong,
                                      c_float, c_float, c_int, c_void_p]),
    "dlm_gemm_f32": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_float, c_float,
                             c_int, c_int, c_void_p]),
    "dlm_bias_add_rowvec": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_void_p]),
    "dlm_bias_add_channel": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int,
                                     c_void_p]),
    "dlm_conv_bias_biasch": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int,
                                     c_int, c_void_p]),
    "dlm_conv_bias_residual": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int,
                                       c_int, c_void_p]),
    "dlm_silu": (c_int, [c_void_p, c_void_p, c_int, c_void_p]),
    "dlm_gelu": (c_int, [c_void_p, c_void_p, c_int, c_void_p]),
    "dlm_gelu_tanh": (c_int, [c_void_p, c_void_p, c_int, c_void_p]),
    "dlm_add": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_void_p]),
    "dlm_upsample_nearest2x": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p]),
    "dlm_geglu": (c_int, [c_void_p, c_void_p, c_int, c_int, c_void_p]),
    "dlm_timestep_embedding": (c_int, [c_void_p, c_float, c_int, c_float, c_void_p]),
    "dlm_gemm_workspace_bytes": (ctypes.c_size_t, []),
    "dlm_gemm_fp16_ws": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_int, c_int, c_int, c_int,
                                 ctypes.c_uint, c_void_p, c_void_p, c_int, c_void_p, ctypes.c_size_t,
                                 c_void_p]),
    "dlm_conv2d_nhwc_scratch_bytes": (c_size_t, [c_int, c_int, c_int, c_int, c_int, c_int]),
    "dlm_conv2d_nhwc": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_void_p,
                                c_void_p, c_int, c_int, c_int, c_void_p, c_size_t, c_void_p]),
    "dlm_pack_conv_weight": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p]),
    "dlm_nchw_to_nhwc": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_void_p]),
    "dlm_nhwc_to_nchw": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_void_p]),
    "dlm_launch_attention": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int,
                                     c_int, c_int, c_float, c_void_p]),
    "dlm_attention_workspace_bytes": (ctypes.c_size_t, [c_int, c_int, c_int]),
    "dlm_launch_attention_ws": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int,
                                        c_int, c_int, c_float, c_void_p, ctypes.c_size_t,
                                        c_void_p]),
    "dlm_attention_tokens": (c_int, [c_void_p, c_int, c_void_p, c_int, c_void_p, c_int, c_void_p,
                                     c_int, c_int, c_int, c_int, c_int, c_int, c_float, c_void_p]),
    "dlm_group_norm_nhwc_scratch_bytes": (c_size_t, [c_int, c_int]),
    "dlm_group_norm_nhwc": (c_int, [c_void_p, c_int, c_void_p, c_int, c_int, c_int, c_void_p,
                                    c_void_p, c_float, c_int, c_int, c_void_p, c_void_p, c_size_t,
                                    c_void_p]),
    "dlm_group_norm_nchw_scratch_bytes": (c_size_t, [c_int, c_int]),
    "dlm_group_norm_nchw": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int,
                                    c_int, c_int, c_float, c_int, c_void_p, c_size_t, c_void_p]),
    "dlm_conv2d_direct_nchw": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_int,
                                       c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_int,
                                       c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_void_p]),
    "dlm_conv2d_uses_gemm_bias_path": (c_int, [c_int] * 13),
    "dlm_group_norm_nhwc_noalloc_capacity": (c_size_t, []),
    "dlm_group_norm_nhwc_noalloc": (c_int, [c_void_p, c_int, c_void_p, c_int, c_int, c_int,
                                            c_void_p, c_void_p, c_float, c_int, c_int, c_void_p,
                                            c_void_p]),
    "dlm_launch_layer_norm": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_float,
                                      c_void_p]),
    "dlm_ternary_pack": (c_int, [c_void_p, c_int, c_int, c_void_p, c_void_p, c_void_p]),
    "dlm_quantize_act_i8": (c_int, [c_void_p, c_int, c_int, c_void_p, c_void_p, c_void_p]),
    "dlm_ternary_gemm_i8": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int,
                                    c_int, c_void_p]),
    "dlm_bitlinear": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p,
                              c_void_p, c_void_p]),
    "dlm_unet_create": (c_int, [ctypes.POINTER(c_int), c_int, c_int, ctypes.POINTER(c_char_p),
                                ctypes.POINTER(c_void_p), ctypes.POINTER(ctypes.c_int64),
                                ctypes.POINTER(c_void_p), c_void_p]),
    "dlm_unet_destroy": (c_int, [c_void_p]),
    "dlm_unet_forward": (c_int, [c_void_p, c_int, c_int, c_int, c_void_p, c_float, c_void_p,
                                 c_void_p, c_void_p, c_void_p, c_void_p]),
    "dlm_unet_set_graph": (c_int, [c_void_p, c_int]),
    "dlm_unet_apply_loras": (c_int, [c_void_p, c_void_p, c_int, c_void_p]),
    "dlm_unet_apply_lora": (c_int, [c_void_p, c_char_p, c_void_p, c_void_p, c_int, c_int, c_int,
                                    c_float, c_void_p]),
    "dlm_unet_clear_loras": (c_int, [c_void_p, c_void_p]),
    "dlm_unet_weight_count": (c_int, [ctypes.POINTER(c_int), c_int]),
    "dlm_unet_weight_info": (c_int, [ctypes.POINTER(c_int), c_int, c_int, ctypes.c_char_p, c_int,
                                     ctypes.POINTER(ctypes.c_int64), ctypes.POINTER(c_int)]),
    "dlm_unet_forward_host": (c_int, [c_void_p, c_int, c_int, c_int, c_void_p, c_float, c_void_p,
                                      c_void_p, c_void_p, c_void_p, c_void_p]),
    "dlm_unet_time_ops": (c_int, [c_void_p, ctypes.POINTER(ctypes.c_double),
                                  ctypes.POINTER(ctypes.c_double), ctypes.POINTER(c_int), c_void_p]),
    "dlm_unet_stage": (c_int, [c_void_p, c_char_p, ctypes.POINTER(c_void_p), ctypes.POINTER(c_int),
                               ctypes.POINTER(c_int), ctypes.POINTER(c_int)]),
    "dlm_unet_info": (c_int, [c_void_p, ctypes.POINTER(ctypes.c_int64),
                              ctypes.POINTER(ctypes.c_int64), ctypes.POINTER(c_int)]),
    "dlm_bitnet_create": (c_int, [c_void_p, c_int, ctypes.POINTER(c_char_p), ctypes.POINTER(c_void_p),
                                  ctypes.POINTER(ctypes.c_int64), ctypes.POINTER(c_void_p),
                                  c_void_p]),
    "dlm_bitnet_destroy": (c_int, [c_void_p]),
    "dlm_bitnet_forward": (c_int, [c_void_p, c_void_p, c_int, c_int, c_void_p, c_void_p]),
    "dlm_bitnet_generate": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_void_p, c_void_p,
                                    c_void_p]),
    "dlm_bitnet_weight_count": (c_int, [c_void_p]),
    "dlm_bitnet_weight_info": (c_int, [c_void_p, c_int, ctypes.c_char_p, c_int,
                                       ctypes.POINTER(ctypes.c_int64), ctypes.POINTER(c_int)]),
    "dlm_sdxl_schedule": (c_int, [c_int, ctypes.POINTER(ctypes.c_float),
                                  ctypes.POINTER(ctypes.c_float)]),
    "dlm_sdxl_denoise": (c_int, [c_void_p, c_int, c_int, c_void_p, c_int, c_float, c_void_p,
                                 c_void_p, c_void_p, c_void_p, c_void_p]),
    "dlm_sdxl_generate": (c_int, [c_void_p, c_void_p, c_int, c_int, c_void_p, c_int, c_float,
                                  c_void_p, c_void_p, c_void_p, c_float, c_void_p, c_void_p]),
    "dlm_vae_create": (c_int, [c_int, ctypes.POINTER(c_char_p), ctypes.POINTER(c_void_p),
                               ctypes.POINTER(ctypes.c_int64), ctypes.POINTER(c_void_p), c_void_p]),
    "dlm_vae_destroy": (c_int, [c_void_p]),
    "dlm_vae_decode": (c_int, [c_void_p, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p]),
    "dlm_vae_decode_host": (c_int, [c_void_p, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p]),
    "dlm_vae_set_graph": (c_int, [c_void_p, c_int]),
    "dlm_vae_stage": (c_int, [c_void_p, c_char_p, ctypes.POINTER(c_void_p), ctypes.POINTER(c_int),
                              ctypes.POINTER(c_int), ctypes.POINTER(c_int), ctypes.POINTER(c_int)]),
    "dlm_vae_info": (c_int, [c_void_p, ctypes.POINTER(ctypes.c_int64),
                             ctypes.POINTER(ctypes.c_int64), ctypes.POINTER(c_int)]),
    "dlm_vae_time_ops": (c_int, [c_void_p, ctypes.POINTER(ctypes.c_double),
                                 ctypes.POINTER(ctypes.c_double), ctypes.POINTER(c_int), c_void_p]),
    "dlm_vae_weight_count": (c_int, []),
    "dlm_vae_weight_info": (c_int, [c_int, ctypes.c_char_p, c_int, ctypes.POINTER(ctypes.c_int64),
                                    ctypes.POINTER(c_int)]),
}

EPI_BIAS = 1
EPI_RESID = 2
EPI_GEGLU = 4
EPI_SILU = 8
EPI_BIAS2D = 16


class DlmError(RuntimeError):
    def __init__(self, fn: str, code: int, msg: str):
        super().__init__(f"{fn} failed with status {code}: {msg}")
        self.code = code


def header_symbols() -> list[str]:
    """Names of every function the C header declares."""
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\**\s+\**(dlm_\w+)\s*\(", text, re.M)))


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise RuntimeError(
            f"{LIB_PATH} is missing: build it with `python -m dollama_b200.build` "
            "(there is no fallback path)")
    mode = getattr(os, "RTLD_GLOBAL", 0)
    L = ctypes.CDLL(str(LIB_PATH), mode=mode)
    for name, (res, args) in _SIGS.items():
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args
    _lib = L
    return L


def last_error() -> str:
    return (lib().dlm_last_error() or b"").decode(errors="replace")


def check(fn: str, rc: int) -> None:
    if rc != 0:
        raise DlmError(fn, rc, last_error())


def call(fn: str, *args) -> None:
    check(fn, getattr(lib(), fn)(*args))
