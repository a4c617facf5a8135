"""Runtime LoRA host logic: kohya-named LoRA tensors -> modules for `dlm_unet_apply_loras`.

Restates the reference's `load_lora_modules` (src/infer/lora.hpp:300-455; its DTO `LoraModule`,
lora.hpp:136-145, and report `LoraLoadReport`, lora.hpp:148-154):

  * keys `lora_unet_<flat>.lora_down.weight` (A [rank, in(, kh, kw)]), `.lora_up.weight`
    (B [out, rank(, 1, 1)]) and `.alpha` (scalar; rank when absent) are grouped per module; the
    fully flattened spellings `_lora_down_weight` / `_lora_up_weight` / `_alpha` are accepted
    too (lora.hpp:308-345);
  * text-encoder keys (`lora_te_`, `lora_te1_`, `lora_te2_`) are skipped and counted; other
    keys are counted; modules missing A or B are skipped and counted;
  * a module resolves to the base key whose dots-to-underscores spelling equals
    `<flat>_weight` (lora.hpp:160-176, 360-368); an unresolved module raises;
  * A / B shapes: rank = A.shape[0], in_flat = prod(A.shape[1:]), out = B.shape[0],
    prod(B.shape[1:]) must equal rank; a 2-D base must be exactly [out, in_flat], a conv base
    must have out * in_flat elements (lora.hpp:375-425);
  * scale = strength * alpha / rank (lora.hpp:427-429); fp32 tensors are rounded to fp16 with
    round-to-nearest-even (numpy's astype, as lora.hpp:53-112 does by hand).

The merge itself (W += h(scale * B @ A) on the device-resident weights) is
`SDXLUNet.apply_loras`, which calls the C ABI.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field

import numpy as np

_TE_PREFIXES = ("lora_te1_", "lora_te2_", "lora_te_")
_SUFFIXES = ((".lora_down.weight", "down"), (".lora_up.weight", "up"), (".alpha", "alpha"),
             ("_lora_down_weight", "down"), ("_lora_up_weight", "up"), ("_alpha", "alpha"))


@dataclass
class LoraModule:
    """One resolved LoRA module (the reference's LoraModule): fp16 A [rank, in_flat] and
    B [out_dim, rank] as host arrays, and the merge scale."""
    base_key: str
    a_fp16: np.ndarray
    b_fp16: np.ndarray
    rank: int
    in_flat: int
    out_dim: int
    scale: float = 1.0


@dataclass
class LoraLoadReport:
    te_skipped: int = 0
    other_keys: int = 0
    incomplete: int = 0
    modules: int = 0


def _to_numpy(t) -> np.ndarray:
    if hasattr(t, "detach"):  # torch tensor
        t = t.detach().cpu()
        if str(t.dtype) == "torch.bfloat16":
            t = t.float()
        t = t.numpy()
    return np.asarray(t)


def _as_f16(t, key: str) -> np.ndarray:
    a = _to_numpy(t)
    if a.dtype == np.float16:
        return np.ascontiguousarray(a)
    if a.dtype == np.float32:
        return np.ascontiguousarray(a.astype(np.float16))  # round to nearest even
    raise ValueError(f"lora: tensor '{key}' must be F16/F32 (dtype={a.dtype})")


def _alpha(t, key: str) -> float:
    a = _to_numpy(t)
    if a.dtype not in (np.float16, np.float32) or a.size < 1:
        raise ValueError(f"lora: alpha '{key}' must be F32/F16 scalar (dtype={a.dtype})")
    return float(a.reshape(-1)[0])


def load_lora_modules(base_shapes: dict, lora: dict, strength: float = 1.0):
    """Resolve a kohya LoRA (`lora`: name -> tensor / array) against the base UNet's weights
    (`base_shapes`: diffusers name -> shape, e.g. `dollama_b200.unet.weight_spec()`).
    Returns (modules sorted by module name, LoraLoadReport)."""
    rep = LoraLoadReport()
    groups: dict = {}
    for k in sorted(lora):
        if k.startswith(_TE_PREFIXES):
            rep.te_skipped += 1
            continue
        if not k.startswith("lora_unet_"):
            rep.other_keys += 1
            continue
        body = k[len("lora_unet_"):]
        for suf, kind in _SUFFIXES:
            if body.endswith(suf):
                g = groups.setdefault(body[: -len(suf)], {})
                if kind == "alpha":
                    g["alpha"] = _alpha(lora[k], k)
                else:
                    g[kind] = k
                break
        else:
            rep.other_keys += 1
    index = {name.replace(".", "_"): name for name in base_shapes}
    mods = []
    for mod in sorted(groups):
        g = groups[mod]
        if "down" not in g or "up" not in g:
            rep.incomplete += 1
            continue
        base_key = index.get(mod + "_weight")
        if base_key is None:
            raise KeyError(f"lora: module 'lora_unet_{mod}' does not resolve to any base key "
                           "(naming mismatch)")
        a = _as_f16(lora[g["down"]], g["down"])
        b = _as_f16(lora[g["up"]], g["up"])
        if a.ndim == 0 or b.ndim == 0:
            raise ValueError(f"lora: module 'lora_unet_{mod}' has empty A/B shape")
        rank, out_dim = a.shape[0], b.shape[0]
        in_flat = int(np.prod(a.shape[1:], dtype=np.int64))
        b_trail = int(np.prod(b.shape[1:], dtype=np.int64))
        if b_trail != rank:
            raise ValueError(f"lora: module 'lora_unet_{mod}' B trailing dims ({b_trail}) != "
                             f"rank ({rank})")
        if rank == 0 or in_flat == 0 or out_dim == 0:
            raise ValueError(f"lora: module 'lora_unet_{mod}' has zero dim")
        wshape = tuple(base_shapes[base_key])
        if len(wshape) == 2:
            if wshape != (out_dim, in_flat):
                raise ValueError(f"lora: module 'lora_unet_{mod}' -> '{base_key}' shape mismatch "
                                 f"(Linear): base {list(wshape)} vs B@A [{out_dim},{in_flat}]")
        elif int(np.prod(wshape, dtype=np.int64)) != out_dim * in_flat:
            raise ValueError(f"lora: module 'lora_unet_{mod}' -> '{base_key}' numel mismatch "
                             f"(Conv): base {int(np.prod(wshape))} vs B@A {out_dim * in_flat}")
        alpha = g.get("alpha", float(rank))
        scale = float(np.float32(strength) * (np.float32(alpha) / np.float32(rank)))
        mods.append(LoraModule(base_key, a.reshape(rank, in_flat), b.reshape(out_dim, rank),
                               int(rank), in_flat, int(out_dim), scale))
        rep.modules += 1
    return mods, rep


class DlmLoraModule(ctypes.Structure):
    """ctypes mirror of `dlm_lora_module` (include/dollama_b200.h)."""
    _fields_ = [("base_key", ctypes.c_char_p), ("a_fp16", ctypes.c_void_p),
                ("b_fp16", ctypes.c_void_p), ("rank", ctypes.c_int), ("in_flat", ctypes.c_int),
                ("out_dim", ctypes.c_int), ("scale", ctypes.c_float)]


def pack_modules(mods):
    """ctypes array of `dlm_lora_module` over the modules' host buffers; returns (array, keepalive)."""
    arr = (DlmLoraModule * max(1, len(mods)))()
    keep = []
    for i, m in enumerate(mods):
        a = np.ascontiguousarray(m.a_fp16, dtype=np.float16)
        b = np.ascontiguousarray(m.b_fp16, dtype=np.float16)
        if a.size != m.rank * m.in_flat or b.size != m.out_dim * m.rank:
            raise ValueError(f"lora: '{m.base_key}' A/B buffer size mismatch vs shape")
        key = m.base_key.encode()
        keep += [a, b, key]
        arr[i] = DlmLoraModule(key, a.ctypes.data, b.ctypes.data, m.rank, m.in_flat, m.out_dim,
                               m.scale)
    return arr, keep
