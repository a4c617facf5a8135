"""Python host mirror of the reference's LM inference API over the C ABI.

Mirrors BitNetGpuInfer / BitNetDenseInfer's forward / generate (reference
src/infer/bitnet_gpu.cuh:103-160, src/infer/bitnet.hpp:282-318) for the ternary BitNet of
src/models/bitnet.hpp, batched over sequences: `forward(tokens [B, S])` -> logits [B, S, vocab],
`generate(prompts [B, P], max_len)` -> the generated ids of every sequence.  All compute runs in
`libdollama_b200.so`; this module only marshals arrays.
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import _lib as L


class BitNetConfig(ctypes.Structure):
    """dlm_bitnet_config (by default the benchmarked tag LM: vocab 16000, d 512, 8 layers, FFN 1536;
    head_dim = d_model / n_heads = 64)."""
    _fields_ = [("vocab", ctypes.c_int), ("d_model", ctypes.c_int), ("n_layers", ctypes.c_int),
                ("n_heads", ctypes.c_int), ("ffn_dim", ctypes.c_int), ("max_seq", ctypes.c_int),
                ("rope_base", ctypes.c_double), ("rms_eps", ctypes.c_double),
                ("per_tensor_scale", ctypes.c_int)]

    def __init__(self, vocab=16000, d_model=512, n_layers=8, n_heads=8, ffn_dim=1536, max_seq=128,
                 rope_base=10000.0, rms_eps=1e-5, per_tensor_scale=0):
        super().__init__(vocab, d_model, n_layers, n_heads, ffn_dim, max_seq, rope_base, rms_eps,
                         per_tensor_scale)

    def as_dict(self):
        return {f: getattr(self, f) for f, _ in self._fields_}


def _stream_ptr(stream=None):
    if not torch.cuda.is_available():
        return ctypes.c_void_p()
    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


def _ptr(x):
    return ctypes.c_void_p(x.data_ptr() if isinstance(x, torch.Tensor) else x.ctypes.data)


class BitNetLM:
    """The ternary BitNet tag LM on the GPU.  `weights` maps the reference loader's names to fp32
    arrays (numpy or torch, host or CUDA)."""

    def __init__(self, cfg: BitNetConfig, weights: dict, stream=None):
        self.cfg = cfg
        names = list(weights.keys())
        tens = [weights[n] for n in names]
        keep = []
        for n, t in zip(names, tens):
            if isinstance(t, np.ndarray):
                t = np.ascontiguousarray(t, dtype=np.float32)
            elif not (t.dtype == torch.float32 and t.is_contiguous()):
                raise ValueError(f"{n}: expected a contiguous fp32 tensor")
            keep.append(t)
        n = len(names)
        c_names = (ctypes.c_char_p * n)(*[x.encode() for x in names])
        c_ptrs = (ctypes.c_void_p * n)(*[_ptr(t).value for t in keep])
        c_numel = (ctypes.c_int64 * n)(*[int(t.size if isinstance(t, np.ndarray) else t.numel())
                                         for t in keep])
        h = ctypes.c_void_p()
        L.call("dlm_bitnet_create", ctypes.byref(cfg), n, c_names, c_ptrs, c_numel, ctypes.byref(h),
               _stream_ptr(stream))
        self._h = h

    def forward(self, tokens, stream=None) -> np.ndarray:
        """tokens [B, S] int -> logits [B, S, vocab] float32 (numpy)."""
        tokens = np.ascontiguousarray(np.atleast_2d(tokens), dtype=np.int32)
        B, S = tokens.shape
        out = np.zeros((B, S, self.cfg.vocab), dtype=np.float32)
        L.call("dlm_bitnet_forward", self._h, _ptr(tokens), B, S, _ptr(out), _stream_ptr(stream))
        return out

    def generate(self, prompts, max_len: int, stream=None):
        """prompts [B, P] int -> list of B lists of generated ids (greedy, <eos> excluded)."""
        prompts = np.ascontiguousarray(np.atleast_2d(prompts), dtype=np.int32)
        B, P = prompts.shape
        G = max(max_len - P, 0)
        out = np.zeros((B, max(G, 1)), dtype=np.int32)
        lens = np.zeros(B, dtype=np.int32)
        L.call("dlm_bitnet_generate", self._h, _ptr(prompts), B, P, int(max_len), _ptr(out),
               _ptr(lens), _stream_ptr(stream))
        return [out[b, :lens[b]].tolist() for b in range(B)]

    def generate_from_text(self, tok, text: str, max_len: int = None, stream=None):
        """Tags for a natural-language prompt: [<bos>] + the text's greedy tag matches + [<sep>],
        greedy decode, decoded tag strings (the reference's generate_from_text,
        src/infer/bitnet.hpp:321-336, with the tokenizer of dollama_b200.tokenizer)."""
        from .tokenizer import text_prompt
        ids = self.generate(np.asarray([text_prompt(tok, text)], dtype=np.int32),
                            max_len or self.cfg.max_seq, stream)[0]
        return tok.decode(ids)

    def generate_with_identity(self, tok, identity_tags, scene_text: str, max_len: int = None,
                               stream=None):
        """<bos> identity <sep> scene tags <sep> prompt, greedy decode, decoded tags
        (generate_with_identity, src/infer/bitnet.hpp:379-385)."""
        from .tokenizer import identity_prompt
        ids = self.generate(np.asarray([identity_prompt(tok, identity_tags, scene_text)], dtype=np.int32),
                            max_len or self.cfg.max_seq, stream)[0]
        return tok.decode(ids)

    def generate_device(self, prompts: torch.Tensor, max_len: int, out: torch.Tensor,
                        lens: torch.Tensor, stream=None):
        """The same decode on CUDA int32 tensors (no host copies)."""
        B, P = prompts.shape
        L.call("dlm_bitnet_generate", self._h, _ptr(prompts), B, P, int(max_len), _ptr(out),
               _ptr(lens), _stream_ptr(stream))
        return out, lens

    def close(self):
        if getattr(self, "_h", None):
            L.lib().dlm_bitnet_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def weight_spec(cfg: BitNetConfig) -> dict:
    """name -> shape of every tensor dlm_bitnet_create expects (from the C library)."""
    lib = L.lib()
    n = lib.dlm_bitnet_weight_count(ctypes.byref(cfg))
    out = {}
    buf = ctypes.create_string_buffer(256)
    shape = (ctypes.c_int64 * 4)()
    nd = ctypes.c_int()
    for i in range(n):
        L.call("dlm_bitnet_weight_info", ctypes.byref(cfg), i, buf, 256, shape, ctypes.byref(nd))
        out[buf.value.decode()] = tuple(shape[j] for j in range(nd.value))
    return out


def random_weights(cfg: BitNetConfig, seed: int = 10, device="cuda") -> dict:
    """Synthetic weights of the benchmarked tag LM on `device`: BitLinear weights uniform over
    {-1, 0, +1}, embed ~ N(0, 0.02), norms ~ N(1, 0.01) (fp32)."""
    g = torch.Generator(device=device).manual_seed(seed)
    out = {}
    for name, shape in weight_spec(cfg).items():
        key = name.rsplit(".", 1)[-1]
        if key in ("attn_norm", "ffn_norm", "final_norm"):
            t = 1.0 + 0.01 * torch.randn(shape, generator=g, device=device)
        elif key == "embed":
            t = 0.02 * torch.randn(shape, generator=g, device=device)
        else:
            t = torch.randint(-1, 2, shape, generator=g, device=device).float()
        out[name] = t.contiguous()
    return out
