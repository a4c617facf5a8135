"""ctypes access to the BitNet oracles — TEST INFRASTRUCTURE ONLY.

`oracle()` loads the plain-C restatements (bitnet_oracle.c, bitnet_lm.c); `reference()` loads the
reference's own code compiled from src/models/bitnet.hpp (oracle/_ref/libref_bitnet.so), or
returns None when it was not built (no reference tree here).  numpy in / numpy out.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
_O = None
_R = None

F32P = ctypes.POINTER(ctypes.c_float)


class LMConfigC(ctypes.Structure):
    _fields_ = [("vocab", ctypes.c_int), ("d_model", ctypes.c_int), ("n_layers", ctypes.c_int),
                ("n_heads", ctypes.c_int), ("ffn_dim", ctypes.c_int), ("max_seq", ctypes.c_int),
                ("rope_base", ctypes.c_double), ("rms_eps", ctypes.c_double),
                ("per_tensor_scale", ctypes.c_int)]
I8P = ctypes.POINTER(ctypes.c_int8)
I32P = ctypes.POINTER(ctypes.c_int32)


def _p(a, t):
    return a.ctypes.data_as(t)


def oracle():
    global _O
    if _O is None:
        path = HERE / "_build" / "liboracle_bitnet.so"
        if not path.exists():
            from oracle.build_oracle import build
            build()
        L = ctypes.CDLL(str(path))
        L.oracle_quantize_weight_ternary.restype = ctypes.c_float
        L.oracle_quantize_weight_ternary.argtypes = [F32P, ctypes.c_size_t, I8P]
        L.oracle_quantize_activation_int8.restype = ctypes.c_float
        L.oracle_quantize_activation_int8.argtypes = [F32P, ctypes.c_size_t, I8P]
        L.oracle_bitlinear.argtypes = [F32P, F32P, ctypes.c_int, ctypes.c_int, F32P, I8P, I8P]
        L.oracle_quantize_weight_rows.argtypes = [F32P, ctypes.c_int, ctypes.c_int, I8P, F32P]
        L.oracle_quantize_act_rows.argtypes = [F32P, ctypes.c_int, ctypes.c_int, I8P, F32P]
        L.oracle_ternary_gemm.argtypes = [I8P, F32P, I8P, F32P, ctypes.c_int, ctypes.c_int,
                                          ctypes.c_int, F32P, I32P]
        L.oracle_lm_create.restype = ctypes.c_void_p
        L.oracle_lm_create.argtypes = [ctypes.POINTER(LMConfigC), F32P, F32P, ctypes.c_void_p]
        L.oracle_lm_destroy.argtypes = [ctypes.c_void_p]
        L.oracle_lm_forward.argtypes = [ctypes.c_void_p, I32P, ctypes.c_int, F32P]
        L.oracle_lm_generate.argtypes = [ctypes.c_void_p, I32P, ctypes.c_int, ctypes.c_int,
                                         ctypes.c_int, I32P]
        _O = L
    return _O


def reference():
    global _R
    if _R is None:
        path = HERE / "_ref" / "libref_bitnet.so"
        if not path.exists():
            return None
        L = ctypes.CDLL(str(path))
        L.ref_quantize_weight_ternary.restype = ctypes.c_float
        L.ref_quantize_weight_ternary.argtypes = [F32P, ctypes.c_size_t, I8P]
        L.ref_quantize_activation_int8.restype = ctypes.c_float
        L.ref_quantize_activation_int8.argtypes = [F32P, ctypes.c_size_t, I8P]
        L.ref_bitlinear.argtypes = [F32P, F32P, ctypes.c_int, ctypes.c_int, F32P]
        L.ref_bitnet_dims.argtypes = [I32P]
        L.ref_bitnet_forward.argtypes = [F32P, F32P, ctypes.c_void_p, I32P, ctypes.c_int, F32P]
        L.ref_bitnet_forward.restype = ctypes.c_int
        _R = L
    return _R


def quant_weight(w, lib=None):
    lib = lib or oracle()
    w = np.ascontiguousarray(w, dtype=np.float32)
    q = np.zeros(w.size, dtype=np.int8)
    fn = lib.oracle_quantize_weight_ternary if hasattr(lib, "oracle_quantize_weight_ternary") \
        else lib.ref_quantize_weight_ternary
    s = fn(_p(w, F32P), w.size, _p(q, I8P))
    return float(s), q


def quant_act(x, lib=None):
    lib = lib or oracle()
    x = np.ascontiguousarray(x, dtype=np.float32)
    q = np.zeros(x.size, dtype=np.int8)
    fn = lib.oracle_quantize_activation_int8 if hasattr(lib, "oracle_quantize_activation_int8") \
        else lib.ref_quantize_activation_int8
    s = fn(_p(x, F32P), x.size, _p(q, I8P))
    return float(s), q


def bitlinear(w, x):
    """Oracle bitlinear: w [out, in] fp32, x [in] fp32 -> y [out] fp32."""
    L = oracle()
    w = np.ascontiguousarray(w, dtype=np.float32)
    x = np.ascontiguousarray(x, dtype=np.float32)
    out_dim, in_dim = w.shape
    y = np.zeros(out_dim, dtype=np.float32)
    s1 = np.zeros(in_dim, dtype=np.int8)
    s2 = np.zeros(in_dim, dtype=np.int8)
    L.oracle_bitlinear(_p(w, F32P), _p(x, F32P), out_dim, in_dim, _p(y, F32P), _p(s1, I8P), _p(s2, I8P))
    return y


def ref_bitlinear(w, x):
    R = reference()
    if R is None:
        return None
    w = np.ascontiguousarray(w, dtype=np.float32)
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.zeros(w.shape[0], dtype=np.float32)
    R.ref_bitlinear(_p(w, F32P), _p(x, F32P), w.shape[0], w.shape[1], _p(y, F32P))
    return y


def quant_weight_rows(w):
    L = oracle()
    w = np.ascontiguousarray(w, dtype=np.float32)
    N, K = w.shape
    q = np.zeros((N, K), dtype=np.int8)
    a = np.zeros(N, dtype=np.float32)
    L.oracle_quantize_weight_rows(_p(w, F32P), N, K, _p(q, I8P), _p(a, F32P))
    return q, a


def quant_act_rows(x):
    L = oracle()
    x = np.ascontiguousarray(x, dtype=np.float32)
    M, K = x.shape
    q = np.zeros((M, K), dtype=np.int8)
    s = np.zeros(M, dtype=np.float32)
    L.oracle_quantize_act_rows(_p(x, F32P), M, K, _p(q, I8P), _p(s, F32P))
    return q, s


def ternary_gemm(wq, alpha, xq, xscale):
    """y [M, N] and the raw int32 sums from quantized operands (bitlinear's arithmetic)."""
    L = oracle()
    wq = np.ascontiguousarray(wq, dtype=np.int8)
    xq = np.ascontiguousarray(xq, dtype=np.int8)
    alpha = np.ascontiguousarray(alpha, dtype=np.float32)
    xscale = np.ascontiguousarray(xscale, dtype=np.float32)
    N, K = wq.shape
    M = xq.shape[0]
    y = np.zeros((M, N), dtype=np.float32)
    acc = np.zeros((M, N), dtype=np.int32)
    L.oracle_ternary_gemm(_p(wq, I8P), _p(alpha, F32P), _p(xq, I8P), _p(xscale, F32P), M, N, K,
                          _p(y, F32P), _p(acc, I32P))
    return y, acc


# ------------------------------------------------------------------ LM forward / greedy decode

LAYER_KEYS = ("attn_norm", "wq", "wk", "wv", "wo", "ffn_norm", "w_gate", "w_up", "w_down")
TOK_EOS = 2   # src/io/tokenizer.hpp:44


def lm_config(vocab=16000, d_model=512, n_layers=8, n_heads=8, ffn_dim=1536, max_seq=128,
              rope_base=10000.0, rms_eps=1e-5, per_tensor_scale=0) -> dict:
    """Model dimensions (the benchmarked tag LM's by default; the reference's compiled-in ones are
    vocab 4999, FFN 1792, max_seq 64, src/models/bitnet_config.hpp:41-58)."""
    return dict(vocab=vocab, d_model=d_model, n_layers=n_layers, n_heads=n_heads, ffn_dim=ffn_dim,
                max_seq=max_seq, rope_base=rope_base, rms_eps=rms_eps,
                per_tensor_scale=per_tensor_scale)


def lm_shapes(cfg) -> dict:
    """name -> shape of the fp32 state dict (names of the reference loader,
    src/infer/bitnet.hpp:116-135: embed, final_norm, layers.N.*)."""
    D, F = cfg["d_model"], cfg["ffn_dim"]
    S = {"embed": (cfg["vocab"], D), "final_norm": (D,)}
    per = {"attn_norm": (D,), "wq": (D, D), "wk": (D, D), "wv": (D, D), "wo": (D, D),
           "ffn_norm": (D,), "w_gate": (F, D), "w_up": (F, D), "w_down": (D, F)}
    for l in range(cfg["n_layers"]):
        for k in LAYER_KEYS:
            S[f"layers.{l}.{k}"] = per[k]
    return S


def lm_random_weights(cfg, seed=10, kind="ternary") -> dict:
    """Seeded fp32 weights.  embed ~ N(0, 0.02) and norms ~ N(1, 0.01) as the reference's
    init_random (src/models/bitnet.hpp:300-331); BitLinear weights either uniform over {-1, 0, +1}
    (kind="ternary", the benchmarked tag LM) or N(0, 0.02) (kind="normal", the reference's init)."""
    rng = np.random.default_rng(seed)
    out = {}
    for name, shape in lm_shapes(cfg).items():
        key = name.rsplit(".", 1)[-1]
        if key in ("attn_norm", "ffn_norm", "final_norm"):
            t = 1.0 + 0.01 * rng.standard_normal(shape)
        elif key == "embed" or kind == "normal":
            t = 0.02 * rng.standard_normal(shape)
        else:
            t = rng.integers(-1, 2, size=shape)
        out[name] = np.ascontiguousarray(t, dtype=np.float32)
    return out


class OracleLM:
    """The C restatement of BitNet::forward / greedy decode over numpy weights."""

    def __init__(self, cfg, weights):
        self.cfg = dict(cfg)
        self._keep = {k: np.ascontiguousarray(v, dtype=np.float32) for k, v in weights.items()}
        L = oracle()
        c = LMConfigC(**self.cfg)
        ptrs = (ctypes.c_void_p * (9 * cfg["n_layers"]))()
        for l in range(cfg["n_layers"]):
            for j, k in enumerate(LAYER_KEYS):
                ptrs[9 * l + j] = self._keep[f"layers.{l}.{k}"].ctypes.data
        self._h = L.oracle_lm_create(ctypes.byref(c), _p(self._keep["embed"], F32P),
                                     _p(self._keep["final_norm"], F32P), ptrs)

    def forward(self, tokens):
        tokens = np.ascontiguousarray(tokens, dtype=np.int32)
        out = np.zeros((tokens.size, self.cfg["vocab"]), dtype=np.float32)
        rc = oracle().oracle_lm_forward(self._h, _p(tokens, I32P), tokens.size, _p(out, F32P))
        if rc != 0:
            raise ValueError("oracle_lm_forward: invalid input")
        return out

    def generate(self, prompt, max_len, eos=TOK_EOS):
        prompt = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.zeros(max_len, dtype=np.int32)
        n = oracle().oracle_lm_generate(self._h, _p(prompt, I32P), prompt.size, max_len, eos,
                                        _p(out, I32P))
        if n < 0:
            raise ValueError("oracle_lm_generate: invalid input")
        return out[:n].tolist()

    def close(self):
        if getattr(self, "_h", None):
            oracle().oracle_lm_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def ref_dims():
    """(vocab, d_model, n_layers, n_heads, ffn_dim, max_seq) of the compiled reference, or None."""
    R = reference()
    if R is None:
        return None
    d = np.zeros(6, dtype=np.int32)
    R.ref_bitnet_dims(_p(d, I32P))
    return tuple(int(x) for x in d)


def ref_forward(weights, tokens):
    """logits [S, vocab] of the reference's own BitNet::forward (None when not built)."""
    R = reference()
    if R is None:
        return None
    dims = ref_dims()
    keep = {k: np.ascontiguousarray(v, dtype=np.float32) for k, v in weights.items()}
    ptrs = (ctypes.c_void_p * (9 * dims[2]))()
    for l in range(dims[2]):
        for j, k in enumerate(LAYER_KEYS):
            ptrs[9 * l + j] = keep[f"layers.{l}.{k}"].ctypes.data
    tokens = np.ascontiguousarray(tokens, dtype=np.int32)
    out = np.zeros((tokens.size, dims[0]), dtype=np.float32)
    rc = R.ref_bitnet_forward(_p(keep["embed"], F32P), _p(keep["final_norm"], F32P), ptrs,
                              _p(tokens, I32P), tokens.size, _p(out, F32P))
    if rc != 0:
        raise ValueError("reference BitNet::forward threw")
    return out
