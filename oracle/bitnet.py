"""ctypes access to the BitNet oracles — TEST INFRASTRUCTURE ONLY.

`oracle()` loads the plain-C restatement (bitnet_oracle.c); `reference()` loads the reference's
own integer path compiled from src/models/bitnet.hpp (oracle/_ref/libref_bitnet.so), or returns
None when it was not built (no reference tree here).  numpy in / numpy out.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
_O = None
_R = None

F32P = ctypes.POINTER(ctypes.c_float)
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
