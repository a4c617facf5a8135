"""The UNet / VAE oracle's operations (oracle/sdxl_unet.py) against the CPU reference
implementations inside the reference's own kernel tests (src/tests/test_groupnorm.cu,
test_layernorm.cu, test_geglu.cu, test_activation.cu, test_attention.cu, test_timeembed.cu,
test_conv2d.cu,
compiled where they lie into oracle/_ref/libref_cpu_*.so by oracle/build_oracle.py).

Those CPU references define what each reference kernel computes (eps placement, biased variance,
affine order, erf / tanh GELU, softmax scale, [cos | sin] order); the oracle computes the same in
fp32 with other summation orders, so the bar is fp32 rounding: max|oracle - ref| <= 2e-5 of the
output scale (1e-4 for the GroupNorm reference's one-pass fp32 variance).  This pins the whole-
model oracle's building blocks to the reference; the whole-model goldens stay unavailable.
"""
import ctypes
import math
import os

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import sdxl_unet as U
from oracle import sdxl_vae as V
from oracle.build_oracle import build

FP = ctypes.POINTER(ctypes.c_float)


@pytest.fixture(scope="module")
def libs():
    out = build()
    need = ["gn", "ln", "geglu", "act", "attn", "timeembed", "conv"]
    if any(f"ref_cpu_{k}" not in out for k in need):
        pytest.skip("reference tree absent: the kernel tests' CPU references are not built")
    # lazy binding: the convolution test's GPU entry points are never called nor linked
    return {k: ctypes.CDLL(out[f"ref_cpu_{k}"], mode=os.RTLD_LAZY | os.RTLD_LOCAL) for k in need}


def _p(a):
    return a.ctypes.data_as(FP)


def _rel(got, ref):
    return float(np.max(np.abs(got - ref)) / max(np.max(np.abs(ref)), 1e-30))


def _rng(seed):
    return np.random.default_rng(seed)


# amplitude 0.003 puts the variance next to eps, so the eps placement shows
@pytest.mark.parametrize("N,C,H,W,eps,amp", [(2, 64, 8, 8, 1e-5, 2.0), (1, 320, 16, 16, 1e-6, 2.0),
                                             (2, 96, 5, 7, 1e-5, 2.0), (2, 64, 8, 8, 1e-5, 0.003),
                                             (1, 64, 8, 8, 1e-6, 0.001)])
def test_group_norm(libs, N, C, H, W, eps, amp):
    r = _rng(C + H)
    x = (r.standard_normal((N, C, H, W)) * amp + 0.25 * amp).astype(np.float32)
    g = (1 + 0.1 * r.standard_normal(C)).astype(np.float32)
    b = (0.1 * r.standard_normal(C)).astype(np.float32)
    out = np.zeros_like(x)
    libs["gn"].ref_cpu_group_norm(_p(x), _p(g), _p(b), N, C, H, W, 32, ctypes.c_float(eps), _p(out))
    sd = {"n.weight": torch.from_numpy(g), "n.bias": torch.from_numpy(b)}
    got = U.group_norm(torch.from_numpy(x), sd, "n", 32, eps).numpy()
    assert _rel(got, out) <= 1e-4


@pytest.mark.parametrize("rows,C,amp", [(37, 320, 3.0), (8, 1280, 3.0), (16, 640, 0.003)])
def test_layer_norm(libs, rows, C, amp):
    r = _rng(rows)
    x = (r.standard_normal((rows, C)) * amp - amp / 3).astype(np.float32)
    g = (1 + 0.1 * r.standard_normal(C)).astype(np.float32)
    b = (0.1 * r.standard_normal(C)).astype(np.float32)
    out = np.zeros_like(x)
    libs["ln"].ref_cpu_layer_norm(_p(x), _p(g), _p(b), rows, C, ctypes.c_float(1e-5), _p(out))
    sd = {"n.weight": torch.from_numpy(g), "n.bias": torch.from_numpy(b)}
    got = U.layer_norm(torch.from_numpy(x), sd, "n").numpy()
    assert _rel(got, out) <= 2e-5


def test_geglu(libs):
    r = _rng(3)
    tokens, d = 33, 160
    x = (r.standard_normal((tokens, 2 * d)) * 2).astype(np.float32)
    out = np.zeros((tokens, d), np.float32)
    libs["geglu"].ref_cpu_geglu(_p(x), tokens, d, _p(out))
    hid, gate = torch.from_numpy(x).chunk(2, dim=-1)          # the oracle's GEGLU (transformer_block)
    got = (hid * F.gelu(gate)).numpy()
    assert _rel(got, out) <= 2e-5


@pytest.mark.parametrize("act", [0, 1, 2])
def test_activations(libs, act):
    x = np.linspace(-12, 12, 4097, dtype=np.float32)
    out = np.zeros_like(x)
    libs["act"].ref_cpu_activation(_p(x), ctypes.c_size_t(x.size), act, _p(out))
    t = torch.from_numpy(x)
    got = (F.silu(t) if act == 0 else F.gelu(t) if act == 1 else F.gelu(t, approximate="tanh")).numpy()
    assert _rel(got, out) <= 2e-5


@pytest.mark.parametrize("B,H,Sq,Sk", [(2, 2, 64, 77), (1, 3, 50, 130)])
def test_attention(libs, B, H, Sq, Sk):
    r = _rng(Sq + Sk)
    q = r.standard_normal((B, H, Sq, 64)).astype(np.float32)
    k = r.standard_normal((B, H, Sk, 64)).astype(np.float32)
    v = r.standard_normal((B, H, Sk, 64)).astype(np.float32)
    out = np.zeros_like(q)
    libs["attn"].ref_cpu_attention(_p(q), _p(k), _p(v), B, H, Sq, Sk, 64, ctypes.c_float(0.125), _p(out))
    tok = lambda a: torch.from_numpy(a).transpose(1, 2).reshape(B, a.shape[2], H * 64)
    got = U.attention(tok(q), tok(k), tok(v), H).view(B, Sq, H, 64).transpose(1, 2).numpy()
    assert _rel(got, out) <= 2e-5


@pytest.mark.parametrize("t", [0.0, 1.0, 261.0, 999.0])
def test_timestep_embedding(libs, t):
    dim = 320
    out = np.zeros(dim, np.float32)
    libs["timeembed"].ref_cpu_time_embedding(ctypes.c_float(t), dim, ctypes.c_float(10000.0), _p(out))
    got = U.timestep_embedding(torch.tensor([t]), dim)[0].numpy()
    # both evaluate cos / sin of a float argument; the argument t * f_i may differ by an ulp of a
    # value up to ~1e3, so the bound is on that argument's rounding
    assert float(np.max(np.abs(got - out))) <= 2.0 * max(t, 1.0) * 2.0 ** -23


@pytest.mark.parametrize("Cin,Cout,H,W,K,stride,pad", [(8, 16, 9, 7, 3, 1, 1), (8, 8, 10, 10, 3, 2, 1),
                                                       (12, 6, 5, 6, 1, 1, 0), (4, 32, 8, 8, 3, 1, 1)])
def test_conv2d(libs, Cin, Cout, H, W, K, stride, pad):
    r = _rng(Cin * Cout + H)
    N = 2
    x = r.standard_normal((N, Cin, H, W)).astype(np.float32)
    w = (r.standard_normal((Cout, Cin, K, K)) / math.sqrt(Cin * K * K)).astype(np.float32)
    b = (0.1 * r.standard_normal(Cout)).astype(np.float32)
    Ho = (H + 2 * pad - K) // stride + 1
    Wo = (W + 2 * pad - K) // stride + 1
    out = np.zeros((N, Cout, Ho, Wo), np.float32)
    libs["conv"].ref_cpu_conv2d(_p(x), _p(w), _p(b), N, Cin, H, W, Cout, K, K, stride, pad, _p(out))
    sd = {"c.weight": torch.from_numpy(w), "c.bias": torch.from_numpy(b)}
    got = U.conv(torch.from_numpy(x), sd, "c", stride=stride, padding=pad).numpy()
    assert _rel(got, out) <= 2e-5


def test_vae_mid_attention(libs):
    """The VAE decoder's single-head mid attention (head dim 512, scale 1 / sqrt(512))."""
    r = _rng(512)
    B, S, C = 1, 96, 512
    q, k, v = (r.standard_normal((B, 1, S, C)).astype(np.float32) for _ in range(3))
    out = np.zeros_like(q)
    libs["attn"].ref_cpu_attention(_p(q), _p(k), _p(v), B, 1, S, S, C, ctypes.c_float(1.0 / math.sqrt(C)),
                                   _p(out))
    got = V.mid_attention(*(torch.from_numpy(a[:, 0]) for a in (q, k, v))).numpy()
    assert _rel(got, out[:, 0]) <= 2e-5
