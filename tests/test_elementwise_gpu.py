"""The reference's small kernel host functions (bias adds, activations, add, upsample, GEGLU,
timestep embedding, fp32 GEMM, batched / transposed fp16 GEMM) against PyTorch on the GPU.

Rounding sequences follow the reference (src/kernels/bias_add.cuh:32-103, activation.cu:25-69,
elementwise.cuh:26-37, geglu.cu:26-48, timeembed.cu:30-49): the pure add / broadcast ops must be
bit-exact; the transcendental ones (CUDA's __expf / erff / tanhf / cosf / sinf against torch's)
within two fp16 units in the last place (fp32 evaluation, then one rounding to fp16, against a
float64 reference).
"""
import ctypes
import math

import pytest
import torch

from dollama_b200 import _lib as L
from tests.helpers import max_rel_err

pytestmark = pytest.mark.gpu


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def _s():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _rand(*shape, seed=0, scale=1.0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).half().cuda()


def _ulp_close(got, ref, ulps=1):
    """|got - ref| <= ulps fp16 units of ref (ref rounded to fp16 first)."""
    r = ref.half().float()
    spacing = torch.where(r.abs() < 6.1e-5, torch.full_like(r, 2.0 ** -24),
                          2.0 ** (torch.floor(torch.log2(r.abs().clamp_min(6.1e-5))) - 10))
    return bool(((got.float() - r).abs() <= ulps * spacing + 1e-30).all())


def test_bias_add_rowvec_exact_and_inplace():
    x, b = _rand(37, 320, seed=1), _rand(320, seed=2)
    ref = (x.float() + b.float()).half()
    out = torch.empty_like(x)
    L.call("dlm_bias_add_rowvec", _p(x), _p(b), _p(out), 37, 320, _s())
    L.call("dlm_bias_add_rowvec", _p(x), _p(b), _p(x), 37, 320, _s())  # in place
    torch.cuda.synchronize()
    assert torch.equal(out, ref) and torch.equal(x, ref)


def test_bias_add_channel_exact():
    x, b = _rand(2, 5, 3, 7, seed=3), _rand(5, seed=4)
    ref = (x.float() + b.float()[None, :, None, None]).half()
    out = torch.empty_like(x)
    L.call("dlm_bias_add_channel", _p(x), _p(b), _p(out), 2, 5, 3, 7, _s())
    torch.cuda.synchronize()
    assert torch.equal(out, ref)


def test_conv_bias_biasch_two_roundings():
    B, C, H, W = 2, 6, 4, 5
    conv, cb, tp = _rand(B, C, H, W, seed=5), _rand(C, seed=6), _rand(B, C, seed=7)
    t = (conv.float() + cb.float()[None, :, None, None]).half()
    ref = (t.float() + tp.float()[:, :, None, None]).half()
    out = torch.empty_like(conv)
    L.call("dlm_conv_bias_biasch", _p(conv), _p(cb), _p(tp), _p(out), B, C, H, W, _s())
    torch.cuda.synchronize()
    assert torch.equal(out, ref)


def test_conv_bias_residual_two_roundings():
    B, C, H, W = 2, 6, 4, 5
    conv, cb, res = _rand(B, C, H, W, seed=8), _rand(C, seed=9), _rand(B, C, H, W, seed=10)
    t = (conv.float() + cb.float()[None, :, None, None]).half()
    ref = (t.float() + res.float()).half()
    L.call("dlm_conv_bias_residual", _p(conv), _p(cb), _p(res), _p(conv), B, C, H, W, _s())  # in place
    torch.cuda.synchronize()
    assert torch.equal(conv, ref)


@pytest.mark.parametrize("name", ["dlm_silu", "dlm_gelu", "dlm_gelu_tanh"])
def test_activations(name):
    x = _rand(4099, seed=11, scale=3.0)
    xf = x.float().cpu().double()
    if name == "dlm_silu":
        ref = xf / (1.0 + torch.exp(-xf))
    elif name == "dlm_gelu":
        ref = 0.5 * xf * (1.0 + torch.erf(xf / math.sqrt(2.0)))
    else:
        ref = 0.5 * xf * (1.0 + torch.tanh(math.sqrt(2.0 / math.pi) * (xf + 0.044715 * xf ** 3)))
    out = torch.empty_like(x)
    L.call(name, _p(x), _p(out), x.numel(), _s())
    torch.cuda.synchronize()
    assert _ulp_close(out.cpu(), ref.float(), ulps=2)


def test_add_and_upsample_exact():
    a, b = _rand(1000, seed=12), _rand(1000, seed=13)
    out = torch.empty_like(a)
    L.call("dlm_add", _p(a), _p(b), _p(out), 1000, _s())
    x = _rand(2, 3, 5, 7, seed=14)
    up = torch.empty(2, 3, 10, 14, dtype=torch.float16, device="cuda")
    L.call("dlm_upsample_nearest2x", _p(x), _p(up), 2, 3, 5, 7, _s())
    torch.cuda.synchronize()
    assert torch.equal(out, (a.float() + b.float()).half())
    assert torch.equal(up, torch.nn.functional.interpolate(x, scale_factor=2, mode="nearest"))


def test_geglu():
    tokens, d = 33, 96
    x = _rand(tokens, 2 * d, seed=15, scale=2.0)
    xf = x.float().cpu().double()
    x1, x2 = xf[:, :d], xf[:, d:]
    ref = x1 * (0.5 * x2 * (1.0 + torch.erf(x2 / math.sqrt(2.0))))
    out = torch.empty(tokens, d, dtype=torch.float16, device="cuda")
    L.call("dlm_geglu", _p(x), _p(out), tokens, d, _s())
    torch.cuda.synchronize()
    # the reference's fp32 formula loses bits in 1 + erf(x2 / sqrt 2) for negative x2 (one fp32
    # ulp of erf, 2^-24, times 0.5 |x1 x2|), on top of the two fp16 units of the rounding
    got = out.cpu().double()
    r16 = ref.float().half().double()
    spacing = torch.clamp(2.0 ** (torch.floor(torch.log2(r16.abs().clamp_min(6.1e-5))) - 10), min=2.0 ** -24)
    bound = 2 * spacing + 0.5 * (x1 * x2).abs() * 2.0 ** -23
    assert bool(((got - ref).abs() <= bound).all())


@pytest.mark.parametrize("t", [0.0, 1.0, 499.0, 999.0])
def test_timestep_embedding(t):
    dim = 320
    half = dim // 2
    i = torch.arange(half, dtype=torch.float64)
    args = t * torch.exp(-math.log(10000.0) * i / half)
    ref = torch.cat([torch.cos(args), torch.sin(args)])
    out = torch.empty(dim, dtype=torch.float16, device="cuda")
    L.call("dlm_timestep_embedding", _p(out), t, dim, 10000.0, _s())
    torch.cuda.synchronize()
    # fp32 argument rounding at t ~ 1e3 moves cos / sin by up to ~1e-4
    assert (out.float().cpu() - ref.float()).abs().max().item() < 2e-3


@pytest.mark.parametrize("ta,tb", [(0, 0), (0, 1), (1, 0), (1, 1)])
def test_gemm_f32(ta, tb):
    M, N, K = 77, 130, 45
    g = torch.Generator(device="cpu").manual_seed(16)
    A = torch.randn(K, M, generator=g) if ta else torch.randn(M, K, generator=g)
    B = torch.randn(N, K, generator=g) if tb else torch.randn(K, N, generator=g)
    C = torch.randn(M, N, generator=g)
    ref = 0.5 * ((A.t() if ta else A).double() @ (B.t() if tb else B).double()) + 0.25 * C.double()
    A, B, C = A.cuda(), B.cuda(), C.cuda()
    L.call("dlm_gemm_f32", _p(A), _p(B), _p(C), M, N, K, 0.5, 0.25, ta, tb, _s())
    torch.cuda.synchronize()
    assert (C.cpu().double() - ref).abs().max().item() < 1e-4


@pytest.mark.parametrize("ta,tb", [(0, 0), (1, 1), (1, 0)])
def test_gemm_fp16_transposes(ta, tb):
    M, N, K = 256, 320, 192
    A = _rand(K, M, seed=17) if ta else _rand(M, K, seed=17)
    B = _rand(N, K, seed=18, scale=K ** -0.5) if tb else _rand(K, N, seed=18, scale=K ** -0.5)
    C = _rand(M, N, seed=19)
    ref = 1.5 * ((A.t() if ta else A).float() @ (B.t() if tb else B).float()) + 0.5 * C.float()
    L.call("dlm_launch_gemm_fp16", _p(A), _p(B), _p(C), M, N, K, 1.5, 0.5, ta, tb, _s())
    torch.cuda.synchronize()
    assert max_rel_err(C, ref) < 3e-3


def test_gemm_fp16_batched_shared_a():
    batch, M, N, K = 3, 128, 256, 128
    A = _rand(M, K, seed=20)  # stride_a = 0: shared by every item
    B = _rand(batch, N, K, seed=21, scale=K ** -0.5)
    C = _rand(batch, M, N, seed=22)
    ref = torch.stack([A.float() @ B[i].float().t() + 2.0 * C[i].float() for i in range(batch)])
    L.call("dlm_gemm_fp16_batched", _p(A), _p(B), _p(C), batch, M, N, K, 0, N * K, M * N, 1.0, 2.0, 1,
           _s())
    torch.cuda.synchronize()
    assert max_rel_err(C, ref) < 3e-3


def test_empty_sizes_return_ok():
    assert L.lib().dlm_add(None, None, None, 0, None) == 0
    assert L.lib().dlm_geglu(None, None, 0, 8, None) == 0
    assert L.lib().dlm_gemm_f32(None, None, None, 0, 4, 4, 1.0, 0.0, 0, 0, None) == 0
