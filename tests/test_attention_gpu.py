"""tcgen05 flash attention parity against a PyTorch fp32 softmax(QK^T/8)V (GPU).

Shapes are the UNet's (src/infer/unet.cu:677-797): self-attention at 32^2 / 64^2 tokens,
cross-attention to 77 context tokens (keys masked beyond Sk), both in the reference's
[B, H, S, 64] layout and in the token-major layout the UNet uses.  Tolerance: the per-layer
bar max|err|/max|ref| <= 2e-3 plus the reference's attention tolerance
(src/tests/test_attention_fast.cu:56-63).
"""
import ctypes
import math

import pytest
import torch

from dollama_b200 import _lib as L
from tests.helpers import max_rel_err, allclose_k

pytestmark = pytest.mark.gpu


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def _s():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def ref_attn(q, k, v):
    s = (q.float() @ k.float().transpose(-1, -2)) / 8.0
    return torch.softmax(s, dim=-1) @ v.float()


@pytest.mark.parametrize("B,H,Sq,Sk", [(1, 1, 128, 128), (2, 10, 1024, 1024), (2, 10, 4096, 4096),
                                       (2, 20, 1024, 77), (1, 2, 256, 300), (2, 3, 200, 130)])
def test_attention_bhsd(B, H, Sq, Sk):
    g = torch.Generator().manual_seed(B * 100 + Sq + Sk)
    q = torch.randn(B, H, Sq, 64, generator=g).half().cuda()
    k = torch.randn(B, H, Sk, 64, generator=g).half().cuda()
    v = torch.randn(B, H, Sk, 64, generator=g).half().cuda()
    o = torch.empty_like(q)
    L.call("dlm_launch_attention", _p(q), _p(k), _p(v), _p(o), B, H, Sq, Sk, 64, 1.0 / 8.0, _s())
    torch.cuda.synchronize()
    ref = ref_attn(q, k, v)
    assert max_rel_err(o, ref) < 2e-3
    assert allclose_k(o, ref, Sk)


def test_attention_tokens_cross():
    B, H, Sq, Sk = 2, 10, 4096, 77
    C = H * 64
    g = torch.Generator().manual_seed(5)
    qkv = torch.randn(B * Sq, C, generator=g).half().cuda()
    kv = torch.randn(B * Sk, 2 * C, generator=g).half().cuda()
    out = torch.empty(B * Sq, C, dtype=torch.float16, device="cuda")
    L.call("dlm_attention_tokens", _p(qkv), C, _p(kv), 2 * C, ctypes.c_void_p(kv.data_ptr() + 2 * C),
           2 * C, _p(out), C, B, H, Sq, Sk, 64, 0.125, _s())
    torch.cuda.synchronize()
    q = qkv.view(B, Sq, H, 64).transpose(1, 2)
    k = kv[:, :C].reshape(B, Sk, H, 64).transpose(1, 2)
    v = kv[:, C:].reshape(B, Sk, H, 64).transpose(1, 2)
    ref = ref_attn(q, k, v).transpose(1, 2).reshape(B * Sq, C)
    assert max_rel_err(out, ref) < 2e-3


def test_attention_tokens_self_fused_qkv():
    B, H, S = 2, 20, 1024
    C = H * 64
    g = torch.Generator().manual_seed(6)
    qkv = torch.randn(B * S, 3 * C, generator=g).half().cuda()
    out = torch.empty(B * S, C, dtype=torch.float16, device="cuda")
    base = qkv.data_ptr()
    L.call("dlm_attention_tokens", ctypes.c_void_p(base), 3 * C, ctypes.c_void_p(base + 2 * C), 3 * C,
           ctypes.c_void_p(base + 4 * C), 3 * C, _p(out), C, B, H, S, S, 64, 0.125, _s())
    torch.cuda.synchronize()
    t = qkv.view(B, S, 3, H, 64)
    q, k, v = (t[:, :, i].transpose(1, 2) for i in range(3))
    ref = ref_attn(q, k, v).transpose(1, 2).reshape(B * S, C)
    assert max_rel_err(out, ref) < 2e-3


@pytest.fixture(scope="module")
def attn_ws():
    nbytes = L.lib().dlm_attention_workspace_bytes(2, 20, 4096)
    return torch.zeros(nbytes, dtype=torch.uint8, device="cuda"), nbytes


@pytest.mark.parametrize("B,H,Sq,Sk", [(2, 10, 4096, 4096),   # 320 groups x 32 tiles
                                       (2, 20, 1024, 1024),   # 160 groups x 8 tiles
                                       (1, 1, 256, 8192),     # one group over 64 CTAs
                                       (2, 20, 1024, 77),     # one tile per group
                                       (2, 3, 200, 1300),     # ragged queries and keys
                                       (1, 2, 256, 300)])
def test_attention_stream_k(B, H, Sq, Sk, attn_ws):
    ws, nbytes = attn_ws
    g = torch.Generator().manual_seed(B * 1000 + Sq + Sk)
    q = torch.randn(B, H, Sq, 64, generator=g).half().cuda()
    k = torch.randn(B, H, Sk, 64, generator=g).half().cuda()
    v = torch.randn(B, H, Sk, 64, generator=g).half().cuda()
    outs = []
    for _ in range(2):   # the second launch checks that the first left the counters clear
        o = torch.empty_like(q)
        L.call("dlm_launch_attention_ws", _p(q), _p(k), _p(v), _p(o), B, H, Sq, Sk, 64, 0.125,
               _p(ws), nbytes, _s())
        torch.cuda.synchronize()
        outs.append(o)
    assert torch.equal(outs[0], outs[1])   # fixed-order merges: deterministic
    ref = ref_attn(q, k, v)
    assert max_rel_err(outs[0], ref) < 2e-3
    assert allclose_k(outs[0], ref, Sk)
    code = ctypes.c_int()
    L.call("dlm_get_device_status", ctypes.byref(code), 1, _s())
    assert code.value == 0


@pytest.mark.parametrize("use_ws", [False, True])
def test_attention_growing_scores(use_ws, attn_ws):
    """Keys whose scale grows along the sequence, so a row's maximum keeps rising past the running
    maximum by more than 2^8 in later key tiles and inside a tile's second half (the lazy-max
    rescale of P already written, of the partial sums and of O)."""
    B, H, Sq, Sk = 2, 3, 256, 1024
    g = torch.Generator().manual_seed(77)
    q = (2.0 * torch.randn(B, H, Sq, 64, generator=g)).half().cuda()
    grow = (1.0 + 0.02 * torch.arange(Sk, dtype=torch.float32)).view(1, 1, Sk, 1)
    k = (torch.randn(B, H, Sk, 64, generator=g) * grow).half().cuda()
    v = torch.randn(B, H, Sk, 64, generator=g).half().cuda()
    o = torch.empty_like(q)
    if use_ws:
        ws, nbytes = attn_ws
        L.call("dlm_launch_attention_ws", _p(q), _p(k), _p(v), _p(o), B, H, Sq, Sk, 64, 0.125,
               _p(ws), nbytes, _s())
    else:
        L.call("dlm_launch_attention", _p(q), _p(k), _p(v), _p(o), B, H, Sq, Sk, 64, 0.125, _s())
    torch.cuda.synchronize()
    ref = ref_attn(q, k, v)
    assert max_rel_err(o, ref) < 2e-3
    assert allclose_k(o, ref, Sk)


# ---------------------------------------------------------------- wide heads (Dh 128..512)
# The VAE mid-block attention: one head of Dh = 512 over S = h*w tokens, which the reference runs
# through launch_attention (src/kernels/vae_decode.cu:682-683); other multiples of 64 up to 512
# and ragged query / key counts exercise the masking and the output split.

def ref_attn_scaled(q, k, v, scale):
    s = (q.float() @ k.float().transpose(-1, -2)) * scale
    return torch.softmax(s, dim=-1) @ v.float()


@pytest.mark.parametrize("B,H,Sq,Sk,Dh", [(1, 1, 256, 256, 512), (1, 1, 1024, 1024, 512),
                                          (2, 1, 200, 300, 512), (1, 2, 384, 130, 256),
                                          (1, 1, 128, 77, 128), (2, 2, 256, 512, 384)])
def test_attention_wide_bhsd(B, H, Sq, Sk, Dh):
    g = torch.Generator().manual_seed(B * 1000 + Sq + Sk + Dh)
    q = torch.randn(B, H, Sq, Dh, generator=g).half().cuda()
    k = torch.randn(B, H, Sk, Dh, generator=g).half().cuda()
    v = torch.randn(B, H, Sk, Dh, generator=g).half().cuda()
    o = torch.full_like(q, float("nan"))
    scale = 1.0 / math.sqrt(Dh)
    L.call("dlm_launch_attention", _p(q), _p(k), _p(v), _p(o), B, H, Sq, Sk, Dh, scale, _s())
    torch.cuda.synchronize()
    ref = ref_attn_scaled(q, k, v, scale)
    assert torch.isfinite(o).all()
    assert max_rel_err(o, ref) < 2e-3, max_rel_err(o, ref)
    assert allclose_k(o, ref, Sk)
    code = ctypes.c_int(-1)
    L.call("dlm_get_device_status", ctypes.byref(code), 1, _s())
    assert code.value == 0


def test_attention_wide_vae_mid_block_size():
    """The benchmarked VAE's mid attention: [16384 tokens, 512] token-major q | k | v (one head),
    fed as the VAE feeds it (strided views of one [S, 1536] projection)."""
    S, C = 16384, 512
    g = torch.Generator().manual_seed(77)
    qkv = (torch.randn(S, 3 * C, generator=g) * 0.5).half().cuda()
    out = torch.empty(S, C, dtype=torch.float16, device="cuda")
    scale = 1.0 / math.sqrt(C)
    L.call("dlm_attention_tokens", _p(qkv), 3 * C, ctypes.c_void_p(qkv.data_ptr() + 2 * C), 3 * C,
           ctypes.c_void_p(qkv.data_ptr() + 4 * C), 3 * C, _p(out), C, 1, 1, S, S, C, scale, _s())
    torch.cuda.synchronize()
    q, k, v = qkv[:, :C], qkv[:, C:2 * C], qkv[:, 2 * C:]
    ref = ref_attn_scaled(q, k, v, scale)
    assert max_rel_err(out, ref) < 2e-3, max_rel_err(out, ref)


def test_attention_wide_rejects_unsupported_head_dim():
    q = torch.zeros(1, 1, 128, 96, dtype=torch.float16, device="cuda")
    rc = L.lib().dlm_launch_attention(_p(q), _p(q), _p(q), _p(q), 1, 1, 128, 128, 96, 0.1, _s())
    assert rc == -4
