"""Implicit-GEMM conv2d parity against torch fp32 F.conv2d on the same fp16 inputs (GPU).

Covers the reference's conv shapes (src/infer/unet.cu resnet / down / up convs): 3x3 pad 1
stride 1, 3x3 stride 2 (Downsample2D) and 1x1 (conv_shortcut), at several widths so that the
128-pixel tile covers 1, 2 or 4 image rows, plus zero padding at every border.
"""
import ctypes

import pytest
import torch
import torch.nn.functional as F

from dollama_b200 import _lib as L
from tests.helpers import max_rel_err, allclose_k

pytestmark = pytest.mark.gpu


def _p(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _s():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def run_conv(x_nchw, w, b, ksize, stride):
    N, Cin, H, W = x_nchw.shape
    Cout = w.shape[0]
    x = x_nchw.permute(0, 2, 3, 1).contiguous()
    wp = torch.empty(Cout, ksize, ksize, Cin, dtype=torch.float16, device="cuda")
    L.call("dlm_pack_conv_weight", _p(w), _p(wp), Cout, Cin, ksize, ksize, _s())
    oH, oW = H // stride, W // stride
    out = torch.empty(N, oH, oW, Cout, dtype=torch.float16, device="cuda")
    nbytes = L.lib().dlm_conv2d_nhwc_scratch_bytes(N, H, W, Cin, ksize, stride)
    scratch = torch.empty(max(nbytes, 16), dtype=torch.uint8, device="cuda")
    L.call("dlm_conv2d_nhwc", _p(x), N, H, W, Cin, _p(wp), _p(b), _p(out), Cout, ksize, stride,
           _p(scratch), nbytes, _s())
    torch.cuda.synchronize()
    return out.permute(0, 3, 1, 2)


@pytest.fixture(params=[0, 1, 2], ids=["auto", "single", "pair"])
def tile_mode(request):
    L.call("dlm_gemm_set_tile_mode", request.param)
    yield request.param
    L.call("dlm_gemm_set_tile_mode", 0)


@pytest.mark.parametrize("N,Cin,H,W,Cout,k,s", [
    (1, 64, 16, 16, 64, 3, 1),
    (2, 320, 32, 32, 320, 3, 1),
    (2, 128, 64, 64, 640, 3, 1),
    (1, 192, 128, 128, 320, 3, 1),
    (1, 64, 8, 256, 128, 3, 1),
    (2, 320, 64, 64, 320, 3, 2),
    (2, 640, 32, 32, 1280, 1, 1),
])
def test_conv(N, Cin, H, W, Cout, k, s, tile_mode):
    g = torch.Generator().manual_seed(N * 1000 + Cin + H)
    x = torch.randn(N, Cin, H, W, generator=g).half().cuda()
    bound = (Cin * k * k) ** -0.5
    w = ((torch.rand(Cout, Cin, k, k, generator=g) * 2 - 1) * bound).half().cuda()
    b = ((torch.rand(Cout, generator=g) * 2 - 1) * bound).half().cuda()
    got = run_conv(x, w, b, k, s)
    ref = F.conv2d(x.float(), w.float(), b.float(), stride=s, padding=k // 2)
    assert got.shape == ref.shape
    err = max_rel_err(got, ref)
    assert err < 2e-3, f"max rel err {err}"
    assert allclose_k(got, ref, Cin * k * k)
