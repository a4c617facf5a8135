"""tcgen05 GEMM parity against a PyTorch fp32 reference of the same op (GPU).

The reference's Linear path is launch_gemm_fp16(transB=1) + launch_bias_add_rowvec +
launch_add / launch_geglu (src/infer/unet.cu:517-526, 759-770); the fused epilogues here must
match that math within the fp16 storage tolerance.
"""
import ctypes

import pytest
import torch

from dollama_b200 import _lib as L
from tests.helpers import max_rel_err

pytestmark = pytest.mark.gpu


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _rand(*shape, scale=1.0, seed=0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).half().cuda()


@pytest.fixture(params=[0, 1, 2], ids=["auto", "single", "pair"])
def tile_mode(request):
    L.call("dlm_gemm_set_tile_mode", request.param)
    yield request.param
    L.call("dlm_gemm_set_tile_mode", 0)


@pytest.mark.parametrize("M,N,K", [(128, 128, 64), (256, 320, 640), (8192, 640, 640),
                                   (2048, 1280, 1280), (154, 1280, 2048), (300, 96, 72),
                                   (8192, 1920, 640), (2048, 10240, 1280),
                                   (2, 1280, 2816), (64, 256, 128)])
def test_gemm_plain(M, N, K, tile_mode):
    A = _rand(M, K, seed=1)
    W = _rand(N, K, scale=K ** -0.5, seed=2)
    C = torch.empty(M, N, dtype=torch.float16, device="cuda")
    L.call("dlm_launch_gemm_fp16", _ptr(A), _ptr(W), _ptr(C), M, N, K, 1.0, 0.0, 0, 1, _stream())
    torch.cuda.synchronize()
    ref = A.float() @ W.float().t()
    err = max_rel_err(C, ref)
    assert err < 2e-3, f"max rel err {err}"


def test_gemm_bias_resid_inplace(tile_mode):
    M, N, K = 1024, 640, 640
    A = _rand(M, K, seed=3)
    W = _rand(N, K, scale=K ** -0.5, seed=4)
    b = _rand(N, seed=5)
    X = _rand(M, N, seed=6)
    ref = X.float() + A.float() @ W.float().t() + b.float()
    L.call("dlm_gemm_fp16_ex", _ptr(A), K, _ptr(W), _ptr(X), N, M, N, K,
           L.EPI_BIAS | L.EPI_RESID, _ptr(b), None, 0, _ptr(X), N, _stream())
    torch.cuda.synchronize()
    assert max_rel_err(X, ref) < 2e-3


def test_gemm_geglu_interleaved(tile_mode):
    M, C = 512, 320
    ff = 4 * C
    A = _rand(M, C, seed=7)
    W = _rand(2 * ff, C, scale=C ** -0.5, seed=8)
    b = _rand(2 * ff, scale=0.1, seed=9)
    # interleave rows (x1_j, x2_j) as the model's weight prep does
    Wi = torch.stack([W[:ff], W[ff:]], dim=1).reshape(2 * ff, C).contiguous()
    bi = torch.stack([b[:ff], b[ff:]], dim=1).reshape(2 * ff).contiguous()
    out = torch.empty(M, ff, dtype=torch.float16, device="cuda")
    L.call("dlm_gemm_fp16_ex", _ptr(A), C, _ptr(Wi), _ptr(out), ff, M, 2 * ff, C,
           L.EPI_BIAS | L.EPI_GEGLU, _ptr(bi), None, 0, None, 0, _stream())
    torch.cuda.synchronize()
    h = A.float() @ W.float().t() + b.float()
    ref = h[:, :ff] * torch.nn.functional.gelu(h[:, ff:])
    assert max_rel_err(out, ref) < 2e-3


def test_gemm_bias2d_silu(tile_mode):
    M, N, K, rows = 512, 256, 128, 128
    A = _rand(M, K, seed=10)
    W = _rand(N, K, scale=K ** -0.5, seed=11)
    b2 = _rand(M // rows, N, seed=12)
    out = torch.empty(M, N, dtype=torch.float16, device="cuda")
    L.call("dlm_gemm_fp16_ex", _ptr(A), K, _ptr(W), _ptr(out), N, M, N, K,
           L.EPI_BIAS2D | L.EPI_SILU, None, _ptr(b2), rows, None, 0, _stream())
    torch.cuda.synchronize()
    h = A.float() @ W.float().t() + b2.float().repeat_interleave(rows, dim=0)
    ref = torch.nn.functional.silu(h)
    assert max_rel_err(out, ref) < 2e-3


def test_device_status_clean():
    code = ctypes.c_int(-1)
    L.call("dlm_get_device_status", ctypes.byref(code), 1, _stream())
    assert code.value == 0


@pytest.mark.parametrize("M,N,K,ta,tb,beta", [(320, 36, 4, 0, 0, 0.0),     # a LoRA delta B @ A
                                                (37, 50, 13, 0, 1, 0.0),
                                                (64, 96, 72, 1, 0, 0.5),
                                                (33, 17, 40, 1, 1, -1.0),
                                                (128, 64, 64, 0, 0, 1.0)])
def test_gemm_any_shape_and_orientation(M, N, K, ta, tb, beta):
    """The reference's launch_gemm_fp16 (cuBLAS) takes any M, N, K and both orientations
    (src/kernels/gemm.cuh:44-53): sizes off the tensor-core kernel's granularity go through
    zero-padded scratch."""
    A = _rand(*((K, M) if ta else (M, K)), seed=3)
    B = _rand(*((N, K) if tb else (K, N)), scale=K ** -0.5, seed=4)
    C = _rand(M, N, seed=5)
    C0 = C.clone()
    L.call("dlm_launch_gemm_fp16", _ptr(A), _ptr(B), _ptr(C), M, N, K, 0.75, beta, ta, tb, _stream())
    torch.cuda.synchronize()
    a = A.float().t() if ta else A.float()
    b = B.float() if tb else B.float().t()
    ref = 0.75 * (a @ b.t()) + beta * C0.float()
    assert max_rel_err(C, ref) < 2e-3, max_rel_err(C, ref)


def test_gemm_invalid_arguments():
    # every orientation is provided (transposed operands go through scratch); a null operand is
    # an invalid argument, reported without launching
    A = _rand(128, 64)
    rc = L.lib().dlm_launch_gemm_fp16(_ptr(A), None, _ptr(A), 128, 64, 64, 1.0, 0.0, 1, 1, _stream())
    assert rc == -1


# ---------------------------------------------------------------- stream-K

@pytest.fixture(scope="module")
def sk_workspace():
    nbytes = L.lib().dlm_gemm_workspace_bytes()
    ws = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    return ws, nbytes


@pytest.mark.parametrize("mode", [3, 3 + 16 * 160, 3 + 16 * 128, 0], ids=["sk256", "sk160", "sk128", "auto"])
@pytest.mark.parametrize("M,N,K", [(2048, 1280, 5120),   # tiles cut between two or three CTAs
                                   (300, 320, 1280),     # partial M and N tiles
                                   (128, 256, 8192),     # one tile over 128 CTAs (one k-block each)
                                   (256, 512, 128),      # fewer k-blocks than CTAs: idle CTAs
                                   (8192, 640, 2560)])
def test_gemm_stream_k(M, N, K, mode, sk_workspace):
    ws, nbytes = sk_workspace
    L.call("dlm_gemm_set_tile_mode", mode)
    try:
        A = _rand(M, K, seed=11)
        W = _rand(N, K, scale=K ** -0.5, seed=12)
        b = _rand(N, seed=13)
        X = _rand(M, N, seed=14)
        ref = X.float() + A.float() @ W.float().t() + b.float()
        outs = []
        for _ in range(2):   # the second launch checks that the first left the flags clear
            C = X.clone()
            L.call("dlm_gemm_fp16_ws", _ptr(A), K, _ptr(W), _ptr(C), N, M, N, K,
                   L.EPI_BIAS | L.EPI_RESID, _ptr(b), _ptr(C), N, _ptr(ws), nbytes, _stream())
            torch.cuda.synchronize()
            outs.append(C)
        assert torch.equal(outs[0], outs[1])   # fixed-order partial sums: deterministic
        err = max_rel_err(outs[0], ref)
        assert err < 2e-3, f"max rel err {err}"
        code = ctypes.c_int()
        L.call("dlm_get_device_status", ctypes.byref(code), 1, _stream())
        assert code.value == 0
    finally:
        L.call("dlm_gemm_set_tile_mode", 0)


def test_gemm_stream_k_geglu(sk_workspace):
    ws, nbytes = sk_workspace
    L.call("dlm_gemm_set_tile_mode", 3)
    try:
        M, N, K = 512, 1024, 4096
        A = _rand(M, K, seed=21)
        W = _rand(N, K, scale=K ** -0.5, seed=22)
        b = _rand(N, seed=23)
        C = torch.empty(M, N // 2, dtype=torch.float16, device="cuda")
        L.call("dlm_gemm_fp16_ws", _ptr(A), K, _ptr(W), _ptr(C), N // 2, M, N, K,
               L.EPI_BIAS | L.EPI_GEGLU, _ptr(b), None, 0, _ptr(ws), nbytes, _stream())
        torch.cuda.synchronize()
        y = A.float() @ W.float().t() + b.float()
        ref = y[:, 0::2] * torch.nn.functional.gelu(y[:, 1::2])
        assert max_rel_err(C, ref) < 2e-3
    finally:
        L.call("dlm_gemm_set_tile_mode", 0)
