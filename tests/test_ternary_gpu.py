"""BitNet ternary x int8 linear on the GPU, bit-exact against the CPU oracle
(oracle/bitnet_oracle.c, itself pinned to the reference's src/models/bitnet.hpp).

Covers: weight packing (codes + per-row alpha), per-token activation quantization (codes +
scale), the GEMM at the tag LM's shapes for batched decode (M = 256 sequences) and a prefill
slice, ragged M / N, all-zero rows (alpha = 0) and all-zero tokens (scale = 0), and the fused
dlm_bitlinear call; y must match bit for bit (compared as raw 32-bit patterns).
"""
import ctypes

import numpy as np
import pytest
import torch

from dollama_b200 import _lib as L
from oracle import bitnet as B

pytestmark = pytest.mark.gpu


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def _s():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def unpack(packed, N, K):
    """[N, K/16] uint32 codes -> int8 {-1,0,1} [N, K]."""
    p = packed.view(np.uint32).reshape(N, K // 16)
    out = np.zeros((N, K), np.int8)
    for j in range(16):
        c = (p >> (2 * j)) & 3
        out[:, j::16] = np.where(c == 1, 1, np.where(c == 3, -1, 0))
    return out


def gpu_pack(w):
    N, K = w.shape
    wt = torch.from_numpy(w).cuda()
    packed = torch.zeros(N * K // 16, dtype=torch.int32, device="cuda")
    alpha = torch.zeros(N, dtype=torch.float32, device="cuda")
    L.call("dlm_ternary_pack", _p(wt), N, K, _p(packed), _p(alpha), _s())
    torch.cuda.synchronize()
    return packed, alpha


@pytest.mark.parametrize("N,K", [(512, 512), (1536, 512), (512, 1536), (64, 64), (70, 128)])
def test_pack_bit_exact(N, K):
    rng = np.random.default_rng(N + K)
    w = (rng.standard_normal((N, K)) * 0.05).astype(np.float32)
    w[3] = 0.0  # alpha = 0 row
    packed, alpha = gpu_pack(w)
    q_ref, a_ref = B.quant_weight_rows(w)
    assert np.array_equal(alpha.cpu().numpy().view(np.uint32), a_ref.view(np.uint32))
    assert np.array_equal(unpack(packed.cpu().numpy(), N, K), q_ref)


@pytest.mark.parametrize("M,K", [(256, 512), (256, 1536), (33, 64), (1, 512)])
def test_quant_act_bit_exact(M, K):
    rng = np.random.default_rng(M * 3 + K)
    x = (rng.standard_normal((M, K)) * 3).astype(np.float32)
    x[0] = 0.0  # scale = 0 token
    if M > 2:
        x[1, :] = 0.5  # ties for round-half-away
    xt = torch.from_numpy(x).cuda()
    xq = torch.zeros(M * K, dtype=torch.int8, device="cuda")
    xs = torch.zeros(M, dtype=torch.float32, device="cuda")
    L.call("dlm_quantize_act_i8", _p(xt), M, K, _p(xq), _p(xs), _s())
    torch.cuda.synchronize()
    q_ref, s_ref = B.quant_act_rows(x)
    assert np.array_equal(xs.cpu().numpy().view(np.uint32), s_ref.view(np.uint32))
    assert np.array_equal(xq.cpu().numpy().reshape(M, K), q_ref)


# M >= 1024 runs the tcgen05 kind::i8 tensor-core path (prefill); smaller M runs the decode
# tensor-core path (32-output tiles, 64-output ones when 32 would need more than two CTAs per SM;
# a four-block activation ring beyond K = 512) where K is a multiple of 128 up to 2048 and N a
# multiple of 32, else dp4a
@pytest.mark.parametrize("M,N,K", [(256, 512, 512), (256, 1536, 512), (256, 512, 1536),
                                   (2048, 512, 512), (37, 70, 192), (1, 64, 64),
                                   (1040, 3072, 512), (1024, 512, 1536), (1152, 96, 256),
                                   (256, 3072, 512), (512, 3072, 512), (100, 96, 256),
                                   (1, 32, 128), (300, 640, 384), (200, 96, 1024),
                                   (256, 64, 2048)])
def test_bitlinear_bit_exact(M, N, K):
    rng = np.random.default_rng(M + 7 * N + K)
    w = (rng.standard_normal((N, K)) * 0.05).astype(np.float32)
    x = (rng.standard_normal((M, K)) * 2).astype(np.float32)
    w[-1] = 0.0
    x[0] = 0.0
    packed, alpha = gpu_pack(w)
    xt = torch.from_numpy(x).cuda()
    y = torch.empty(M, N, dtype=torch.float32, device="cuda")
    xq = torch.zeros(M * K, dtype=torch.int8, device="cuda")
    xs = torch.zeros(M, dtype=torch.float32, device="cuda")
    L.call("dlm_bitlinear", _p(packed), _p(alpha), _p(xt), _p(y), M, N, K, _p(xq), _p(xs), _s())
    torch.cuda.synchronize()
    wq, a = B.quant_weight_rows(w)
    q, s = B.quant_act_rows(x)
    y_ref, _ = B.ternary_gemm(wq, a, q, s)
    got = y.cpu().numpy()
    assert np.array_equal(got.view(np.uint32), y_ref.view(np.uint32))
    if M <= 4:
        for m in range(M):
            assert np.array_equal(got[m], B.bitlinear(w, x[m]))


def test_gemm_linearity_full_prefill():
    """Prefill size (256 x 64 tokens): exactness via a size-independent property — the integer
    sums are linear, so y(xq1 + xq2) scaled back equals the sum of the parts when both share
    the same scales."""
    M, N, K = 16384, 512, 512
    rng = np.random.default_rng(11)
    w = (rng.standard_normal((N, K)) * 0.05).astype(np.float32)
    packed, alpha = gpu_pack(w)
    xq1 = torch.from_numpy(rng.integers(-63, 64, (M, K), dtype=np.int8)).cuda()
    xq2 = torch.from_numpy(rng.integers(-63, 64, (M, K), dtype=np.int8)).cuda()
    ones = torch.ones(M, dtype=torch.float32, device="cuda")
    ones_a = torch.ones(N, dtype=torch.float32, device="cuda")
    ys = []
    for xq in (xq1, xq2, (xq1.int() + xq2.int()).to(torch.int8)):
        y = torch.empty(M, N, dtype=torch.float32, device="cuda")
        L.call("dlm_ternary_gemm_i8", _p(packed), _p(ones_a), _p(xq), _p(ones), _p(y), M, N, K, _s())
        ys.append(y)
    torch.cuda.synchronize()
    assert torch.equal(ys[0] + ys[1], ys[2])
    # spot-check a slice against the oracle
    wq = unpack(packed.cpu().numpy(), N, K)
    sl = slice(0, 64)
    y_ref, acc = B.ternary_gemm(wq, np.ones(N, np.float32), xq1[sl].cpu().numpy(), np.ones(64, np.float32))
    assert np.array_equal(ys[0][sl].cpu().numpy(), acc.astype(np.float32))
