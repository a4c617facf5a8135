"""GPU test of the GroupNorm entry point that allocates nothing (dlm_group_norm_nhwc_noalloc).

It exists for callers that cannot hand the library a scratch buffer: a host whose device memory
is owned entirely by its own pre-reserved arena, or a loop that must not pay cudaMalloc's
implicit synchronisation.  Its partial sums live in a static device array of the library.

The tests call it through the C ABI several times in a row, on different inputs and batch sizes
(the array keeps the previous call's partial sums and statistics, which must not leak into the
next result), and compare each output with the existing scratch-buffer entry point
dlm_group_norm_nhwc and with an fp32 GroupNorm, within the per-layer tolerance of the other
parity tests.  It also checks that a problem too large for the static
array is rejected.  This file is collected last, and passes alone in a fresh process as well as
after the other tests.
"""
import ctypes

import pytest
import torch

from dollama_b200 import _lib as L
from tests.helpers import max_rel_err

pytestmark = pytest.mark.gpu


def _p(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _s():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _inputs(seed, N, H, W, C1, C2):
    g = torch.Generator().manual_seed(seed)
    x1 = (torch.randn(N, H, W, C1, generator=g) * 1.5 + 0.25 * seed).half().cuda()
    x2 = (torch.randn(N, H, W, C2, generator=g) - 0.5).half().cuda() if C2 else None
    C = C1 + C2
    gam = (1 + 0.1 * torch.randn(C, generator=g)).half().cuda()
    bet = (0.1 * torch.randn(C, generator=g)).half().cuda()
    return x1, x2, gam, bet


def _with_scratch(x1, x2, C1, C2, N, HW, gam, bet, eps, silu):
    out = torch.empty(N * HW * (C1 + C2), dtype=torch.float16, device="cuda")
    nb = L.lib().dlm_group_norm_nhwc_scratch_bytes(N, HW)
    scratch = torch.empty(nb, dtype=torch.uint8, device="cuda")
    L.call("dlm_group_norm_nhwc", _p(x1), C1, _p(x2), C2, N, HW, _p(gam), _p(bet), eps, 32, silu,
           _p(out), _p(scratch), nb, _s())
    return out


def _no_alloc(x1, x2, C1, C2, N, HW, gam, bet, eps, silu):
    out = torch.empty(N * HW * (C1 + C2), dtype=torch.float16, device="cuda")
    L.call("dlm_group_norm_nhwc_noalloc", _p(x1), C1, _p(x2), C2, N, HW, _p(gam), _p(bet), eps, 32,
           silu, _p(out), _s())
    return out


def test_no_alloc_group_norm_matches_scratch_entry_point_twice():
    shapes = [(2, 64, 64, 640, 320, 1, 1e-5), (2, 32, 32, 1280, 0, 0, 1e-6)]
    for call, (N, H, W, C1, C2, silu, eps) in enumerate(shapes):
        x1, x2, gam, bet = _inputs(100 + call, N, H, W, C1, C2)
        ref = _with_scratch(x1, x2, C1, C2, N, H * W, gam, bet, eps, silu)
        got = _no_alloc(x1, x2, C1, C2, N, H * W, gam, bet, eps, silu)
        torch.cuda.synchronize()
        assert max_rel_err(got, ref) < 2e-3, (call, max_rel_err(got, ref))
        f32 = _fp32_group_norm(x1, x2, N, H, W, gam, bet, eps, silu)
        assert max_rel_err(got, f32) < 2e-3, (call, max_rel_err(got, f32))
    code = ctypes.c_int(-1)
    L.call("dlm_get_device_status", ctypes.byref(code), 1, _s())
    assert code.value == 0


def _fp32_group_norm(x1, x2, N, H, W, gam, bet, eps, silu):
    x = x1.float().view(N, H, W, -1)
    if x2 is not None:
        x = torch.cat([x, x2.float().view(N, H, W, -1)], dim=3)
    y = torch.nn.functional.group_norm(x.permute(0, 3, 1, 2), 32, gam.float(), bet.float(), eps)
    if silu:
        y = torch.nn.functional.silu(y)
    return y.permute(0, 2, 3, 1).reshape(-1)


def test_no_alloc_group_norm_batch_changes_between_calls():
    """The arrival counters sit after the N x 32 statistics slots, so a call with another batch
    finds the previous call's statistics where its counters go.  Sequences that grow and shrink N
    (with and without SiLU, with different image sizes) must each match the scratch entry point
    and an fp32 GroupNorm."""
    seq = [(2, 16, 16, 320, 0, 1, 1e-5), (1, 24, 24, 320, 0, 0, 1e-5),
           (3, 8, 8, 640, 640, 1, 1e-6), (1, 32, 16, 256, 64, 0, 1e-6),
           (2, 16, 16, 320, 0, 1, 1e-5), (5, 12, 12, 512, 0, 1, 1e-6),
           (1, 40, 40, 320, 320, 1, 1e-5)]
    for call, (N, H, W, C1, C2, silu, eps) in enumerate(seq):
        x1, x2, gam, bet = _inputs(200 + call, N, H, W, C1, C2)
        got = _no_alloc(x1, x2, C1, C2, N, H * W, gam, bet, eps, silu)
        ref = _with_scratch(x1, x2, C1, C2, N, H * W, gam, bet, eps, silu)
        torch.cuda.synchronize()
        assert max_rel_err(got, ref) < 2e-3, (call, max_rel_err(got, ref))
        f32 = _fp32_group_norm(x1, x2, N, H, W, gam, bet, eps, silu)
        assert max_rel_err(got, f32) < 2e-3, (call, max_rel_err(got, f32))
    code = ctypes.c_int(-1)
    L.call("dlm_get_device_status", ctypes.byref(code), 1, _s())
    assert code.value == 0


def test_no_alloc_group_norm_rejects_oversized_problem():
    cap = L.lib().dlm_group_norm_nhwc_noalloc_capacity()
    assert cap > 0
    N = cap  # far more images than the static partial-sum array can hold
    x1 = torch.zeros(64, dtype=torch.float16, device="cuda")
    gam = torch.ones(64, dtype=torch.float16, device="cuda")
    bet = torch.zeros(64, dtype=torch.float16, device="cuda")
    out = torch.empty(64, dtype=torch.float16, device="cuda")
    rc = L.lib().dlm_group_norm_nhwc_noalloc(_p(x1), 64, None, 0, N, 1, _p(gam), _p(bet), 1e-5, 32,
                                              0, _p(out), _s())
    assert rc == -1
    assert "static" in L.last_error()
