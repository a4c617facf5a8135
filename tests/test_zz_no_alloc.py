"""GPU test of the GroupNorm entry point that allocates nothing (dlm_group_norm_nhwc_noalloc).

It exists for callers that cannot hand the library a scratch buffer: a host whose device memory
is owned entirely by its own pre-reserved arena, or a loop that must not pay cudaMalloc's
implicit synchronisation.  Its partial sums live in a static device array of the library.

The test calls it through the C ABI twice in a row, on different inputs (the array keeps the
previous call's partial sums, which must not leak into the next result), and compares each
output with the existing scratch-buffer entry point dlm_group_norm_nhwc within the per-layer
tolerance of the other parity tests.  It also checks that a problem too large for the static
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
