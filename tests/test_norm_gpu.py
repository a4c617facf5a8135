"""GroupNorm / LayerNorm parity against torch fp32 (GPU): NHWC GN with eps 1e-5 / 1e-6,
optional SiLU, two-source channel concat (the up-path skip concat), group sizes that straddle
8-channel vectors and the concat boundary; LN eps 1e-5 on the transformer widths."""
import ctypes

import pytest
import torch
import torch.nn.functional as F

from dollama_b200 import _lib as L
from tests.helpers import max_rel_err

pytestmark = pytest.mark.gpu


def _p(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _s():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("N,C1,C2,H,W,silu,eps", [
    (2, 320, 0, 128, 128, 1, 1e-5), (2, 640, 320, 64, 64, 1, 1e-5), (2, 1280, 1280, 32, 32, 0, 1e-6),
    (1, 1280, 640, 32, 32, 1, 1e-5), (2, 64, 0, 8, 8, 0, 1e-6)])
def test_group_norm(N, C1, C2, H, W, silu, eps):
    g = torch.Generator().manual_seed(C1 + C2 + H)
    x1 = (torch.randn(N, H, W, C1, generator=g) * 2 + 0.5).half().cuda()
    x2 = (torch.randn(N, H, W, C2, generator=g) - 0.3).half().cuda() if C2 else None
    C = C1 + C2
    gam = (1 + 0.1 * torch.randn(C, generator=g)).half().cuda()
    bet = (0.1 * torch.randn(C, generator=g)).half().cuda()
    out = torch.empty(N, H, W, C, dtype=torch.float16, device="cuda")
    nb = L.lib().dlm_group_norm_nhwc_scratch_bytes(N, H * W)
    scratch = torch.empty(nb, dtype=torch.uint8, device="cuda")
    L.call("dlm_group_norm_nhwc", _p(x1), C1, _p(x2), C2, N, H * W, _p(gam), _p(bet), eps, 32, silu,
           _p(out), _p(scratch), nb, _s())
    torch.cuda.synchronize()
    x = torch.cat([x1, x2], dim=-1) if C2 else x1
    ref = F.group_norm(x.float().permute(0, 3, 1, 2), 32, gam.float(), bet.float(), eps)
    if silu:
        ref = F.silu(ref)
    ref = ref.permute(0, 2, 3, 1)
    assert max_rel_err(out, ref) < 2e-3
    # determinism: a second run is bit-identical
    out2 = torch.empty_like(out)
    L.call("dlm_group_norm_nhwc", _p(x1), C1, _p(x2), C2, N, H * W, _p(gam), _p(bet), eps, 32, silu,
           _p(out2), _p(scratch), nb, _s())
    torch.cuda.synchronize()
    assert torch.equal(out, out2)


@pytest.mark.parametrize("rows,C", [(8192, 640), (2048, 1280), (100, 320), (7, 2048)])
def test_layer_norm(rows, C):
    g = torch.Generator().manual_seed(rows + C)
    x = (torch.randn(rows, C, generator=g) * 3 + 1).half().cuda()
    gam = (1 + 0.1 * torch.randn(C, generator=g)).half().cuda()
    bet = (0.1 * torch.randn(C, generator=g)).half().cuda()
    out = torch.empty_like(x)
    L.call("dlm_launch_layer_norm", _p(x), _p(gam), _p(bet), _p(out), rows, C, 1e-5, _s())
    torch.cuda.synchronize()
    ref = F.layer_norm(x.float(), (C,), gam.float(), bet.float(), 1e-5)
    assert max_rel_err(out, ref) < 2e-3
