"""Error metrics used by the parity tests.

`max_rel_err` is the per-layer metric of the north-star bar: max |got - ref| / max |ref|
(the bar is <= 2e-3 per layer).  `allclose_k` is the reference kernel tests' tolerance that
grows with the accumulation length K (src/tests/test_conv2d.cu:78-85,
src/tests/test_gemm.cu:129-130).
"""
import torch


def max_rel_err(got: torch.Tensor, ref: torch.Tensor) -> float:
    got = got.detach().float().cpu()
    ref = ref.detach().float().cpu()
    denom = ref.abs().max().item()
    if denom == 0.0:
        return (got - ref).abs().max().item()
    return (got - ref).abs().max().item() / denom


def conv_tol(K: int):
    """atol, rtol of the reference conv/attention tests for accumulation length K."""
    return 3e-3 + 2e-5 * K, 5e-3 + 1e-5 * K


def allclose_k(got: torch.Tensor, ref: torch.Tensor, K: int) -> bool:
    atol, rtol = conv_tol(K)
    got = got.detach().float().cpu()
    ref = ref.detach().float().cpu()
    return bool(((got - ref).abs() <= atol + rtol * ref.abs()).all())
