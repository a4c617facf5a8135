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


STAGE_BAR = 2e-3        # north-star per-layer bar (max|err| / max|ref|)
STORAGE_FACTOR = 1.5    # allowance over the fp16-storage oracle's own error at a stage


def stage_bound(err16: float) -> float:
    """Bound on a stage's max|err|/max|ref| against the fp32 oracle: the north-star 2e-3, or,
    where the fp16-storage oracle (the same fp32 oracle rounding every stored activation to
    fp16, as an fp16-storage implementation such as the reference does) is itself further than
    that from fp32, 1.5x that storage error — an fp16-storage pipeline cannot be closer to fp32
    than fp16 storage allows."""
    return max(STAGE_BAR, STORAGE_FACTOR * err16)
