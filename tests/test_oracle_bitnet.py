"""CPU: pin the BitNet oracle (oracle/bitnet_oracle.c) to the reference.

(1) the reference's own known-answer quantizer tests (src/tests/test_bitnet.cpp:107-253),
restated here as vectors; (2) bit-exact agreement with the reference's own integer path compiled
from src/models/bitnet.hpp (oracle/_ref, built when the reference tree is present) on seeded
random inputs, including bitlinear at the LM's shapes (bitnet.hpp:447-471); (3) the committed
golden vectors tests/golden/bitnet_ref_vectors.npz produced by that compiled reference
(tests/golden/make_bitnet_vectors.py), which travel where the reference does not.
"""
from pathlib import Path

import numpy as np
import pytest

from oracle import bitnet as B

GOLD = Path(__file__).resolve().parent / "golden" / "bitnet_ref_vectors.npz"


def test_ternary_kats():
    # test_bitnet.cpp:107-183
    s, q = B.quant_weight([1.0, 2.0, 3.0, 4.0])
    assert abs(s - 2.5) < 1e-6 and q.tolist() == [0, 1, 1, 1]
    s, q = B.quant_weight([-1.0, -2.0, -3.0, -4.0])
    assert abs(s - 2.5) < 1e-6 and q.tolist() == [0, -1, -1, -1]
    s, q = B.quant_weight([0.1, -0.1, 0.0, 0.2])
    assert abs(s - 0.1) < 1e-6 and q.tolist() == [1, -1, 0, 1]
    s, q = B.quant_weight([0.0, 0.0, 0.0])
    assert s == 0.0 and q.tolist() == [0, 0, 0]


def test_int8_kats():
    # test_bitnet.cpp:188-253
    s, q = B.quant_act([1.0, -2.0, 4.0, 0.5])
    assert abs(s - 4.0 / 127.0) < 1e-9 and q.tolist() == [32, -64, 127, 16]
    s, q = B.quant_act([-7.0, 3.5, 7.0])
    assert q[0] == -127 and q[-1] == 127
    s, q = B.quant_act([0.0, 0.0])
    assert s == 0.0 and q.tolist() == [0, 0]


def _ref_or_skip():
    R = B.reference()
    if R is None:
        pytest.skip("reference not compiled here (oracle/_ref absent)")
    return R


@pytest.mark.parametrize("n", [1, 7, 512, 1536, 4099])
def test_quantizers_bit_exact_vs_reference(n):
    R = _ref_or_skip()
    rng = np.random.default_rng(n)
    for scale in (1e-3, 0.02, 1.0, 30.0):
        w = (rng.standard_normal(n) * scale).astype(np.float32)
        a1, q1 = B.quant_weight(w)
        a2, q2 = B.quant_weight(w, lib=R)
        assert a1 == a2 and np.array_equal(q1, q2)
        x = (rng.standard_normal(n) * scale).astype(np.float32)
        s1, p1 = B.quant_act(x)
        s2, p2 = B.quant_act(x, lib=R)
        assert s1 == s2 and np.array_equal(p1, p2)


@pytest.mark.parametrize("out_dim,in_dim", [(512, 512), (1536, 512), (512, 1536), (1792, 512), (5, 3)])
def test_bitlinear_bit_exact_vs_reference(out_dim, in_dim):
    _ref_or_skip()
    rng = np.random.default_rng(out_dim * 7 + in_dim)
    w = rng.standard_normal((out_dim, in_dim)).astype(np.float32) * 0.05
    x = rng.standard_normal(in_dim).astype(np.float32)
    assert np.array_equal(B.bitlinear(w, x), B.ref_bitlinear(w, x))


def test_gemm_path_equals_bitlinear():
    rng = np.random.default_rng(3)
    w = rng.standard_normal((64, 96)).astype(np.float32)
    x = rng.standard_normal((5, 96)).astype(np.float32)
    wq, a = B.quant_weight_rows(w)
    xq, s = B.quant_act_rows(x)
    y, _ = B.ternary_gemm(wq, a, xq, s)
    for m in range(5):
        assert np.array_equal(y[m], B.bitlinear(w, x[m]))


def test_golden_vectors():
    if not GOLD.exists():
        pytest.skip("golden vectors not generated")
    g = np.load(GOLD)
    for i in range(int(g["count"])):
        w, x, y = g[f"w{i}"], g[f"x{i}"], g[f"y{i}"]
        assert np.array_equal(B.bitlinear(w, x), y), i
