"""CPU checks of the BitNet LM oracle (oracle/bitnet_lm.c): pinned bit for bit to the reference's
own BitNet::forward (golden logits from the compiled reference, tests/golden/bitnet_lm_ref.npz,
and a live comparison when oracle/_ref is built), and its KV-cached greedy decode equal to the
reference rule of recomputing the whole prefix (src/infer/bitnet.hpp:282-318)."""
import hashlib
from pathlib import Path

import numpy as np
import pytest

from oracle import bitnet as B

GOLD = Path(__file__).resolve().parent / "golden" / "bitnet_lm_ref.npz"


def _ref_cfg(dims):
    return B.lm_config(vocab=int(dims[0]), d_model=int(dims[1]), n_layers=int(dims[2]),
                       n_heads=int(dims[3]), ffn_dim=int(dims[4]), max_seq=int(dims[5]))


@pytest.mark.parametrize("case", [0, 1])
def test_oracle_matches_reference_golden(case):
    g = np.load(GOLD)
    cfg = _ref_cfg(g["dims"])
    w = B.lm_random_weights(cfg, seed=int(g[f"wseed{case}"]), kind=str(g[f"kind{case}"]))
    o = B.OracleLM(cfg, w)
    logits = o.forward(g[f"tokens{case}"])
    assert np.array_equal(logits[0], g[f"first{case}"])
    assert np.array_equal(logits[-1], g[f"last{case}"])
    assert hashlib.sha256(logits.tobytes()).hexdigest() == str(g[f"sha{case}"])


def test_oracle_matches_compiled_reference_live():
    dims = B.ref_dims()
    if dims is None:
        pytest.skip("reference not built here")
    cfg = _ref_cfg(dims)
    w = B.lm_random_weights(cfg, seed=31, kind="normal")
    toks = np.array([1, 4998, 3, 17, 2], dtype=np.int32)  # specials and the last id
    assert np.array_equal(B.OracleLM(cfg, w).forward(toks), B.ref_forward(w, toks))


SMALL = B.lm_config(vocab=300, d_model=128, n_layers=2, n_heads=2, ffn_dim=192, max_seq=24)


@pytest.mark.parametrize("kind,per_tensor", [("normal", 0), ("ternary", 0), ("ternary", 1)])
def test_kv_cached_generate_equals_prefix_recompute(kind, per_tensor):
    cfg = dict(SMALL, per_tensor_scale=per_tensor)
    w = B.lm_random_weights(cfg, seed=5, kind=kind)
    o = B.OracleLM(cfg, w)
    prompt = np.random.default_rng(6).integers(0, cfg["vocab"], size=7)
    gen = o.generate(prompt, max_len=cfg["max_seq"])
    seq = list(prompt)
    for t in gen + [None]:
        if len(seq) >= cfg["max_seq"]:
            assert t is None
            break
        last = o.forward(np.array(seq))[-1]
        best = int(np.argmax(last))          # first maximum = smallest id among ties
        if t is None:
            assert best == B.TOK_EOS
            break
        assert best == t
        seq.append(t)


def test_forward_rejects_bad_input():
    o = B.OracleLM(SMALL, B.lm_random_weights(SMALL, seed=1))
    with pytest.raises(ValueError):
        o.forward(np.array([0, SMALL["vocab"]]))
    with pytest.raises(ValueError):
        o.forward(np.zeros(SMALL["max_seq"] + 1, dtype=np.int32))
