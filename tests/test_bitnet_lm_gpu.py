"""BitNet tag LM on the GPU (C ABI) against the C oracle of BitNet::forward (oracle/bitnet_lm.c,
itself pinned bit for bit to the reference's compiled forward) and against the reference's own
golden logits (tests/golden/bitnet_lm_ref.npz).

The LM reproduces the reference's double-precision context arithmetic operation by operation and
BitLinear exactly; the one source of last-bit differences is CUDA's double exp (softmax, SiLU)
against the host C library's.  So logits are compared bit for bit where possible and otherwise
within LOGIT_TOL of max|logit|, and greedy tokens must be identical.
"""
import hashlib
from pathlib import Path

import numpy as np
import pytest

from oracle import bitnet as B

pytestmark = pytest.mark.gpu

LOGIT_TOL = 1e-5
GOLD = Path(__file__).resolve().parent / "golden" / "bitnet_lm_ref.npz"
SMALL = B.lm_config(vocab=300, d_model=128, n_layers=2, n_heads=2, ffn_dim=192, max_seq=24)


def _gpu(cfg, w):
    from dollama_b200.bitnet_lm import BitNetConfig, BitNetLM
    return BitNetLM(BitNetConfig(**cfg), w)


def _cmp(got, ref):
    eq = float(np.mean(got == ref))
    err = float(np.max(np.abs(got - ref)) / max(np.max(np.abs(ref)), 1e-30))
    print(f"logits: {100 * eq:.3f}% bit-identical, max rel err {err:.2e}")
    assert err <= LOGIT_TOL
    return eq


@pytest.mark.parametrize("kind,per_tensor", [("normal", 0), ("ternary", 0), ("ternary", 1)])
def test_forward_matches_oracle(kind, per_tensor):
    cfg = dict(SMALL, per_tensor_scale=per_tensor)
    w = B.lm_random_weights(cfg, seed=3, kind=kind)
    toks = np.random.default_rng(4).integers(0, cfg["vocab"], size=(3, 10)).astype(np.int32)
    lm = _gpu(cfg, w)
    got = lm.forward(toks)
    o = B.OracleLM(cfg, w)
    ref = np.stack([o.forward(t) for t in toks])
    assert _cmp(got, ref) > 0.99
    lm.close()


@pytest.mark.parametrize("case", [0, 1])
def test_forward_matches_reference_golden(case):
    g = np.load(GOLD)
    d = [int(x) for x in g["dims"]]
    cfg = B.lm_config(vocab=d[0], d_model=d[1], n_layers=d[2], n_heads=d[3], ffn_dim=d[4],
                      max_seq=d[5])
    w = B.lm_random_weights(cfg, seed=int(g[f"wseed{case}"]), kind=str(g[f"kind{case}"]))
    lm = _gpu(cfg, w)
    logits = lm.forward(g[f"tokens{case}"][None])[0]
    _cmp(logits[0], g[f"first{case}"])
    _cmp(logits[-1], g[f"last{case}"])
    same = hashlib.sha256(logits.tobytes()).hexdigest() == str(g[f"sha{case}"])
    print("whole logits bit-identical to the reference:", same)
    lm.close()


def test_generate_matches_oracle_with_eos_stops():
    # a long <eos> (id 2) embedding row makes <eos> win at state-dependent steps, so sequences
    # stop at different lengths (0, 6 and 19 of 19 here)
    cfg = B.lm_config(vocab=64, d_model=128, n_layers=2, n_heads=2, ffn_dim=128, max_seq=24)
    w = B.lm_random_weights(cfg, seed=8, kind="normal")
    w["embed"][B.TOK_EOS] *= 30.0
    prompts = np.random.default_rng(9).integers(3, cfg["vocab"], size=(16, 5)).astype(np.int32)
    lm = _gpu(cfg, w)
    got = lm.generate(prompts, max_len=24)
    o = B.OracleLM(cfg, w)
    ref = [o.generate(p, 24) for p in prompts]
    assert got == ref
    assert len({len(r) for r in ref}) > 2      # the stops really differ between sequences
    lm.close()


def test_generate_baseline_dims_matches_oracle():
    """The benchmarked tag LM's dims (vocab 16000, d 512, 8 layers, FFN 1536), 64 prompt + 64 greedy
    tokens, ternary weights; 8 sequences on the GPU, two of them re-derived by the oracle."""
    cfg = B.lm_config()
    w = B.lm_random_weights(cfg, seed=10, kind="ternary")
    prompts = np.random.default_rng(11).integers(0, cfg["vocab"], size=(8, 64)).astype(np.int32)
    lm = _gpu(cfg, w)
    got = lm.generate(prompts, max_len=128)
    o = B.OracleLM(cfg, w)
    for b in (0, 5):
        assert got[b] == o.generate(prompts[b], 128)
    lm.close()


def test_generate_sequence_shards_match_full_batch():
    """The multi-GPU LM split: every rank generates its own shard of the sequences.  At the
    benchmarked dims, each shard of 128, 64 or 32 of 256 sequences (the per-rank batches of 2, 4 and
    8 GPUs) generated alone gives the full batch's tokens for those sequences — the decode tile
    choices, which depend on the batch, change no bit."""
    cfg = B.lm_config()
    w = B.lm_random_weights(cfg, seed=10, kind="ternary")
    prompts = np.random.default_rng(13).integers(3, cfg["vocab"], size=(256, 64)).astype(np.int32)
    lm = _gpu(cfg, w)
    full = lm.generate(prompts, max_len=128)
    for b in (128, 64, 32):
        for r0 in (0, 256 - b):
            assert lm.generate(prompts[r0:r0 + b], max_len=128) == full[r0:r0 + b], (b, r0)
    lm.close()


@pytest.mark.parametrize("P,max_len", [(5, 24), (6, 23), (7, 21), (9, 10), (21, 22)])
def test_generate_odd_and_even_cache_lengths(P, max_len):
    """Cache lengths (max_len) of both parities and prefill-only / one-step decodes: the
    attention kernels stage K / V rows in shared memory at offsets that depend on the cache
    length, and must stay 16-byte aligned for every length."""
    cfg = B.lm_config(vocab=64, d_model=128, n_layers=2, n_heads=2, ffn_dim=128, max_seq=24)
    w = B.lm_random_weights(cfg, seed=12, kind="normal")
    prompts = np.random.default_rng(P * 100 + max_len).integers(3, cfg["vocab"], size=(4, P)).astype(np.int32)
    lm = _gpu(cfg, w)
    got = lm.generate(prompts, max_len=max_len)
    o = B.OracleLM(cfg, w)
    assert got == [o.generate(p, max_len) for p in prompts]
    lm.close()


def test_invalid_tokens_rejected():
    from dollama_b200 import _lib as L
    w = B.lm_random_weights(SMALL, seed=1)
    lm = _gpu(SMALL, w)
    with pytest.raises(L.DlmError):
        lm.forward(np.array([[0, SMALL["vocab"]]], dtype=np.int32))
    with pytest.raises(L.DlmError):
        lm.generate(np.zeros((1, 4), dtype=np.int32), max_len=SMALL["max_seq"] + 1)
    lm.close()


def test_text_prompt_end_to_end_matches_oracle():
    """Tokenizer -> LM -> tags (generate_from_text / generate_with_identity) at the reference's
    vocabulary size 4999, against the oracle's greedy decode of the same prompt ids."""
    from dollama_b200.tokenizer import Tokenizer, identity_prompt, text_prompt
    from tests.golden.make_tokenizer_vectors import synthetic_vocab
    tok = Tokenizer(synthetic_vocab())
    cfg = B.lm_config(vocab=4999, d_model=128, n_layers=2, n_heads=2, ffn_dim=192, max_seq=32)
    w = B.lm_random_weights(cfg, seed=12, kind="ternary")
    lm = _gpu(cfg, w)
    o = B.OracleLM(cfg, w)
    text = "1girl with long hair and a white shirt under a blue sky"
    got = lm.generate_from_text(tok, text, max_len=32)
    assert got == tok.decode(o.generate(np.asarray(text_prompt(tok, text), np.int32), 32))
    got2 = lm.generate_with_identity(tok, ["solo", "red eyes"], "open mouth, smile", max_len=32)
    p2 = identity_prompt(tok, ["solo", "red eyes"], "open mouth, smile")
    assert got2 == tok.decode(o.generate(np.asarray(p2, np.int32), 32))
    lm.close()
