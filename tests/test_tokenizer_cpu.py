"""The tag tokenizer (dollama_b200/tokenizer.py) against the reference's own Tokenizer
(src/io/tokenizer.hpp) through golden vectors recorded from it on a synthetic vocabulary
(tests/golden/make_tokenizer_vectors.py): encode with every truncation edge (max_len 0, 1, 2, 3,
5, 64, 1024), encode_text's greedy longest match, decode of specials / out-of-range ids,
normalisation, tag lookup, and the vocabulary checks with the reference's messages; plus the LM
prompt framings of src/infer/bitnet.hpp:321-376 and the reference test's own properties
(src/tests/test_tokenizer.cpp: round trip, multi-word tags kept whole, connectives skipped)."""
import json
from pathlib import Path

import pytest

from dollama_b200.tokenizer import (TOK_BOS, TOK_EOS, TOK_SEP, TOK_UNK, Tokenizer, identity_prompt,
                                    normalize, text_prompt)
from tests.golden.make_tokenizer_vectors import broken_vocabs, synthetic_vocab

GOLD = json.loads((Path(__file__).resolve().parent / "golden" / "tokenizer_vectors.json")
                  .read_text(encoding="utf-8"))


@pytest.fixture(scope="module")
def tok():
    return Tokenizer(synthetic_vocab())


def test_vocab_size(tok):
    assert tok.vocab_size() == GOLD["vocab_size"] == 4999
    assert tok.tag_count() == 4994


def test_encode_matches_reference(tok):
    for case in GOLD["encode"]:
        assert tok.encode(case["tags"], case["max_len"]) == case["ids"], case


def test_encode_text_matches_reference(tok):
    for case in GOLD["encode_text"]:
        assert tok.encode_text(case["text"], case["max_len"]) == case["ids"], case


def test_decode_matches_reference(tok):
    for case in GOLD["decode"]:
        assert tok.decode(case["ids"]) == case["tokens"], case


def test_normalize_and_lookup_match_reference(tok):
    for case in GOLD["normalize"]:
        assert normalize(case["in"]) == case["out"], case
    for case in GOLD["tag_to_id"]:
        assert tok.tag_to_id(case["tag"]) == case["id"], case


@pytest.mark.parametrize("name", sorted(broken_vocabs()))
def test_rejects_like_reference(name):
    msg = GOLD["rejects"][name]
    assert msg is not None
    with pytest.raises(ValueError) as e:
        Tokenizer(broken_vocabs()[name])
    assert str(e.value) == msg


def test_loads_from_path_and_text(tmp_path):
    v = synthetic_vocab()
    p = tmp_path / "vocab.json"
    p.write_text(json.dumps(v), encoding="utf-8")
    assert Tokenizer(str(p)).encode(["solo"]) == Tokenizer(json.dumps(v)).encode(["solo"])


def test_reference_test_properties(tok):
    tags = ["1girl", "solo", "long hair", "white shirt"]
    ids = tok.encode(tags)
    assert ids[0] == TOK_BOS and ids[-1] == TOK_EOS and TOK_UNK not in ids
    assert tok.decode(ids) == tags
    dec = tok.decode(tok.encode_text("she has long hair and a white shirt"))
    assert "long hair" in dec and "white shirt" in dec
    assert "long" not in dec and "hair" not in dec and "shirt" not in dec
    assert tok.encode_text("the and with of") == [TOK_BOS, TOK_EOS]


def test_prompt_framing(tok):
    p = text_prompt(tok, "long hair, blue sky")
    assert p == [TOK_BOS, tok.tag_to_id("long hair"), tok.tag_to_id("blue sky"), TOK_SEP]
    q = identity_prompt(tok, ["1girl", "nope"], "white shirt")
    assert q == [TOK_BOS, tok.tag_to_id("1girl"), TOK_UNK, TOK_SEP, tok.tag_to_id("white shirt"), TOK_SEP]
