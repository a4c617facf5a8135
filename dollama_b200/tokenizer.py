"""Tag tokenizer of the BitNet tag LM (host logic; no device work).

Restates the reference's vocab.json-driven whole-tag tokenizer (src/io/tokenizer.hpp) and the
LM prompt framing built on it (src/infer/bitnet.hpp:320-385):

  * vocab.json: {"version", "separator", "specials": ["<pad>", "<bos>", "<eos>", "<sep>", "<unk>"],
    "tags": [{"id": 5 + i, "tag": ..., "category": ..., "freq": ...}, ...]}; the specials must be
    exactly those five (ids 0..4), tag ids contiguous from 5, and the total vocabulary 4999
    (tokenizer.hpp:487-527; `vocab_size` overrides the total for other vocabularies);
  * normalisation: an underscore between two ASCII alphanumerics becomes a space, every other
    underscore (emoticons such as ^_^) stays (tokenizer.hpp:258-279);
  * encode(tags, max_len=64): <bos>, one id per tag (<unk> = 4 when unknown), <eos>; truncated so
    the whole sequence, framing included, is at most max_len, the last slot then being <eos>;
    max_len <= 0 gives [] (tokenizer.hpp:103-136);
  * encode_text(text, max_len=64): the normalised text split into alphanumeric words; from each
    word the longest run of words (up to the longest tag's word count) whose span of the text
    (separators included) is a tag is emitted, unknown words are skipped; same framing
    (tokenizer.hpp:144-216, 580-602);
  * decode(ids): <bos> / <eos> / <pad> / <sep> dropped, <unk> kept as "<unk>", ids outside the
    vocabulary decode as "<unk>" (tokenizer.hpp:78-92, 223-250).
"""
from __future__ import annotations

import json
from pathlib import Path

TOK_PAD, TOK_BOS, TOK_EOS, TOK_SEP, TOK_UNK = 0, 1, 2, 3, 4
SPECIALS = ("<pad>", "<bos>", "<eos>", "<sep>", "<unk>")
DEFAULT_MAX_SEQ_LEN = 64
REFERENCE_VOCAB_SIZE = 4999


def _alnum(c: str) -> bool:
    # std::isalnum in the "C" locale: ASCII letters and digits only
    return ("0" <= c <= "9") or ("a" <= c <= "z") or ("A" <= c <= "Z")


def normalize(s: str) -> str:
    out = []
    n = len(s)
    for i, c in enumerate(s):
        if c == "_" and i > 0 and i + 1 < n and _alnum(s[i - 1]) and _alnum(s[i + 1]):
            out.append(" ")
        else:
            out.append(c)
    return "".join(out)


def _words(s: str):
    """[begin, end) spans of the maximal runs of ASCII alphanumerics."""
    spans, i, n = [], 0, len(s)
    while i < n:
        while i < n and not _alnum(s[i]):
            i += 1
        if i >= n:
            break
        b = i
        while i < n and _alnum(s[i]):
            i += 1
        spans.append((b, i))
    return spans


class Tokenizer:
    """Whole-tag tokenizer over a vocab.json (path, JSON text or the parsed dict)."""

    def __init__(self, vocab, vocab_size: int = REFERENCE_VOCAB_SIZE):
        if isinstance(vocab, dict):
            d = vocab
        else:
            text = str(vocab)
            if not text.lstrip().startswith("{"):
                text = Path(text).read_text(encoding="utf-8")
            d = json.loads(text)
        specials = list(d.get("specials", []))
        tags = d.get("tags", [])
        if len(specials) != 5:
            raise ValueError(f"tokenizer: specials must be 5 entries, got {len(specials)}")
        for k, (got, want) in enumerate(zip(specials, SPECIALS)):
            if got != want:
                raise ValueError(f"tokenizer: specials[{k}] = '{got}' expected '{want}'")
        for k, t in enumerate(tags):
            if "id" not in t or "tag" not in t:
                raise ValueError("tokenizer: tag object missing id/tag")
            if int(t["id"]) != 5 + k:
                raise ValueError(f"tokenizer: tags[{k}].id = {t['id']} expected {5 + k} "
                                 "(id must be 5+i contiguous)")
        if len(specials) + len(tags) != vocab_size:
            raise ValueError(f"tokenizer: total vocab must be {vocab_size}, got "
                             f"{len(specials) + len(tags)}")
        self.version = int(d.get("version", 0))
        self.separator = d.get("separator", "")
        self._specials = specials
        self._tags = [str(t["tag"]) for t in tags]
        self._index = {}
        self._max_words = 1
        for k, t in enumerate(self._tags):
            norm = normalize(t)
            self._index[norm] = 5 + k
            self._max_words = max(self._max_words, len(_words(norm)))

    def tag_count(self) -> int:
        return len(self._tags)

    def vocab_size(self) -> int:
        return len(self._specials) + len(self._tags)

    def id_to_token(self, i: int) -> str:
        if 0 <= i < len(self._specials):
            return self._specials[i]
        if 0 <= i - len(self._specials) < len(self._tags) and i >= 0:
            return self._tags[i - len(self._specials)]
        return self._specials[TOK_UNK]

    def tag_to_id(self, tag: str) -> int:
        return self._index.get(normalize(tag), TOK_UNK)

    @staticmethod
    def _frame(body, max_len):
        out = [TOK_BOS]
        for t in body:
            if len(out) >= max_len - 1:
                break
            out.append(t)
        if len(out) < max_len:
            out.append(TOK_EOS)
        else:
            out[-1] = TOK_EOS
        return out

    def encode(self, tags, max_len: int = DEFAULT_MAX_SEQ_LEN):
        if max_len <= 0:
            return []
        return self._frame((self.tag_to_id(t) for t in tags), max_len)

    def _text_ids(self, text: str):
        norm = normalize(text)
        words = _words(norm)
        wi = 0
        while wi < len(words):
            hit = None
            for j in range(min(self._max_words, len(words) - wi), 0, -1):
                cand = norm[words[wi][0]:words[wi + j - 1][1]]
                k = self._index.get(cand)
                if k is not None:
                    hit = (k, j)
                    break
            if hit is None:
                wi += 1
            else:
                yield hit[0]
                wi += hit[1]

    def encode_text(self, text: str, max_len: int = DEFAULT_MAX_SEQ_LEN):
        if max_len <= 0:
            return []
        return self._frame(self._text_ids(text), max_len)

    def decode(self, ids):
        out = []
        for i in ids:
            i = int(i)
            if i in (TOK_BOS, TOK_EOS, TOK_PAD, TOK_SEP):
                continue
            out.append(self._specials[TOK_UNK] if i == TOK_UNK else self.id_to_token(i))
        return out

    normalize = staticmethod(normalize)


def text_prompt(tok: Tokenizer, text: str, max_seq: int = DEFAULT_MAX_SEQ_LEN):
    """[<bos>] + encode_text(text)'s tags + [<sep>] (the reference's generate_from_text framing,
    src/infer/bitnet.hpp:321-336)."""
    return [TOK_BOS] + tok.encode_text(text, max_seq)[1:-1] + [TOK_SEP]


def identity_prompt(tok: Tokenizer, identity_tags, scene_text: str,
                    max_seq: int = DEFAULT_MAX_SEQ_LEN):
    """<bos> identity ids <sep> scene tags <sep> (build_identity_prompt, bitnet.hpp:352-376)."""
    return ([TOK_BOS] + [tok.tag_to_id(t) for t in identity_tags] + [TOK_SEP]
            + tok.encode_text(scene_text, max_seq)[1:-1] + [TOK_SEP])
