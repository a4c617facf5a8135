"""Generates tests/golden/tokenizer_vectors.json: what the REFERENCE'S OWN tag tokenizer
(src/io/tokenizer.hpp, compiled into oracle/_ref/libref_tokenizer.so by oracle/build_oracle.py)
returns for encode / encode_text / decode / tag_to_id / normalize on a synthetic vocabulary,
and which malformed vocabularies it rejects.  The vocabulary is not stored: `synthetic_vocab()`
rebuilds it (deterministic), so the tests and this script see the same one.  Run where the
reference tree is present:  python tests/golden/make_tokenizer_vectors.py"""
from __future__ import annotations

import ctypes
import json
import sys
import tempfile
from pathlib import Path

ROOT = Path(__file__).resolve().parents[2]
OUT = Path(__file__).resolve().parent / "tokenizer_vectors.json"

# hand-picked tags: multi-word runs, digits, emoticons kept with their underscores, a tag written
# with underscores (normalised to spaces), a later duplicate of an earlier tag after
# normalisation (the later id wins), non-ASCII text
_NAMED = ["1girl", "solo", "long hair", "looking at viewer", "blush", "smile", "shirt", "white shirt",
          "blonde hair", "short_hair", "hair", "red eyes", "open mouth", "long", "^_^", ">_<", "o_o",
          "2boys", "hat", "holding umbrella", "very long hair", "a b c d e", "café", "x_x_x",
          "red_eyes", "school uniform", "sky", "blue sky", "cloud", "cloudy sky"]


def synthetic_vocab(total: int = 4999) -> dict:
    tags = list(_NAMED)
    i = 0
    while len(tags) < total - 5:
        tags.append(f"t{i}" if i % 3 else f"t{i} s{i % 7}")
        i += 1
    return {"version": 1, "separator": "space",
            "specials": ["<pad>", "<bos>", "<eos>", "<sep>", "<unk>"],
            "tags": [{"id": 5 + k, "tag": t, "category": k % 5, "freq": 1000000 - k}
                     for k, t in enumerate(tags)]}


TAG_LISTS = [
    ["1girl", "solo", "long hair"],
    ["long_hair", "looking_at_viewer", "^_^", ">_<", "nope", "Blush"],
    [],
    ["t5", "t6 s6", "t7", "unknown tag", "café", "x_x_x", "short hair", "red eyes"],
    [f"t{k}" for k in range(100)],
]
MAX_LENS = [64, 0, 1, 2, 3, 5, 1024]
TEXTS = [
    "1girl with long hair, looking at viewer; white shirt and blonde hair",
    "she has long hair",
    "very long hair under a blue sky with cloudy sky",
    "",
    "the and with of",
    "long_hair and school_uniform, o_o ^_^",
    "a b c d e f a b c",
    "t3 s3 t3 t9 s2 t12 s5 café",
    "LONG HAIR long-hair long  hair",
    " ".join(f"t{k}" for k in range(1, 90)),
]
DECODES = [
    [1, 5, 6, 7, 2],
    [0, 1, 2, 3, 4, 9, -1, 5000, 4998, 4999],
    [],
]
NORMALIZE = ["long_hair", "^_^", "a_b_c", "_x_", "x__y", "café_b", "9_9"]
TAG_TO_ID = ["long hair", "long_hair", "Long hair", "red_eyes", "red eyes", "", "^_^", "nope"]


def broken_vocabs() -> dict:
    v = synthetic_vocab()
    out = {}
    b = json.loads(json.dumps(v))
    b["specials"] = b["specials"][:4]
    out["four_specials"] = b
    b = json.loads(json.dumps(v))
    b["specials"][3] = "<SEP>"
    out["wrong_special"] = b
    b = json.loads(json.dumps(v))
    b["tags"][10]["id"] = 99
    out["gap_in_ids"] = b
    b = json.loads(json.dumps(v))
    b["tags"] = b["tags"][:-1]
    out["short_vocab"] = b
    return out


def main():
    sys.path.insert(0, str(ROOT))
    from oracle.build_oracle import build
    lib_path = build().get("ref_tokenizer")
    if lib_path is None:
        raise SystemExit("reference tokenizer not built (reference tree missing)")
    lib = ctypes.CDLL(lib_path)
    lib.ref_tok_create.restype = ctypes.c_void_p
    lib.ref_tok_create.argtypes = [ctypes.c_char_p]
    lib.ref_tok_error.restype = ctypes.c_char_p
    lib.ref_tok_destroy.argtypes = [ctypes.c_void_p]
    lib.ref_tok_vocab_size.argtypes = [ctypes.c_void_p]
    lib.ref_tok_tag_to_id.argtypes = [ctypes.c_void_p, ctypes.c_char_p]
    lib.ref_tok_encode.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_char_p), ctypes.c_int,
                                   ctypes.c_int, ctypes.POINTER(ctypes.c_int), ctypes.c_int]
    lib.ref_tok_encode_text.argtypes = [ctypes.c_void_p, ctypes.c_char_p, ctypes.c_int,
                                        ctypes.POINTER(ctypes.c_int), ctypes.c_int]
    lib.ref_tok_decode.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_int), ctypes.c_int,
                                   ctypes.c_char_p, ctypes.c_int]
    lib.ref_tok_normalize.argtypes = [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_int]

    def load(vocab: dict):
        with tempfile.NamedTemporaryFile("w", suffix=".json", delete=False, encoding="utf-8") as f:
            json.dump(vocab, f, ensure_ascii=False)
            path = f.name
        h = lib.ref_tok_create(path.encode())
        Path(path).unlink()
        return h

    h = load(synthetic_vocab())
    if not h:
        raise SystemExit("reference rejected the synthetic vocabulary: " + lib.ref_tok_error().decode())
    buf = (ctypes.c_int * 4096)()
    res = {"vocab_size": lib.ref_tok_vocab_size(h), "encode": [], "encode_text": [], "decode": [],
           "normalize": [], "tag_to_id": [], "rejects": {}}
    for tags in TAG_LISTS:
        for ml in MAX_LENS:
            arr = (ctypes.c_char_p * max(1, len(tags)))(*[t.encode() for t in tags])
            n = lib.ref_tok_encode(h, arr, len(tags), ml, buf, 4096)
            res["encode"].append({"tags": tags, "max_len": ml, "ids": list(buf[:n])})
    for text in TEXTS:
        for ml in MAX_LENS:
            n = lib.ref_tok_encode_text(h, text.encode(), ml, buf, 4096)
            res["encode_text"].append({"text": text, "max_len": ml, "ids": list(buf[:n])})
    sbuf = ctypes.create_string_buffer(1 << 16)
    for ids in DECODES:
        arr = (ctypes.c_int * max(1, len(ids)))(*ids)
        lib.ref_tok_decode(h, arr, len(ids), sbuf, 1 << 16)
        s = sbuf.value.decode()
        res["decode"].append({"ids": ids, "tokens": s.split("\n") if s else []})
    for s in NORMALIZE:
        lib.ref_tok_normalize(s.encode(), sbuf, 1 << 16)
        res["normalize"].append({"in": s, "out": sbuf.value.decode()})
    for t in TAG_TO_ID:
        res["tag_to_id"].append({"tag": t, "id": lib.ref_tok_tag_to_id(h, t.encode())})
    lib.ref_tok_destroy(h)
    for name, vocab in broken_vocabs().items():
        hb = load(vocab)
        res["rejects"][name] = lib.ref_tok_error().decode() if not hb else None
        if hb:
            lib.ref_tok_destroy(hb)
    OUT.write_text(json.dumps(res, ensure_ascii=False, indent=0), encoding="utf-8")
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes)")


if __name__ == "__main__":
    main()
