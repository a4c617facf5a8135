"""Generates tests/golden/bitnet_lm_ref.npz: logits of the REFERENCE'S OWN BitNet::forward
(src/models/bitnet.hpp:376-440, compiled into oracle/_ref/libref_bitnet.so by
oracle/build_oracle.py) at its compiled-in dimensions, for seeded weights (oracle.bitnet.
lm_random_weights, numpy's default_rng: platform-stable) and seeded token ids.  Stored per case:
the tokens, the first and last positions' logits, and the SHA-256 of the whole logits array, so
the oracle's full output can be checked bit for bit without committing it.  Run where the
reference tree is present:  python tests/golden/make_bitnet_lm_vectors.py"""
import hashlib
from pathlib import Path
import sys

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
from oracle.build_oracle import build  # noqa: E402
from oracle import bitnet as B  # noqa: E402

CASES = [("normal", 10, 11, 6), ("ternary", 12, 13, 6)]   # (weight kind, weight seed, token seed, S)


def main():
    build()
    dims = B.ref_dims()
    if dims is None:
        raise SystemExit("reference not built")
    cfg = B.lm_config(vocab=dims[0], d_model=dims[1], n_layers=dims[2], n_heads=dims[3],
                      ffn_dim=dims[4], max_seq=dims[5])
    out = {"dims": np.array(dims, dtype=np.int32)}
    for i, (kind, wseed, tseed, S) in enumerate(CASES):
        w = B.lm_random_weights(cfg, seed=wseed, kind=kind)
        toks = np.random.default_rng(tseed).integers(0, dims[0], size=S).astype(np.int32)
        logits = B.ref_forward(w, toks)
        out[f"kind{i}"] = np.array(kind)
        out[f"wseed{i}"] = np.int64(wseed)
        out[f"tokens{i}"] = toks
        out[f"first{i}"] = logits[0]
        out[f"last{i}"] = logits[-1]
        out[f"sha{i}"] = np.array(hashlib.sha256(logits.tobytes()).hexdigest())
    dst = Path(__file__).resolve().parent / "bitnet_lm_ref.npz"
    np.savez_compressed(dst, **out)
    print("wrote", dst, dst.stat().st_size, "bytes")


if __name__ == "__main__":
    main()
