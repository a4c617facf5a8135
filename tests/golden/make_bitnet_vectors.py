"""Generates tests/golden/bitnet_ref_vectors.npz: bitlinear outputs of the REFERENCE'S OWN code
(src/models/bitnet.hpp, compiled into oracle/_ref/libref_bitnet.so by oracle/build_oracle.py) on
seeded inputs at the tag LM's shapes (and small edge cases).  Run where the reference tree is
present:  python tests/golden/make_bitnet_vectors.py"""
from pathlib import Path
import sys

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
from oracle.build_oracle import build  # noqa: E402
from oracle import bitnet as B  # noqa: E402


def main():
    build()
    if B.reference() is None:
        raise SystemExit("reference not built")
    rng = np.random.default_rng(20261201)
    cases = [(8, 512), (16, 1536), (32, 512), (4, 3), (3, 1)]
    out = {"count": np.int64(len(cases) + 2)}
    for i, (o, n) in enumerate(cases):
        w = (rng.standard_normal((o, n)) * 0.05).astype(np.float32)
        x = rng.standard_normal(n).astype(np.float32)
        out[f"w{i}"], out[f"x{i}"], out[f"y{i}"] = w, x, B.ref_bitlinear(w, x)
    i = len(cases)
    w = np.zeros((4, 64), np.float32)          # all-zero weights (alpha = 0)
    x = rng.standard_normal(64).astype(np.float32)
    out[f"w{i}"], out[f"x{i}"], out[f"y{i}"] = w, x, B.ref_bitlinear(w, x)
    i += 1
    w = (rng.standard_normal((4, 64)) * 0.05).astype(np.float32)
    x = np.zeros(64, np.float32)               # all-zero activations (scale = 0)
    out[f"w{i}"], out[f"x{i}"], out[f"y{i}"] = w, x, B.ref_bitlinear(w, x)
    dst = Path(__file__).resolve().parent / "bitnet_ref_vectors.npz"
    np.savez_compressed(dst, **out)
    print("wrote", dst, dst.stat().st_size, "bytes")


if __name__ == "__main__":
    main()
