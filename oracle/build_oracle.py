"""Build recipe of the test oracles (test infrastructure only).

* oracle/_build/liboracle_bitnet.so — the plain-C restatements (bitnet_oracle.c: quantizers and
  BitLinear; bitnet_lm.c: LM forward and greedy decode), always built;
* oracle/_ref/libref_bitnet.so      — the reference's own BitNet integer path, compiled from
  its header where it lies (src/models/bitnet.hpp under the reference tree) through
  ref_bitnet_shim.cpp, built only when the reference tree exists (it does not on GPU boxes,
  which use the prebuilt file).  Outputs go only to oracle/_ref/ (git-ignored);
* oracle/_ref/libref_tokenizer.so   — the reference's tag tokenizer (src/io/tokenizer.hpp, header
  only) through ref_tokenizer_shim.cpp, for the tokenizer golden vectors; same conditions;
* oracle/_ref/libref_scheduler.so   — the reference's Euler scheduler (src/infer/scheduler.hpp,
  header only) through ref_scheduler_shim.cpp; same conditions;
* oracle/_ref/libref_lora.so        — the reference's kohya LoRA loader (src/infer/lora.hpp with
  src/io/safetensors.hpp, header only) through ref_lora_shim.cpp; same conditions;
* oracle/_ref/libref_cpu_<op>.so    — the CPU reference functions of the reference's kernel tests
  (GroupNorm, LayerNorm, GEGLU, activations, attention, timestep embedding, convolution),
  nvcc-compiled with the test file and the reference kernels it links (ref_cpu/*.cu; the
  convolution test's kernels need cuBLAS, so its GPU entry points are left unresolved and the
  library is opened with lazy binding); same conditions.

Usage:  python oracle/build_oracle.py
"""
from __future__ import annotations

import os
import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
BUILD = HERE / "_build"
REF_OUT = HERE / "_ref"
# the reference checkout: $DOLLAMA_REFERENCE, else a `reference` directory beside this repository
REFERENCE = Path(os.environ.get("DOLLAMA_REFERENCE", str(HERE.parent.parent / "reference")))


def _run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")


def _stale(out: Path, *srcs: Path) -> bool:
    return not out.exists() or any(out.stat().st_mtime < s.stat().st_mtime for s in srcs)


def build() -> dict:
    BUILD.mkdir(exist_ok=True)
    out = {}
    lib = BUILD / "liboracle_bitnet.so"
    srcs = [HERE / "bitnet_oracle.c", HERE / "bitnet_lm.c"]
    if _stale(lib, *srcs):
        # no -ffast-math / -mfma: double expressions are evaluated exactly as written, like the
        # reference's own build of the same formulas
        _run(["gcc", "-O2", "-fPIC", "-shared", "-std=c11", "-ffp-contract=off", "-o", str(lib)]
             + [str(x) for x in srcs] + ["-lm"])
    out["oracle_bitnet"] = str(lib)
    hdr = REFERENCE / "src" / "models" / "bitnet.hpp"
    if hdr.exists():
        REF_OUT.mkdir(exist_ok=True)
        ref = REF_OUT / "libref_bitnet.so"
        shim = HERE / "ref_bitnet_shim.cpp"
        if _stale(ref, shim, hdr):
            _run(["g++", "-O2", "-fPIC", "-shared", "-std=c++17", "-ffp-contract=off",
                  "-I", str(REFERENCE / "src"), "-o", str(ref), str(shim)])
        out["ref_bitnet"] = str(ref)
    tok_hdr = REFERENCE / "src" / "io" / "tokenizer.hpp"
    if tok_hdr.exists():
        REF_OUT.mkdir(exist_ok=True)
        ref = REF_OUT / "libref_tokenizer.so"
        shim = HERE / "ref_tokenizer_shim.cpp"
        if _stale(ref, shim, tok_hdr):
            _run(["g++", "-O2", "-fPIC", "-shared", "-std=c++17", "-I", str(REFERENCE / "src"),
                  "-o", str(ref), str(shim)])
        out["ref_tokenizer"] = str(ref)
    sched_hdr = REFERENCE / "src" / "infer" / "scheduler.hpp"
    if sched_hdr.exists():
        REF_OUT.mkdir(exist_ok=True)
        ref = REF_OUT / "libref_scheduler.so"
        shim = HERE / "ref_scheduler_shim.cpp"
        if _stale(ref, shim, sched_hdr):
            _run(["g++", "-O2", "-fPIC", "-shared", "-std=c++17", "-ffp-contract=off",
                  "-I", str(REFERENCE / "src"), "-o", str(ref), str(shim)])
        out["ref_scheduler"] = str(ref)
    lora_hdr = REFERENCE / "src" / "infer" / "lora.hpp"
    if lora_hdr.exists():
        REF_OUT.mkdir(exist_ok=True)
        ref = REF_OUT / "libref_lora.so"
        shim = HERE / "ref_lora_shim.cpp"
        if _stale(ref, shim, lora_hdr):
            _run(["g++", "-O2", "-fPIC", "-shared", "-std=c++17", "-I", str(REFERENCE / "src"),
                  "-o", str(ref), str(shim)])
        out["ref_lora"] = str(ref)
    # the CPU references inside the reference's kernel tests (see ref_cpu/README.txt): each shim
    # includes its test file and links the reference kernels that test calls
    kernels = REFERENCE / "src" / "kernels"
    ops = {"gn": ["groupnorm.cu", "activation.cu"], "ln": ["layernorm.cu"], "geglu": ["geglu.cu"],
           "act": ["activation.cu"], "attn": ["attention.cu"], "timeembed": ["timeembed.cu"],
           "conv": []}  # conv: its test's GPU entry points stay unresolved (opened lazily)
    if kernels.exists():
        REF_OUT.mkdir(exist_ok=True)
        for op, ks in ops.items():
            shim = HERE / "ref_cpu" / f"{op}.cu"
            deps = [kernels / k for k in ks]
            ref = REF_OUT / f"libref_cpu_{op}.so"
            if _stale(ref, shim, *deps):
                _run(["nvcc", "-gencode", "arch=compute_100a,code=sm_100a", "-O2", "-std=c++17",
                      "-DHAVE_CUDA", "-Xcompiler", "-fPIC", "-shared", "-I", str(REFERENCE / "src"),
                      "-o", str(ref), str(shim)] + [str(d) for d in deps])
            out[f"ref_cpu_{op}"] = str(ref)
    return out


if __name__ == "__main__":
    print(build())
