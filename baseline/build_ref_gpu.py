"""Build recipe of the GPU comparator: the reference's OWN CUDA SDXL UNet and VAE decoder,
unchanged, recompiled for sm_100a (not product code; nothing in dollama_b200/ loads it).

    python baseline/build_ref_gpu.py

compiles ref_sdxl_gpu.cu (C entry points over the reference API) together with the reference's
sources where they lie — src/infer/unet.cu, src/kernels/vae_decode.cu and the kernels they call,
with cuBLAS, exactly the reference build's diffusion source list — into
baseline/_ref_gpu/libref_sdxl_gpu.so (git-ignored; it travels to the GPU box with the working
tree).  The reference tree is $DOLLAMA_REFERENCE or a `reference` directory beside this
repository; without it (as on a GPU box) the
prebuilt library is used as is and nothing is built.
"""
from __future__ import annotations

import os
import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref_gpu" / "libref_sdxl_gpu.so"
KERNELS = ["vae_decode.cu", "conv2d.cu", "device_arena.cu", "groupnorm.cu", "layernorm.cu",
           "activation.cu", "geglu.cu", "attention.cu", "attention_fast.cu", "gemm.cu",
           "elementwise.cu", "bias_add.cu", "timeembed.cu"]


def reference_root() -> Path | None:
    """$DOLLAMA_REFERENCE, else a `reference` directory beside this repository."""
    r = Path(os.environ.get("DOLLAMA_REFERENCE", str(HERE.parent.parent / "reference")))
    return r if (r / "src" / "infer" / "unet.cu").exists() else None


def build() -> str | None:
    ref = reference_root()
    if ref is None:
        return str(OUT) if OUT.exists() else None
    src = ref / "src"
    srcs = [HERE / "ref_sdxl_gpu.cu", src / "infer" / "unet.cu"] + [src / "kernels" / k for k in KERNELS]
    if OUT.exists() and all(OUT.stat().st_mtime >= s.stat().st_mtime for s in srcs):
        return str(OUT)
    OUT.parent.mkdir(exist_ok=True)
    cmd = ["nvcc", "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17", "-DHAVE_CUDA",
           "-Xcompiler", "-fPIC", "-shared", "-w", "-I", str(src), "-o", str(OUT)] \
        + [str(s) for s in srcs] + ["-lcublas"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return str(OUT)


if __name__ == "__main__":
    print(build())
