"""Build recipe of tests/shim/_build/shim_driver, the C++ program through which the tests call
the library by the reference's own names (include/dollama_b200_shim.hpp).

It compiles against the reference's headers (src/io/safetensors.hpp, src/infer/lora.hpp), so it is
built where the reference tree is ($DOLLAMA_REFERENCE, else a `reference` directory beside this
repository) and the binary travels with the working tree to the GPU box (git-ignored).

    python tests/shim/build_shim_driver.py [OUT]
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
OUT = HERE / "_build" / "shim_driver"
CUDA = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))


def reference_root() -> Path | None:
    r = Path(os.environ.get("DOLLAMA_REFERENCE", str(ROOT.parent / "reference")))
    return r if (r / "src" / "io" / "safetensors.hpp").exists() else None


def build(out: Path = OUT) -> Path | None:
    ref = reference_root()
    if ref is None:
        return out if out.exists() else None
    src = HERE / "shim_driver.cpp"
    deps = [src, ROOT / "include" / "dollama_b200_shim.hpp", ROOT / "include" / "dollama_b200.h",
            ROOT / "include" / "dollama_b200_runner.hpp"]
    if out.exists() and all(out.stat().st_mtime >= d.stat().st_mtime for d in deps):
        return out
    out.parent.mkdir(parents=True, exist_ok=True)
    libdir = ROOT / "dollama_b200"
    rpath = os.path.relpath(libdir, out.parent)
    cmd = ["g++", "-std=c++17", "-O2", "-Wall", "-Wno-unused-function",
           "-I", str(ROOT / "include"), "-I", str(ref / "src"), "-I", str(CUDA / "include"),
           "-o", str(out), str(src), "-L", str(libdir), "-ldollama_b200",
           "-L", str(CUDA / "lib64"), "-lcudart", f"-Wl,-rpath,$ORIGIN/{rpath}",
           f"-Wl,-rpath,{CUDA / 'lib64'}"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return out


if __name__ == "__main__":
    print(build(Path(sys.argv[1]) if len(sys.argv) > 1 else OUT))
