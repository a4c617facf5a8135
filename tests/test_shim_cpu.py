"""The reference-side C++ binding (include/dollama_b200_shim.hpp) compiles against the reference's
own headers and links the library, with no GPU: the shim's test driver is built with g++ against
src/io/safetensors.hpp and src/infer/lora.hpp of the reference tree and libdollama_b200.so, then
started without arguments (it loads the library and prints its usage)."""
import subprocess
import tempfile
from pathlib import Path

import pytest

from tests.shim import build_shim_driver as B


@pytest.mark.skipif(B.reference_root() is None, reason="reference tree not present")
def test_shim_compiles_against_reference_headers_and_links():
    with tempfile.TemporaryDirectory() as d:
        exe = B.build(Path(d) / "shim_driver")
        assert exe is not None and exe.exists()
        r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
        assert r.returncode == 2 and "usage" in r.stderr
        nm = subprocess.run(["nm", "-u", str(exe)], capture_output=True, text=True).stdout
        for sym in ("dlm_unet_create", "dlm_unet_forward", "dlm_vae_decode", "dlm_group_norm_nchw",
                    "dlm_conv2d_direct_nchw", "dlm_conv2d_uses_gemm_bias_path", "dlm_conv2d_nhwc",
                    "dlm_launch_attention", "dlm_unet_apply_loras", "dlm_unet_clear_loras"):
            assert sym in nm, sym
