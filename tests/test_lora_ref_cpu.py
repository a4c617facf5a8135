"""The kohya LoRA loader (dollama_b200/lora.py) against the reference's OWN load_lora_modules
(src/infer/lora.hpp, with its safetensors reader, compiled from the headers into
oracle/_ref/libref_lora.so): on safetensors files written here, both must give the same modules
in the same order — base key, rank, in_flat, out_dim, the float32 scale, the fp16 bits of A and
B — the same report counters, and reject the same malformed LoRAs."""
import ctypes

import numpy as np
import pytest

from dollama_b200.lora import load_lora_modules
from oracle.build_oracle import build

safetensors_np = pytest.importorskip("safetensors.numpy")

BASE = {  # a small stand-in for the UNet's key set: real names, small shapes
    "conv_in.weight": (8, 4, 3, 3),
    "down_blocks.1.resnets.0.conv1.weight": (16, 8, 3, 3),
    "down_blocks.1.resnets.0.conv_shortcut.weight": (16, 8, 1, 1),
    "down_blocks.1.attentions.0.transformer_blocks.0.attn1.to_q.weight": (16, 16),
    "down_blocks.1.attentions.0.transformer_blocks.0.attn1.to_out.0.weight": (16, 16),
    "down_blocks.1.attentions.0.transformer_blocks.0.ff.net.0.proj.weight": (64, 16),
    "mid_block.attentions.0.transformer_blocks.0.attn2.to_k.weight": (16, 32),
    "time_embedding.linear_1.weight": (32, 8),
    "down_blocks.1.attentions.0.transformer_blocks.0.norm1.weight": (16,),
}


def _k(name):
    return "lora_unet_" + name[: -len(".weight")].replace(".", "_")


@pytest.fixture(scope="module")
def ref():
    path = build().get("ref_lora")
    if path is None:
        pytest.skip("reference tree absent: libref_lora.so not built")
    lib = ctypes.CDLL(path)
    lib.ref_lora_load.restype = ctypes.c_void_p
    lib.ref_lora_load.argtypes = [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_float]
    lib.ref_lora_error.restype = ctypes.c_char_p
    lib.ref_lora_free.argtypes = [ctypes.c_void_p]
    lib.ref_lora_count.argtypes = [ctypes.c_void_p]
    lib.ref_lora_report.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_longlong)]
    lib.ref_lora_module.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_char_p, ctypes.c_int,
                                    ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_float),
                                    ctypes.c_void_p, ctypes.c_void_p]
    return lib


@pytest.fixture(scope="module")
def base_file(tmp_path_factory):
    p = tmp_path_factory.mktemp("lora") / "base.safetensors"
    safetensors_np.save_file({k: np.zeros(s, np.float16) for k, s in BASE.items()}, str(p))
    return p


def _lora_dict():
    r = np.random.default_rng(5)
    q = "down_blocks.1.attentions.0.transformer_blocks.0.attn1.to_q.weight"
    o = "down_blocks.1.attentions.0.transformer_blocks.0.attn1.to_out.0.weight"
    ff = "down_blocks.1.attentions.0.transformer_blocks.0.ff.net.0.proj.weight"
    kv = "mid_block.attentions.0.transformer_blocks.0.attn2.to_k.weight"
    c1 = "down_blocks.1.resnets.0.conv1.weight"
    sc = "down_blocks.1.resnets.0.conv_shortcut.weight"
    d = {
        _k(q) + ".lora_down.weight": r.standard_normal((4, 16)).astype(np.float16),
        _k(q) + ".lora_up.weight": r.standard_normal((16, 4)).astype(np.float16),
        _k(q) + ".alpha": np.array(2.0, np.float32),
        # flat spelling, fp32 tensors (rounded to fp16 by both), fp16 alpha
        _k(o) + "_lora_down_weight": r.standard_normal((2, 16)).astype(np.float32),
        _k(o) + "_lora_up_weight": r.standard_normal((16, 2)).astype(np.float32),
        _k(o) + "_alpha": np.array(0.7, np.float16),
        _k(ff) + ".lora_down.weight": r.standard_normal((8, 16)).astype(np.float16),
        _k(ff) + ".lora_up.weight": r.standard_normal((64, 8)).astype(np.float16),
        _k(kv) + ".lora_down.weight": r.standard_normal((3, 32)).astype(np.float16),
        _k(kv) + ".lora_up.weight": r.standard_normal((16, 3)).astype(np.float16),
        _k(kv) + ".alpha": np.array(5.0, np.float32),
        # 3x3 conv LoRA: A [rank, in, 3, 3], B [out, rank, 1, 1]; 1x1 shortcut
        _k(c1) + ".lora_down.weight": r.standard_normal((4, 8, 3, 3)).astype(np.float16),
        _k(c1) + ".lora_up.weight": r.standard_normal((16, 4, 1, 1)).astype(np.float16),
        _k(sc) + ".lora_down.weight": r.standard_normal((2, 8, 1, 1)).astype(np.float16),
        _k(sc) + ".lora_up.weight": r.standard_normal((16, 2, 1, 1)).astype(np.float16),
        # skipped / counted
        "lora_te1_text_model_encoder_layers_0_mlp_fc1.lora_down.weight": np.zeros((2, 4), np.float16),
        "lora_te2_text_model_x.alpha": np.array(1.0, np.float32),
        "not_a_lora_key": np.zeros(3, np.float16),
        "lora_unet_conv_in.lora_down.weight": np.zeros((2, 36), np.float16),  # no up: incomplete
        "lora_unet_conv_in.strange_suffix": np.zeros(1, np.float16),
    }
    return d


def _ref_modules(lib, base, lora, strength):
    h = lib.ref_lora_load(str(base).encode(), str(lora).encode(), strength)
    if not h:
        raise RuntimeError(lib.ref_lora_error().decode())
    rep = (ctypes.c_longlong * 4)()
    lib.ref_lora_report(h, rep)
    mods = []
    for i in range(lib.ref_lora_count(h)):
        key = ctypes.create_string_buffer(512)
        dims = (ctypes.c_int * 3)()
        scale = ctypes.c_float()
        lib.ref_lora_module(h, i, key, 512, dims, ctypes.byref(scale), None, None)
        a = np.zeros(dims[0] * dims[1], np.uint16)
        b = np.zeros(dims[2] * dims[0], np.uint16)
        lib.ref_lora_module(h, i, key, 512, dims, ctypes.byref(scale), a.ctypes.data, b.ctypes.data)
        mods.append((key.value.decode(), tuple(dims), scale.value, a, b))
    lib.ref_lora_free(h)
    return mods, tuple(rep)


@pytest.mark.parametrize("strength", [1.0, 0.65])
def test_loader_is_the_reference(ref, base_file, tmp_path, strength):
    d = _lora_dict()
    lp = tmp_path / "lora.safetensors"
    safetensors_np.save_file(d, str(lp))
    rmods, rrep = _ref_modules(ref, base_file, lp, strength)
    mods, rep = load_lora_modules(BASE, d, strength)
    assert (rep.te_skipped, rep.other_keys, rep.incomplete, rep.modules) == rrep
    assert len(mods) == len(rmods) == 6
    for m, (key, dims, scale, a, b) in zip(mods, rmods):
        assert m.base_key == key
        assert (m.rank, m.in_flat, m.out_dim) == dims
        assert np.float32(m.scale) == np.float32(scale)
        assert np.array_equal(m.a_fp16.view(np.uint16).ravel(), a)
        assert np.array_equal(m.b_fp16.view(np.uint16).ravel(), b)


def test_rejections_match_the_reference(ref, base_file, tmp_path):
    q = "down_blocks.1.attentions.0.transformer_blocks.0.attn1.to_q.weight"
    cases = {
        "unresolved": {"lora_unet_no_such_module.lora_down.weight": np.zeros((2, 4), np.float16),
                       "lora_unet_no_such_module.lora_up.weight": np.zeros((4, 2), np.float16)},
        "linear_shape": {_k(q) + ".lora_down.weight": np.zeros((2, 15), np.float16),
                         _k(q) + ".lora_up.weight": np.zeros((16, 2), np.float16)},
        "rank": {_k(q) + ".lora_down.weight": np.zeros((2, 16), np.float16),
                 _k(q) + ".lora_up.weight": np.zeros((16, 3), np.float16)},
    }
    for name, d in cases.items():
        lp = tmp_path / f"{name}.safetensors"
        safetensors_np.save_file(d, str(lp))
        with pytest.raises(RuntimeError):
            _ref_modules(ref, base_file, lp, 1.0)
        with pytest.raises((KeyError, ValueError)):
            load_lora_modules(BASE, d, 1.0)
