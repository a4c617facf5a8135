"""Host logic of the runtime LoRA (dollama_b200/lora.py) against the reference's
load_lora_modules rules (src/infer/lora.hpp:300-455) and its test's synthetic kohya files
(src/tests/test_lora_runtime.cu): module grouping, base-key resolution through the dotless
index, scale = strength * alpha / rank, fp32 -> fp16 rounding, skip counters and the errors."""
import numpy as np
import pytest

from dollama_b200.lora import load_lora_modules, pack_modules
from dollama_b200.unet import weight_spec

DEPTHS, MID = (0, 1, 1), 1
Q = "down_blocks.1.attentions.0.transformer_blocks.0.attn1.to_q.weight"
CONV = "down_blocks.1.resnets.0.conv1.weight"


def _kohya(base_key):
    return "lora_unet_" + base_key[: -len(".weight")].replace(".", "_")


@pytest.fixture(scope="module")
def spec():
    return weight_spec(DEPTHS, MID)


def _rng():
    return np.random.default_rng(0)


def test_linear_and_conv_resolution(spec):
    r = _rng()
    out, inn = spec[Q]
    co, ci, kh, kw = spec[CONV]
    lora = {
        _kohya(Q) + ".lora_down.weight": r.standard_normal((4, inn)).astype(np.float16),
        _kohya(Q) + ".lora_up.weight": r.standard_normal((out, 4)).astype(np.float16),
        _kohya(Q) + ".alpha": np.array(2.0, dtype=np.float32),
        _kohya(CONV) + ".lora_down.weight": r.standard_normal((8, ci, kh, kw)).astype(np.float32),
        _kohya(CONV) + ".lora_up.weight": r.standard_normal((co, 8, 1, 1)).astype(np.float16),
    }
    mods, rep = load_lora_modules(spec, lora, strength=0.5)
    assert rep.modules == 2 and rep.te_skipped == rep.other_keys == rep.incomplete == 0
    by = {m.base_key: m for m in mods}
    q = by[Q]
    assert (q.rank, q.in_flat, q.out_dim) == (4, inn, out)
    assert q.scale == pytest.approx(0.5 * 2.0 / 4)
    c = by[CONV]
    assert (c.rank, c.in_flat, c.out_dim) == (8, ci * kh * kw, co)
    assert c.scale == pytest.approx(0.5)  # no alpha: alpha = rank
    # fp32 A is rounded to fp16 (nearest even) and flattened [rank, in * kh * kw]
    src = lora[_kohya(CONV) + ".lora_down.weight"]
    assert c.a_fp16.dtype == np.float16 and c.a_fp16.shape == (8, ci * kh * kw)
    assert np.array_equal(c.a_fp16, src.reshape(8, -1).astype(np.float16))
    assert c.b_fp16.shape == (co, 8)


def test_flat_spelling_and_counters(spec):
    r = _rng()
    out, inn = spec[Q]
    lora = {
        _kohya(Q) + "_lora_down_weight": r.standard_normal((2, inn)).astype(np.float16),
        _kohya(Q) + "_lora_up_weight": r.standard_normal((out, 2)).astype(np.float16),
        _kohya(Q) + "_alpha": np.array(1.0, dtype=np.float16),
        "lora_te1_text_model_encoder_layers_0_mlp_fc1.lora_down.weight": np.zeros((2, 4), np.float16),
        "lora_te2_x.alpha": np.array(1.0, np.float32),
        "lora_te_x.alpha": np.array(1.0, np.float32),
        "something_else": np.zeros(1, np.float16),
        "lora_unet_conv_in.lora_down.weight": np.zeros((2, 36), np.float16),  # no up: incomplete
        "lora_unet_conv_in.weird_suffix": np.zeros(1, np.float16),
    }
    mods, rep = load_lora_modules(spec, lora, strength=1.0)
    assert len(mods) == 1 and mods[0].scale == pytest.approx(0.5)
    assert (rep.te_skipped, rep.other_keys, rep.incomplete, rep.modules) == (3, 2, 1, 1)


def test_errors(spec):
    out, inn = spec[Q]
    bad_name = {"lora_unet_down_blocks_9_nothing.lora_down.weight": np.zeros((2, 4), np.float16),
                "lora_unet_down_blocks_9_nothing.lora_up.weight": np.zeros((4, 2), np.float16)}
    with pytest.raises(KeyError):
        load_lora_modules(spec, bad_name)
    wrong_shape = {_kohya(Q) + ".lora_down.weight": np.zeros((2, inn + 1), np.float16),
                   _kohya(Q) + ".lora_up.weight": np.zeros((out, 2), np.float16)}
    with pytest.raises(ValueError):
        load_lora_modules(spec, wrong_shape)
    wrong_rank = {_kohya(Q) + ".lora_down.weight": np.zeros((2, inn), np.float16),
                  _kohya(Q) + ".lora_up.weight": np.zeros((out, 3), np.float16)}
    with pytest.raises(ValueError):
        load_lora_modules(spec, wrong_rank)
    bad_dtype = {_kohya(Q) + ".lora_down.weight": np.zeros((2, inn), np.int8),
                 _kohya(Q) + ".lora_up.weight": np.zeros((out, 2), np.float16)}
    with pytest.raises(ValueError):
        load_lora_modules(spec, bad_dtype)


def test_pack_modules_layout(spec):
    r = _rng()
    out, inn = spec[Q]
    lora = {_kohya(Q) + ".lora_down.weight": r.standard_normal((4, inn)).astype(np.float16),
            _kohya(Q) + ".lora_up.weight": r.standard_normal((out, 4)).astype(np.float16)}
    mods, _ = load_lora_modules(spec, lora, strength=2.0)
    arr, keep = pack_modules(mods)
    assert arr[0].base_key.decode() == Q
    assert (arr[0].rank, arr[0].in_flat, arr[0].out_dim) == (4, inn, out)
    assert arr[0].scale == pytest.approx(2.0)
    assert arr[0].a_fp16 == keep[0].ctypes.data
