"""CPU checks of the VAE decoder's host side: the weight set the C library expects equals the
oracle's diffusers state-dict layout, and the oracle's FLOP count matches the reference's
10.47 TFLOP per 1024^2 image."""
from dollama_b200 import vae
from oracle.sdxl_vae import vae_flops, weight_shapes


def test_weight_spec_matches_oracle():
    spec = vae.weight_spec()
    assert len(spec) == 140
    assert spec == {k: tuple(v) for k, v in weight_shapes().items()}


def test_flops_1024():
    assert abs(vae_flops(1, 128, 128) / 1e12 - 10.47) < 0.01
