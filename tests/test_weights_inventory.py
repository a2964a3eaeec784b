"""The shape builders reproduce the reference's production catalog and the fixtures' weight recipes."""

from __future__ import annotations

import json

import pytest

from golden_io import GOLDEN, load
from ctmr_b200 import weights as W

PRODUCTION_UNET = {
    "spatial_dims": 3, "in_channels": 4, "out_channels": 4, "num_channels": [64, 128, 256, 512],
    "attention_levels": [False, False, True, True], "num_head_channels": [0, 0, 32, 32], "num_res_blocks": 2,
    "norm_num_groups": 32, "norm_eps": 1e-6, "include_spacing_input": True, "num_class_embeds": 128,
    "resblock_updown": True, "include_fc": True,
}
PRODUCTION_CONTROLNET = {
    "spatial_dims": 3, "in_channels": 4, "num_channels": [64, 128, 256, 512],
    "attention_levels": [False, False, True, True], "num_head_channels": [0, 0, 32, 32], "num_res_blocks": 2,
    "norm_num_groups": 32, "norm_eps": 1e-6, "conditioning_embedding_in_channels": 8,
    "conditioning_embedding_num_channels": [8, 32, 64], "num_class_embeds": 128, "resblock_updown": True,
    "include_fc": True,
}
PRODUCTION_VAE = {
    "in_channels": 1, "out_channels": 1, "latent_channels": 4, "num_channels": [64, 128, 256],
    "num_res_blocks": [2, 2, 2], "norm_num_groups": 32, "norm_eps": 1e-6,
    "attention_levels": [False, False, False],
}


def _catalog():
    return json.loads((GOLDEN / "production_catalog.json").read_text())


@pytest.mark.parametrize(("net", "builder", "ctor"), [
    ("unet", W.unet_shapes, PRODUCTION_UNET),
    ("controlnet", W.controlnet_shapes, PRODUCTION_CONTROLNET),
    ("vae", W.vae_decoder_shapes, PRODUCTION_VAE),
])
def test_production_inventory(net, builder, ctor):
    expected = {name: tuple(shape) for name, shape in _catalog()[net]}
    assert builder(ctor) == expected


@pytest.mark.parametrize("name", ["mr_brain", "mr"])
def test_fixture_recipe_inventory(name):
    _, meta = load(name)
    shapes = {n: tuple(s) for n, s in meta["recipe"]["shapes"]}
    unet = {n[len("weight.unet."):]: s for n, s in shapes.items() if n.startswith("weight.unet.")}
    vae = {n[len("weight.vae."):]: s for n, s in shapes.items() if n.startswith("weight.vae.")}
    assert W.unet_shapes(meta["constructor"]["unet"]) == unet
    dec = W.vae_decoder_shapes(meta["constructor"]["vae"])
    assert dec == {k: v for k, v in vae.items() if k in dec}
    assert set(dec) <= set(vae)


def test_random_weights_are_reproducible():
    shapes = W.vae_decoder_shapes(PRODUCTION_VAE)
    a = W.random_weights(shapes, seed=3, device="cpu")
    b = W.random_weights(shapes, seed=3, device="cpu")
    assert all((a[k] == b[k]).all() for k in shapes)
    assert (a["decoder.blocks.1.norm1.weight"] == 1).all() and (a["decoder.blocks.9.bias"] == 0).all()
    w = a["decoder.blocks.1.conv1.conv.conv.weight"]
    assert w.abs().max().item() <= (1 + 1e-6) / (256 * 27) ** 0.5
