"""Production MAISI network configurations and freshly initialised parameters for the CPU oracle.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``): used by ``tests/`` and by the
benchmark's CPU legs (``bench.py --impl reference`` and ``cpu_baseline``), which must
time the reference's arithmetic without loading any of the product's code.

* ``UNET``, ``CONTROLNET``, ``VAE``: the constructor keys the oracle reads, as the
  reference sets them for the released networks
  (``maisi_mlx_from_mask.py:20-80``, ``PRODUCTION_*_CONSTRUCTOR``).
* ``parameters(net, seed)``: every parameter name and Torch-layout shape of the
  released checkpoint, read from the reference's production weight catalog
  (``data/maisi_mlx_from_mask_weight_catalog.json``, committed as
  ``tests/golden/production_catalog.json``), filled the way a freshly constructed
  torch module is: convolution / linear weights Kaiming-uniform with a = sqrt(5)
  (bound 1/sqrt(fan_in)), biases U(-1/sqrt(fan_in), 1/sqrt(fan_in)), GroupNorm
  weight 1 and bias 0, embedding tables N(0, 1).
"""

from __future__ import annotations

import json
import math
from pathlib import Path

import torch

CATALOG = Path(__file__).resolve().parents[1] / "tests" / "golden" / "production_catalog.json"

UNET = {
    "in_channels": 4, "out_channels": 4, "num_channels": [64, 128, 256, 512],
    "attention_levels": [False, False, True, True], "num_head_channels": [0, 0, 32, 32], "num_res_blocks": 2,
    "norm_num_groups": 32, "norm_eps": 1e-6, "include_spacing_input": True, "num_class_embeds": 128,
    "resblock_updown": True, "include_fc": True,
}
CONTROLNET = {
    "in_channels": 4, "num_channels": [64, 128, 256, 512], "attention_levels": [False, False, True, True],
    "num_head_channels": [0, 0, 32, 32], "num_res_blocks": 2, "norm_num_groups": 32, "norm_eps": 1e-6,
    "conditioning_embedding_in_channels": 8, "conditioning_embedding_num_channels": [8, 32, 64],
    "num_class_embeds": 128, "resblock_updown": True, "include_fc": True,
}
VAE = {
    "in_channels": 1, "out_channels": 1, "latent_channels": 4, "num_channels": [64, 128, 256],
    "num_res_blocks": [2, 2, 2], "norm_num_groups": 32, "norm_eps": 1e-6,
    "attention_levels": [False, False, False],
}


def catalog(net: str) -> dict[str, tuple[int, ...]]:
    """Parameter names and shapes of one released network ("unet", "controlnet" or "vae")."""
    entries = json.loads(CATALOG.read_text())[net]
    return {str(name): tuple(int(s) for s in shape) for name, shape in entries}


def parameters(net: str, *, seed: int, decoder_only: bool = True) -> dict[str, torch.Tensor]:
    """Fresh-module fp32 CPU parameters of ``net``; for the VAE only the decode path
    (``post_quant_conv`` and ``decoder.*``) unless ``decoder_only`` is False."""
    shapes = catalog(net)
    if net == "vae" and decoder_only:
        shapes = {k: v for k, v in shapes.items() if k.startswith(("post_quant_conv.", "decoder."))}
    gen = torch.Generator().manual_seed(int(seed))
    out: dict[str, torch.Tensor] = {}
    for name, shape in shapes.items():
        stem, kind = name.rsplit(".", 1)
        weight_shape = shapes.get(f"{stem}.weight", shape)
        if name.endswith("embedding.weight"):
            out[name] = torch.randn(shape, generator=gen)
        elif len(weight_shape) == 1:  # a normalisation layer's affine
            out[name] = torch.ones(shape) if kind == "weight" else torch.zeros(shape)
        else:
            bound = 1.0 / math.sqrt(math.prod(weight_shape[1:]))
            out[name] = torch.empty(shape).uniform_(-bound, bound, generator=gen)
    return out
