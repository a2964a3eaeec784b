"""Native checkpoint ingest (``weights.load_network_file``) on the CPU.

Mirrors the reference loader's contract (``weights.py:102-166``): convolution
weights stored channels-last ``(O, k, k, k, I)`` come back in Torch layout, every
tensor is checked for name, shape, dtype and finiteness, ``model.safetensors``
uses ``<network>.``-prefixed keys, and only the UNet carries ``scale_factor``.
Checkpoints here are written by ``save_network_file`` from random weights.
"""

from __future__ import annotations

import pytest
import torch
from safetensors.torch import save_file

from ctmr_b200 import pipeline as P
from ctmr_b200 import weights as W

SMALL = {"conv.weight": (8, 4, 3, 3, 3), "conv.bias": (8,), "norm.weight": (4,), "proj.weight": (6, 8)}


def _small(seed=0):
    g = torch.Generator().manual_seed(seed)
    return {k: torch.randn(s, generator=g) for k, s in SMALL.items()}


def test_vae_round_trip_gives_torch_layout_views(tmp_path):
    shapes = W.vae_decoder_shapes(P.PRODUCTION_VAE)
    w = W.random_weights(shapes, seed=5, device="cpu")
    W.save_network_file(tmp_path / "vae.safetensors", "vae", w)
    got, scale = W.load_network_file(tmp_path / "vae.safetensors", "vae", shapes)
    assert scale is None and set(got) == set(w)
    for k, t in w.items():
        assert got[k].shape == t.shape and torch.equal(got[k], t), k
        if t.dim() == 5 and t.shape[1] > 1 and t.shape[2] > 1:
            # a view of the channels-last storage, not a transposed copy
            assert got[k].is_contiguous(memory_format=torch.channels_last_3d) and not got[k].is_contiguous()


def test_stored_layout_is_channels_last(tmp_path):
    w = _small()
    W.save_network_file(tmp_path / "net.safetensors", "vae", w)
    from safetensors import safe_open

    with safe_open(str(tmp_path / "net.safetensors"), framework="pt") as f:
        stored = f.get_tensor("conv.weight")
    assert tuple(stored.shape) == (8, 3, 3, 3, 4)
    assert torch.equal(stored, w["conv.weight"].permute(0, 2, 3, 4, 1))


def test_consolidated_file_and_unet_scale_factor(tmp_path):
    w = _small(1)
    path = tmp_path / "model.safetensors"
    W.save_network_file(path, "unet", w, scale_factor=0.875)
    got, scale = W.load_network_file(path, "unet", SMALL)
    assert scale == 0.875 and all(torch.equal(got[k], w[k]) for k in w)
    with pytest.raises(ValueError, match="missing"):
        W.load_network_file(path, "vae", SMALL)  # no vae.* keys in this file


@pytest.mark.parametrize("case", ["missing", "unexpected", "dtype", "nonfinite", "shape", "unet_no_scale",
                                  "vae_with_scale", "suffix"])
def test_rejections(tmp_path, case):
    w = _small(2)
    stored = {k: (t.permute(0, 2, 3, 4, 1) if t.dim() == 5 else t).contiguous() for k, t in w.items()}
    network, name = "vae", "net.safetensors"
    if case == "missing":
        del stored["norm.weight"]
    elif case == "unexpected":
        stored["extra.bias"] = torch.zeros(3)
    elif case == "dtype":
        stored["conv.bias"] = stored["conv.bias"].double()
    elif case == "nonfinite":
        stored["proj.weight"][0, 0] = float("nan")
    elif case == "shape":
        stored["conv.weight"] = w["conv.weight"].contiguous()  # Torch layout on disk: wrong
    elif case == "unet_no_scale":
        network = "unet"
    elif case == "vae_with_scale":
        stored["scale_factor"] = torch.tensor(1.0)
    elif case == "suffix":
        name = "net.bin"
    save_file(stored, str(tmp_path / "store.safetensors"))
    (tmp_path / "store.safetensors").rename(tmp_path / name)
    with pytest.raises(ValueError):
        W.load_network_file(tmp_path / name, network, SMALL)
