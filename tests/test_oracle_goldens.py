"""Pin the CPU oracle to the reference's recorded golden vectors (tests/golden/*.npz).

Tolerances are the reference's own (``maisi_mlx_feasibility.py:10-29``):
residual 1e-5/1e-6, attention/VAE/UNet 1e-4/1e-5 (rtol/atol, numpy allclose).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from golden_io import load, t, weights
from oracle import networks_ref as N

RESIDUAL = dict(rtol=1e-5, atol=1e-6)
NET = dict(rtol=1e-4, atol=1e-5)


def _allclose(actual: torch.Tensor, expected: np.ndarray, tol: dict) -> None:
    np.testing.assert_allclose(actual.detach().numpy(), expected, **tol)


def test_residual_block_golden():
    a, meta = load("maisi_residual")
    c = meta["constructor"]
    y = N.residual_block(t(a["x"]), t(a["emb"]), weights(meta), groups=c["norm_num_groups"], eps=c["norm_eps"])
    _allclose(y, a["y"], RESIDUAL)


def test_attention_golden():
    a, meta = load("maisi_attention")
    c = meta["constructor"]
    y = N.spatial_attention(t(a["x"]), weights(meta), groups=c["norm_num_groups"], eps=c["norm_eps"],
                            head_channels=c["num_head_channels"], include_fc=c["include_fc"])
    _allclose(y, a["y"], NET)


def test_vae_decoder_golden():
    a, meta = load("maisi_vae")
    post, dec = N.decode_vae(t(a["z"]), weights(meta), meta["constructor"])
    _allclose(post, a["post_quant"], NET)
    _allclose(dec, a["decoded"], NET)


def test_vae_decode_and_tiled_golden():
    """``tests/fixture_cases.py:80-88``: direct decode and roi (2,2,2) / overlap 0.5 / scale 1.25 tiles."""
    a, meta = load("vae")
    w = weights(meta)
    _, dec = N.decode_vae(t(a["input.z"]), w, meta["constructor"])
    _allclose(dec, a["output.decoded"], NET)
    tiled = N.sliding_window_decode(t(a["input.z"]), w, meta["constructor"], (2, 2, 2), 0.5, scale_factor=1.25)
    _allclose(tiled, a["output.tiled"], NET)


def test_diffusion_unet_golden():
    a, meta = load("maisi_diffusion")
    t_emb, y = N.denoise_unet(t(a["x"]), t(a["timesteps"]), torch.from_numpy(a["class_labels"]), t(a["spacing"]),
                              weights(meta), meta["constructor"])
    _allclose(t_emb, a["t_emb"], NET)
    _allclose(y, a["y"], NET)


def test_unet_case_golden():
    a, meta = load("unet")
    _, y = N.denoise_unet(t(a["input.x"]), t(a["input.timesteps"]), torch.from_numpy(a["input.class_labels"]),
                          t(a["input.spacing"]), weights(meta), meta["constructor"])
    _allclose(y, a["output.velocity"], NET)


def test_scheduler_golden():
    a, meta = load("maisi_scheduler")
    ts, nxt = N.set_timesteps_rflow(30, meta["input_img_size_numel"])
    np.testing.assert_array_equal(ts, a["timesteps"])
    np.testing.assert_array_equal(nxt, a["next_timesteps"])
    dt = N.euler_dt(float(a["timesteps"][0]), float(a["next_timesteps"][0]))
    np.testing.assert_allclose(np.float32(dt), a["dt"], rtol=1e-6)
    z, v = t(a["z"]), t(a["v"])
    np.testing.assert_allclose((z + v * dt).numpy(), a["z_next"], rtol=1e-6, atol=1e-7)


def test_rflow_case_golden():
    """``tests/fixture_cases.py:136-155``: 7-step schedule for 64 voxels, one step, and a toy sample."""
    a, _ = load("rflow")
    ts, nxt = N.set_timesteps_rflow(7, 64)
    np.testing.assert_array_equal(ts, a["output.timesteps"])
    np.testing.assert_array_equal(nxt, a["output.next_timesteps"])
    x = t(a["input.x"])
    dt = N.euler_dt(ts[1], nxt[1])
    np.testing.assert_allclose((x + (x * 0.125) * dt).numpy(), a["output.step"], rtol=1e-6, atol=1e-7)
    np.testing.assert_allclose((x + (x * 0.125) * (float(ts[1]) / 1000.0)).numpy(), a["output.origin"],
                               rtol=1e-6, atol=1e-7)
    sample = N.sample_rflow(x, lambda cur, step: cur * 0.125 + step * 0.0001, ts)
    np.testing.assert_allclose(sample.numpy(), a["output.sample"], rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("name", ["mr_brain", "mr"])
def test_mr_pipeline_golden(name):
    """``tests/test_mr.py:158-247``: conditions, CFG velocity batch, 30-step latent, decode, int16 image."""
    a, meta = load(name)
    ctor = meta["constructor"]
    unet_w, vae_w = weights(meta, "weight.unet."), weights(meta, "weight.vae.")
    spacing = N.image_spacing_tensor(a["input.spacing_mm"].tolist())
    np.testing.assert_array_equal(spacing.numpy(), a["output.spacing"])
    np.testing.assert_array_equal(N.image_spacing_tensor(a["input.spacing_probe"].tolist()).numpy(),
                                  a["output.spacing_probe"])
    ts, _ = N.set_timesteps_rflow(30, 8 ** 3)
    np.testing.assert_array_equal(ts, a["output.timesteps"])
    x = t(a["input.latent"])
    modality = int(meta["modality"])
    np.testing.assert_array_equal(np.array([modality]), a["output.classes"])
    _, v = N.denoise_unet(torch.cat([x, x]), torch.tensor([1000.0, 1000.0]), torch.tensor([modality, 0]),
                          spacing.repeat(2, 1), unet_w, ctor["unet"])
    _allclose(v, a["output.velocity_batch"], NET)
    label = torch.tensor([modality])
    latent = N.sample_rflow(
        x, lambda z, step: N.guided_velocity(z, step, label, spacing, unet_w, ctor["unet"], float(meta["guidance_scale"])),
        ts)
    _allclose(latent, a["output.latent"], NET)
    decoded = N.sliding_window_decode(latent, vae_w, ctor["vae"], (80, 80, 80), 0.4, scale_factor=1.25)
    _allclose(decoded, a["output.decoded"], NET)
    np.testing.assert_array_equal(N.output_intensities(a["output.decoded"], meta["configuration"]), a["output.image"])
