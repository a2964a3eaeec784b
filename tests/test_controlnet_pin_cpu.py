"""The oracle's ControlNet path tied to a reference golden (CPU).

The reference checkout records no ControlNet output. Its ControlNet applies one named
"zero convolution" per skip and one to the middle block (``controlnet.py:156-160, 258-274``), the
1x1x1 projections that the MONAI architecture it evaluates constructs as zeros, as it does the
conditioning embedding's last conv. With those at zero the ControlNet hands the UNet all-zero
residuals, and the controlled UNet must reproduce the plain UNet's recorded output. This runs the
oracle's ``controlnet_residuals`` and the residual-injecting ``denoise_unet`` on the
``maisi_diffusion`` fixture (``unet.py:274-356`` adds the residuals to the skips) against that
golden, and checks the ControlNet's wiring (conv_in + condition, encoder, middle block, one zero
conv per skip) against the oracle's UNet encoder run on the same weights.
"""

from __future__ import annotations

import numpy as np
import torch

from golden_io import load, t, weights
from oracle import networks_ref as N

NET = dict(rtol=1e-4, atol=1e-5)


def _controlnet_weights(unet_w: dict[str, torch.Tensor], ctor: dict, cond_channels: tuple[int, ...], cond_in: int,
                        seed: int, zero: bool) -> dict[str, torch.Tensor]:
    """ControlNet parameters for ``ctor``'s encoder: the UNet's names and shapes for the shared
    parts (time and class embeddings, conv_in, down and middle blocks; no spacing input, so the
    time-embedding projections take the time width), a conditioning embedding of ``cond_channels``,
    and the output convs (zero when ``zero``, as freshly constructed)."""
    g = torch.Generator().manual_seed(seed)
    time_dim = int(unet_w["time_embed.2.weight"].shape[0])
    w: dict[str, torch.Tensor] = {}
    for k, v in unet_w.items():
        if k.startswith(("time_embed.", "class_embedding.", "conv_in.", "down_blocks.", "middle_block.")):
            shape = tuple(v.shape)
            if k.endswith("time_emb_proj.weight"):
                shape = (shape[0], time_dim)
            w[k] = torch.randn(shape, generator=g) * 0.3
    p = "controlnet_cond_embedding"
    chans = list(cond_channels)
    w[f"{p}.conv_in.conv.weight"] = torch.randn((chans[0], cond_in, 3, 3, 3), generator=g) * 0.3
    w[f"{p}.conv_in.conv.bias"] = torch.randn(chans[0], generator=g) * 0.1
    block = 0
    for i in range(len(chans) - 1):
        for c_in, c_out in ((chans[i], chans[i]), (chans[i], chans[i + 1])):
            w[f"{p}.blocks.{block}.conv.weight"] = torch.randn((c_out, c_in, 3, 3, 3), generator=g) * 0.3
            w[f"{p}.blocks.{block}.conv.bias"] = torch.randn(c_out, generator=g) * 0.1
            block += 1
    c0 = int(ctor["num_channels"][0])
    out_w = torch.zeros((c0, chans[-1], 3, 3, 3)) if zero else torch.randn((c0, chans[-1], 3, 3, 3), generator=g)
    w[f"{p}.conv_out.conv.weight"] = out_w
    w[f"{p}.conv_out.conv.bias"] = torch.zeros(c0)
    return w


def _skip_channels(ctor: dict) -> list[int]:
    ch = [int(c) for c in ctor["num_channels"]]
    res = ctor["num_res_blocks"]
    res = list(res) if isinstance(res, (list, tuple)) else [int(res)] * len(ch)
    out = [ch[0]]
    for i, c in enumerate(ch):
        out += [c] * res[i]
        if i != len(ch) - 1:
            out.append(c)
    return out


def _add_output_convs(w: dict[str, torch.Tensor], ctor: dict, make) -> None:
    for i, c in enumerate(_skip_channels(ctor)):
        w[f"controlnet_down_blocks.{i}.conv.weight"], w[f"controlnet_down_blocks.{i}.conv.bias"] = make(c)
    c = int(ctor["num_channels"][-1])
    w["controlnet_mid_block.conv.weight"], w["controlnet_mid_block.conv.bias"] = make(c)


def _cond(shape, seed: int) -> torch.Tensor:
    return (torch.rand(shape, generator=torch.Generator().manual_seed(seed)) > 0.5).float()


def test_fresh_controlnet_leaves_the_unet_golden_unchanged():
    a, meta = load("maisi_diffusion")
    ctor = dict(meta["constructor"], conditioning_embedding_num_channels=[4, 8], conditioning_embedding_in_channels=8)
    unet_w = weights(meta)
    cn_w = _controlnet_weights(unet_w, ctor, (4, 8), 8, seed=3, zero=True)
    _add_output_convs(cn_w, ctor, lambda c: (torch.zeros((c, c, 1, 1, 1)), torch.zeros(c)))
    x, ts = t(a["x"]), t(a["timesteps"])
    labels = torch.from_numpy(a["class_labels"])
    cond = _cond((1, 8, *(2 * n for n in x.shape[2:])), seed=5)  # one stride-2 block: twice the latent grid
    down, mid = N.controlnet_residuals(x, ts, labels, cond, cn_w, ctor)
    assert len(down) == len(_skip_channels(ctor))
    assert all(not r.any() for r in down) and not mid.any()
    _, y = N.denoise_unet(x, ts, labels, t(a["spacing"]), unet_w, meta["constructor"], down_residuals=down,
                          mid_residual=mid)
    np.testing.assert_allclose(y.numpy(), a["y"], **NET)


def test_controlnet_wiring_matches_the_unet_encoder():
    """Identity output convs and a zero condition: the residuals are the encoder's skips and middle
    output, i.e. the oracle's UNet encoder (pinned by the UNet goldens) on the ControlNet's weights."""
    a, meta = load("maisi_diffusion")
    ctor = dict(meta["constructor"], conditioning_embedding_num_channels=[4, 8], conditioning_embedding_in_channels=8,
                include_spacing_input=False)
    unet_w = weights(meta)
    cn_w = _controlnet_weights(unet_w, ctor, (4, 8), 8, seed=11, zero=True)
    _add_output_convs(cn_w, ctor, lambda c: (torch.eye(c).reshape(c, c, 1, 1, 1), torch.zeros(c)))
    x, ts = t(a["x"]), t(a["timesteps"])
    labels = torch.from_numpy(a["class_labels"])
    cond = _cond((1, 8, *(2 * n for n in x.shape[2:])), seed=7)
    down, mid = N.controlnet_residuals(x, ts, labels, cond, cn_w, ctor)
    _, emb = N.condition_embedding(ts, labels, None, cn_w, ctor, with_spacing=False)
    h = N.conv3d_ref(x, cn_w["conv_in.conv.weight"], cn_w["conv_in.conv.bias"])
    h, skips = N.down_blocks(h, emb, cn_w, ctor)
    h = N.mid_block(h, emb, cn_w, ctor)
    for r, s in zip(down, skips, strict=True):
        torch.testing.assert_close(r, s, rtol=1e-6, atol=1e-6)
    torch.testing.assert_close(mid, h, rtol=1e-6, atol=1e-6)
    # A conditioning scale scales every residual.
    half_down, half_mid = N.controlnet_residuals(x, ts, labels, cond, cn_w, ctor, conditioning_scale=0.5)
    for r, s in zip(half_down, down, strict=True):
        torch.testing.assert_close(r, 0.5 * s, rtol=1e-6, atol=1e-7)
    torch.testing.assert_close(half_mid, 0.5 * mid, rtol=1e-6, atol=1e-7)
