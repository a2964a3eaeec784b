"""Network-level oracle: CPU torch restatement of the reference's MAISI modules.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``). Follows the reference's
generic (``medmlx_core.ops``) operation order; tensors are NCDHW, weights keep
their Torch layouts, dtype is the caller's (float32 or float64). File:line
citations are relative to the reference project root.
"""

from __future__ import annotations

import math
from collections.abc import Mapping, Sequence

import numpy as np
import torch
import torch.nn.functional as F

from .ops_ref import avg_pool_ref, conv3d_ref, gaussian_1d_ref, group_norm_ref, silu_ref, upsample_nearest_ref
from .ops_ref import upsample_trilinear_ref

Weights = Mapping[str, torch.Tensor]


def seeded_parameters(recipe: Mapping) -> dict[str, np.ndarray]:
    """Regenerate a fixture's parameters from its recipe (``tests/fixture_parameters.py:15-25``)."""
    rng = np.random.default_rng(int(recipe["seed"]))
    rng.normal(size=int(recipe["skip"]))
    out: dict[str, np.ndarray] = {}
    for name, shape in recipe["shapes"]:
        value = rng.normal(0, 0.02, tuple(shape)).astype(np.float32)
        if value.ndim == 1 and name.endswith("weight"):
            value += np.float32(1)
        out[name] = value
    return out


def prefixed(weights: Weights, prefix: str) -> dict[str, torch.Tensor]:
    """``unet_common.prefixed_weights`` (``unet_common.py:99-104``)."""
    start = prefix + "."
    return {k[len(start):]: v for k, v in weights.items() if k.startswith(start)}


def linear(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor | None) -> torch.Tensor:
    return F.linear(x, w.to(x.dtype), None if b is None else b.to(x.dtype))


def silu_mlp(x, weights: Weights, prefix: str) -> torch.Tensor:
    """``Linear -> SiLU -> Linear`` (``embed.py:58-71``, ``unet_common.py:16-34``)."""
    h = silu_ref(linear(x, weights[f"{prefix}.0.weight"], weights[f"{prefix}.0.bias"]))
    return linear(h, weights[f"{prefix}.2.weight"], weights[f"{prefix}.2.bias"])


def sinusoidal_timestep_embedding(t: torch.Tensor, dim: int, max_period: int = 10000) -> torch.Tensor:
    """``[cos, sin]`` embedding (``embed.py:15-42``), float32 like the reference."""
    half = dim // 2
    exponent = -math.log(max_period) * torch.arange(half, dtype=torch.float32)
    freqs = torch.exp(exponent / half)
    args = t.to(torch.float32).reshape(-1, 1) * freqs.reshape(1, -1)
    emb = torch.cat([torch.cos(args), torch.sin(args)], dim=-1)
    if dim % 2:
        emb = F.pad(emb, (0, 1))
    return emb


def residual_block(x, emb, w: Weights, *, groups: int, eps: float, up=False, down=False) -> torch.Tensor:
    """``DiffusionUNetResnetBlock`` in the generic order of ``residual.py:80-134``."""
    h = silu_ref(group_norm_ref(x, w["norm1.weight"], w["norm1.bias"], groups, eps))
    skip = x
    if up:
        skip, h = upsample_nearest_ref(skip), upsample_nearest_ref(h)
    elif down:
        skip, h = avg_pool_ref(skip), avg_pool_ref(h)
    h = conv3d_ref(h, w["conv1.conv.weight"], w["conv1.conv.bias"])
    temb = linear(silu_ref(emb), w["time_emb_proj.weight"], w["time_emb_proj.bias"])
    h = h + temb[:, :, None, None, None]
    h = silu_ref(group_norm_ref(h, w["norm2.weight"], w["norm2.bias"], groups, eps))
    h = conv3d_ref(h, w["conv2.conv.weight"], w["conv2.conv.bias"])
    if x.shape[1] != w["conv1.conv.weight"].shape[0]:
        skip = conv3d_ref(skip, w["skip_connection.conv.weight"], w["skip_connection.conv.bias"], padding=0)
    return skip + h


def spatial_attention(x, w: Weights, *, groups: int, eps: float, head_channels: int, include_fc=True):
    """``SpatialAttentionBlock`` (``attention.py:92-160``): GN, Q/K/V, softmax(QK^T s)V, out_proj, +x."""
    b, c = x.shape[:2]
    spatial = x.shape[2:]
    heads = c // head_channels
    scale = float(head_channels) ** -0.5
    h = group_norm_ref(x, w["norm.weight"], w["norm.bias"], groups, eps)
    tokens = h.reshape(b, c, -1).transpose(1, 2)
    q, k, v = (linear(tokens, w[f"attn.to_{n}.weight"], w[f"attn.to_{n}.bias"]) for n in "qkv")

    def split(a):
        return a.reshape(b, -1, heads, head_channels).transpose(1, 2)

    scores = torch.matmul(split(q), split(k).transpose(-1, -2)) * scale
    att = torch.matmul(torch.softmax(scores, dim=-1), split(v))
    merged = att.transpose(1, 2).reshape(b, -1, c)
    if include_fc:
        merged = linear(merged, w["attn.out_proj.weight"], w["attn.out_proj.bias"])
    return x + merged.transpose(1, 2).reshape(b, c, *spatial)


def _per_level(value, n):
    return tuple(value) if isinstance(value, (list, tuple)) else (int(value),) * n


def condition_embedding(t, class_labels, spacing, w: Weights, ctor: Mapping, *, with_spacing=True):
    """``unet._condition_embedding`` (``unet.py:190-271``) for the rflow MR/CT networks."""
    t_emb = sinusoidal_timestep_embedding(t, int(ctor["num_channels"][0]))
    emb = silu_mlp(t_emb, w, "time_embed")
    if ctor.get("num_class_embeds") is not None:
        emb = emb + w["class_embedding.weight"].to(emb.dtype)[class_labels.long()]
    if with_spacing and ctor.get("include_spacing_input"):
        emb = torch.cat([emb, silu_mlp(spacing.to(emb.dtype), w, "spacing_layer")], dim=-1)
    return t_emb, emb


def down_blocks(h, emb, w: Weights, ctor: Mapping, down_residuals=None):
    """``unet.apply_down_blocks`` (``unet.py:274-356``)."""
    ch = list(ctor["num_channels"])
    n = len(ch)
    res = _per_level(ctor["num_res_blocks"], n)
    attn = list(ctor["attention_levels"])
    heads = _per_level(ctor["num_head_channels"], n)
    g, eps = int(ctor["norm_num_groups"]), float(ctor["norm_eps"])
    fc = bool(ctor.get("include_fc", True))
    skips = [h]
    for i in range(n):
        for r in range(res[i]):
            h = residual_block(h, emb, prefixed(w, f"down_blocks.{i}.resnets.{r}"), groups=g, eps=eps)
            if attn[i]:
                h = spatial_attention(h, prefixed(w, f"down_blocks.{i}.attentions.{r}"), groups=g, eps=eps,
                                      head_channels=heads[i], include_fc=fc)
            skips.append(h)
        if i != n - 1:
            h = residual_block(h, emb, prefixed(w, f"down_blocks.{i}.downsampler"), groups=g, eps=eps, down=True)
            skips.append(h)
    if down_residuals is not None:
        skips = [s + r for s, r in zip(skips, down_residuals, strict=True)]
        h = skips[-1]
    return h, skips


def mid_block(h, emb, w: Weights, ctor: Mapping):
    """``unet.apply_mid_block`` (``unet.py:359-399``)."""
    n = len(ctor["num_channels"])
    heads = _per_level(ctor["num_head_channels"], n)
    g, eps = int(ctor["norm_num_groups"]), float(ctor["norm_eps"])
    h = residual_block(h, emb, prefixed(w, "middle_block.resnet_1"), groups=g, eps=eps)
    h = spatial_attention(h, prefixed(w, "middle_block.attention"), groups=g, eps=eps, head_channels=heads[-1],
                          include_fc=bool(ctor.get("include_fc", True)))
    return residual_block(h, emb, prefixed(w, "middle_block.resnet_2"), groups=g, eps=eps)


def up_blocks(h, emb, skips, w: Weights, ctor: Mapping):
    """``unet._apply_up_blocks`` (``unet.py:402-487``): concat a skip before every ResBlock."""
    ch = list(ctor["num_channels"])
    n = len(ch)
    res = list(reversed(_per_level(ctor["num_res_blocks"], n)))
    attn = list(reversed(ctor["attention_levels"]))
    heads = list(reversed(_per_level(ctor["num_head_channels"], n)))
    g, eps = int(ctor["norm_num_groups"]), float(ctor["norm_eps"])
    fc = bool(ctor.get("include_fc", True))
    remaining = list(skips)
    for i in range(n):
        k = res[i] + 1
        samples = remaining[-k:]
        remaining = remaining[:-k]
        for r in range(k):
            skip = samples.pop()
            h = torch.cat([h, skip], dim=1)
            h = residual_block(h, emb, prefixed(w, f"up_blocks.{i}.resnets.{r}"), groups=g, eps=eps)
            if attn[i]:
                h = spatial_attention(h, prefixed(w, f"up_blocks.{i}.attentions.{r}"), groups=g, eps=eps,
                                      head_channels=heads[i], include_fc=fc)
        if i != n - 1:
            h = residual_block(h, emb, prefixed(w, f"up_blocks.{i}.upsampler"), groups=g, eps=eps, up=True)
    assert not remaining
    return h


def denoise_unet(x, t, class_labels, spacing, w: Weights, ctor: Mapping, down_residuals=None, mid_residual=None):
    """``unet.denoise_unet_ncdhw`` (``unet.py:42-187``); returns ``(t_emb, y)``."""
    g, eps = int(ctor["norm_num_groups"]), float(ctor["norm_eps"])
    t_emb, emb = condition_embedding(t, class_labels, spacing, w, ctor)
    emb = emb.to(x.dtype)
    h = conv3d_ref(x, w["conv_in.conv.weight"], w["conv_in.conv.bias"])
    h, skips = down_blocks(h, emb, w, ctor, down_residuals)
    h = mid_block(h, emb, w, ctor)
    if mid_residual is not None:
        h = h + mid_residual
    h = up_blocks(h, emb, skips, w, ctor)
    h = silu_ref(group_norm_ref(h, w["out.0.weight"], w["out.0.bias"], g, eps))
    return t_emb, conv3d_ref(h, w["out.2.conv.weight"], w["out.2.conv.bias"])


def controlnet_cond_embed(cond, w: Weights, ctor: Mapping):
    """``controlnet._cond_embed`` (``controlnet.py:197-255``)."""
    chans = list(ctor["conditioning_embedding_num_channels"])
    p = "controlnet_cond_embedding"
    h = silu_ref(conv3d_ref(cond, w[f"{p}.conv_in.conv.weight"], w[f"{p}.conv_in.conv.bias"]))
    block = 0
    for _ in range(len(chans) - 1):
        h = silu_ref(conv3d_ref(h, w[f"{p}.blocks.{block}.conv.weight"], w[f"{p}.blocks.{block}.conv.bias"]))
        block += 1
        h = silu_ref(conv3d_ref(h, w[f"{p}.blocks.{block}.conv.weight"], w[f"{p}.blocks.{block}.conv.bias"],
                                stride=2))
        block += 1
    return conv3d_ref(h, w[f"{p}.conv_out.conv.weight"], w[f"{p}.conv_out.conv.bias"])


def _zero_conv(h, w: Weights, prefix: str):
    """``controlnet._zero_conv`` (``controlnet.py:258-274``)."""
    if f"{prefix}.conv.weight" in w:
        return conv3d_ref(h, w[f"{prefix}.conv.weight"], w[f"{prefix}.conv.bias"], padding=0)
    return conv3d_ref(h, w[f"{prefix}.weight"], w[f"{prefix}.bias"], padding=0)


def controlnet_residuals(x, t, class_labels, cond, w: Weights, ctor: Mapping, conditioning_scale=1.0,
                         conditioning_embedding=None):
    """``controlnet.controlnet_residuals_ncdhw`` (``controlnet.py:31-164``)."""
    _, emb = condition_embedding(t, class_labels, None, w, ctor, with_spacing=False)
    emb = emb.to(x.dtype)
    h = conv3d_ref(x, w["conv_in.conv.weight"], w["conv_in.conv.bias"])
    h = h + (controlnet_cond_embed(cond, w, ctor) if conditioning_embedding is None else conditioning_embedding)
    h, skips = down_blocks(h, emb, w, ctor)
    h = mid_block(h, emb, w, ctor)
    down = [_zero_conv(s, w, f"controlnet_down_blocks.{i}") for i, s in enumerate(skips)]
    mid = _zero_conv(h, w, "controlnet_mid_block")
    if conditioning_scale != 1.0:
        down = [d * conditioning_scale for d in down]
        mid = mid * conditioning_scale
    return down, mid


def _vae_conv_weights(w: Weights, prefix: str):
    """``vae._conv_weights`` (``vae.py:527-537``)."""
    for key in (f"{prefix}.conv.conv", f"{prefix}.conv"):
        if f"{key}.weight" in w:
            return w[f"{key}.weight"], w[f"{key}.bias"]
    raise KeyError(prefix)


def vae_resblock(x, w: Weights, prefix: str, groups: int, eps: float):
    """``MaisiResBlock`` (``vae.py:101-171``)."""
    h = silu_ref(group_norm_ref(x, w[f"{prefix}.norm1.weight"], w[f"{prefix}.norm1.bias"], groups, eps))
    h = conv3d_ref(h, *_vae_conv_weights(w, f"{prefix}.conv1"))
    h = silu_ref(group_norm_ref(h, w[f"{prefix}.norm2.weight"], w[f"{prefix}.norm2.bias"], groups, eps))
    h = conv3d_ref(h, *_vae_conv_weights(w, f"{prefix}.conv2"))
    skip = x
    if f"{prefix}.nin_shortcut.conv.conv.weight" in w or f"{prefix}.nin_shortcut.conv.weight" in w:
        skip = conv3d_ref(x, *_vae_conv_weights(w, f"{prefix}.nin_shortcut"), padding=0)
    return skip + h


def decode_vae(latent, w: Weights, ctor: Mapping):
    """``vae.decode_vae_ncdhw`` + ``run_vae_decoder_ncdhw`` (``vae.py:29-62, 273-379``); returns (post_quant, decoded)."""
    g, eps = int(ctor["norm_num_groups"]), float(ctor["norm_eps"])
    post = conv3d_ref(latent, *_vae_conv_weights(w, "post_quant_conv"), padding=0)
    h = conv3d_ref(post, *_vae_conv_weights(w, "decoder.blocks.0"))
    i = 1
    ch = list(reversed(ctor["num_channels"]))
    nres = list(reversed(ctor["num_res_blocks"]))
    for level in range(len(ch)):
        for _ in range(nres[level]):
            h = vae_resblock(h, w, f"decoder.blocks.{i}", g, eps)
            i += 1
        if level != len(ch) - 1:
            h = conv3d_ref(upsample_trilinear_ref(h), *_vae_conv_weights(w, f"decoder.blocks.{i}.conv"))
            i += 1
    h = group_norm_ref(h, w[f"decoder.blocks.{i}.weight"], w[f"decoder.blocks.{i}.bias"], g, eps)
    return post, conv3d_ref(h, *_vae_conv_weights(w, f"decoder.blocks.{i + 1}"))


# ---------------------------------------------------------------- sliding window (decode.py)

def scan_interval(size, roi, overlap):
    """``decode.scan_interval`` (``decode.py:30-47``)."""
    out = []
    for s, r in zip(size, roi, strict=True):
        if r == s:
            out.append(r)
            continue
        step = int(r * (1.0 - float(overlap)))
        out.append(step if step > 0 else 1)
    return tuple(out)


def window_starts(size, roi, interval):
    """Per-axis window starts of ``decode.dense_patch_slices`` (``decode.py:50-85``)."""
    starts = []
    for s, r, step in zip(size, roi, interval, strict=True):
        count = int(math.ceil(float(s) / float(step)))
        last = next((i for i in range(count) if i * step + r >= s), None)
        n = 1 if last is None else last + 1
        starts.append([i * step - max(i * step + r - s, 0) for i in range(n)])
    return starts


def sliding_window(latent, predict, roi, overlap, sigma_scale=0.125, z_scale=4):
    """``decode.sliding_window_ncdhw`` (``decode.py:115-184``) incl. centred zero padding to the ROI."""
    pads = []
    for axis, r in enumerate(roi):
        extra = max(r - int(latent.shape[axis + 2]), 0)
        pads.append((extra // 2, extra - extra // 2))
    if any(a or b for a, b in pads):
        latent = F.pad(latent, (pads[2][0], pads[2][1], pads[1][0], pads[1][1], pads[0][0], pads[0][1]))
    spatial = tuple(int(n) for n in latent.shape[2:])
    starts = window_starts(spatial, roi, scan_interval(spatial, roi, overlap))
    axes = [torch.from_numpy(gaussian_1d_ref(r, sigma_scale)) for r in roi]
    imp = axes[0].reshape(-1, 1, 1) * axes[1].reshape(1, -1, 1) * axes[2].reshape(1, 1, -1)
    imp = torch.maximum(imp, torch.tensor(1e-3, dtype=torch.float32))
    imp = imp.repeat_interleave(z_scale, 0).repeat_interleave(z_scale, 1).repeat_interleave(z_scale, 2)
    imp = imp.to(latent.dtype)
    out = wsum = None
    for zd in starts[0]:
        for zh in starts[1]:
            for zw in starts[2]:
                pred = predict(latent[:, :, zd:zd + roi[0], zh:zh + roi[1], zw:zw + roi[2]])
                if out is None:
                    out = torch.zeros((pred.shape[0], pred.shape[1], *(n * z_scale for n in spatial)), dtype=pred.dtype)
                    wsum = torch.zeros((1, 1, *(n * z_scale for n in spatial)), dtype=pred.dtype)
                sl = (slice(None), slice(None), slice(zd * z_scale, (zd + roi[0]) * z_scale),
                      slice(zh * z_scale, (zh + roi[1]) * z_scale), slice(zw * z_scale, (zw + roi[2]) * z_scale))
                out[sl] += pred * imp
                wsum[sl] += imp
    stitched = out / wsum
    crop = tuple(slice(a * z_scale, stitched.shape[i + 2] - b * z_scale) for i, (a, b) in enumerate(pads))
    return stitched[(slice(None), slice(None), *crop)]


def sliding_window_decode(latent, w: Weights, ctor: Mapping, roi, overlap, scale_factor=None, sigma_scale=0.125):
    """``decode.sliding_window_decode_ncdhw`` (``decode.py:187-245``)."""
    if scale_factor is not None:
        latent = latent / torch.tensor(float(scale_factor), dtype=torch.float32).to(latent.dtype)
    spatial = tuple(int(n) for n in latent.shape[2:])
    if math.prod(spatial) <= math.prod(roi):
        return decode_vae(latent, w, ctor)[1]
    adjusted = tuple(min(r, s) for r, s in zip(roi, spatial, strict=True))
    return sliding_window(latent, lambda win: decode_vae(win, w, ctor)[1], adjusted, overlap, sigma_scale)


# ---------------------------------------------------------------- rflow sampler (rflow.py, image.py)

def set_timesteps_rflow(num_inference_steps: int, input_img_size_numel: int, base=32 ** 3, train=1000):
    """``rflow.set_timesteps_rflow`` (``rflow.py:48-98``) incl. the FP16 rounding of the schedule."""
    steps = []
    for i in range(num_inference_steps):
        raw = (1.0 - i / num_inference_steps) * train
        u = raw / train
        r = (float(input_img_size_numel) / float(base)) ** (1.0 / 3.0)
        steps.append(train * r * u / (1.0 + (r - 1.0) * u))
    ts = np.asarray(steps, dtype=np.float16).astype(np.float32)
    return ts, np.concatenate([ts[1:], np.zeros((1,), dtype=np.float32)])


def euler_dt(t: float, next_t: float, train: int = 1000) -> float:
    """``rflow.step_rflow``'s ``dt`` with the truncated next timestep (``rflow.py:101-121``)."""
    return (float(t) - int(float(next_t))) / float(train)


def guided_velocity(z, t, class_label, spacing, w: Weights, ctor: Mapping, guidance: float):
    """``image.guided_velocity`` batched CFG (``image.py:118-175``)."""
    tt = torch.full((z.shape[0],), float(t), dtype=torch.float32)
    if guidance == 0.0:
        return denoise_unet(z, tt, class_label, spacing, w, ctor)[1]
    classes = torch.cat([class_label, torch.zeros_like(class_label)])
    _, v = denoise_unet(torch.cat([z, z]), torch.cat([tt, tt]), classes, torch.cat([spacing, spacing]), w, ctor)
    c, u = v[: z.shape[0]], v[z.shape[0]:]
    return u + guidance * (c - u)


def sample_rflow(z, velocity_fn, timesteps):
    """``rflow.sample_rflow`` (``rflow.py:144-177``)."""
    nxt = np.concatenate([timesteps[1:], np.zeros((1,), dtype=np.float32)])
    for t, n in zip(timesteps.tolist(), nxt.tolist(), strict=True):
        v = velocity_fn(z, float(t))
        z = z + v * euler_dt(t, n)
    return z


def image_spacing_tensor(spacing_mm: Sequence[float]) -> torch.Tensor:
    """``spacing_mm * 100`` rounded through FP16 (``image.py:90-115``)."""
    scaled = np.asarray([spacing_mm], dtype=np.float64) * 100.0
    return torch.from_numpy(scaled.astype(np.float16).astype(np.float32))


def output_intensities(decoded: np.ndarray, configuration: str) -> np.ndarray:
    """int16 image of ``image.output_intensities`` (``image.py:68-87``)."""
    data = np.asarray(decoded, dtype=np.float32)
    if configuration == "ct":
        scaled = np.clip(data * 2000.0 - 1000.0, -1000.0, 1000.0)
    else:
        scaled = np.clip(data * 1000.0, 0.0, None)
    return scaled.astype(np.int16)


def binarize_labels(label: torch.Tensor, bits: int = 8) -> torch.Tensor:
    """8 bit-planes of integer labels (``condition.py:20-43``)."""
    ids = label.to(torch.int32)[:, 0]
    planes = [((ids >> k) & 1).to(torch.float32) for k in range(bits)]
    return torch.stack(planes, dim=1)


def spacing_tensor(spacing_mm: Sequence[float]) -> torch.Tensor:
    """CT-path spacing: ``spacing_mm * 100`` as (1, 3) fp32, no FP16 rounding (``condition.py:46-64``)."""
    return torch.tensor([[float(a) * 100.0 for a in spacing_mm]], dtype=torch.float32)


def to_hu(decoded: torch.Tensor, label: torch.Tensor) -> torch.Tensor:
    """``decode.to_hu_ncdhw`` (``decode.py:248-259``)."""
    hu = decoded.clamp(0.0, 1.0) * 2000.0 - 1000.0
    return torch.where(label == 0, torch.tensor(-1000.0, dtype=hu.dtype), hu)


def sample_ct_from_mask(label, spacing_mm, unet_w: Weights, unet_ctor: Mapping, cn_w: Weights, cn_ctor: Mapping,
                        vae_w: Weights, vae_ctor: Mapping, latent, num_inference_steps: int, scale_factor: float,
                        roi, overlap, modality: int = 1):
    """``from_mask.sample_ct_from_mask_ncdhw`` (``from_mask.py:121-295``): ControlNet-conditioned rflow,
    sliding-window decode, HU mapping. Returns ``(latent, decoded, hu)``."""
    cond = binarize_labels(label)
    embedding = controlnet_cond_embed(cond, cn_w, cn_ctor)
    spacing = spacing_tensor(spacing_mm).repeat(latent.shape[0], 1)
    classes = torch.full((latent.shape[0],), int(modality), dtype=torch.int64)
    timesteps, _ = set_timesteps_rflow(num_inference_steps, int(np.prod(latent.shape[2:])))

    def velocity(z, t):
        tt = torch.full((z.shape[0],), float(t), dtype=torch.float32)
        down, mid = controlnet_residuals(z, tt, classes, cond, cn_w, cn_ctor, conditioning_embedding=embedding)
        return denoise_unet(z, tt, classes, spacing, unet_w, unet_ctor, down_residuals=down, mid_residual=mid)[1]

    final = sample_rflow(latent, velocity, timesteps)
    decoded = sliding_window_decode(final, vae_w, vae_ctor, roi, overlap, scale_factor=scale_factor)
    return final, decoded, to_hu(decoded, label)
