"""MAISI networks on the B200 arithmetic (``fast_b200``): rflow UNet, ControlNet and VAE decoder.

Same signatures, weight names (Torch layouts) and validation as the reference's
``unet.py``, ``controlnet.py``, ``vae.py`` and ``residual.py``, restricted to the
path ``fast_fp32`` takes there (the fused ResBlocks and the flash-attention
route). Inputs may be any NCDHW torch CUDA tensors; outputs are NCDHW-shaped
tensors stored channels-last.
"""

from __future__ import annotations

from collections.abc import Mapping, Sequence

import torch

from . import fast_b200 as A
from . import ops

Weights = Mapping[str, torch.Tensor]

_RES_KEYS = ("norm1.weight", "norm1.bias", "conv1.conv.weight", "conv1.conv.bias", "time_emb_proj.weight",
             "time_emb_proj.bias", "norm2.weight", "norm2.bias", "conv2.conv.weight", "conv2.conv.bias")
_SKIP_KEYS = ("skip_connection.conv.weight", "skip_connection.conv.bias")


def required_weight(weights: Weights, key: str) -> torch.Tensor:
    """``unet_common.required_weight`` (``unet_common.py:107-113``)."""
    if key not in weights:
        raise ValueError(f"UNet weights missing: {key}")
    return weights[key]


def prefixed_weights(weights: Weights, prefix: str) -> dict[str, torch.Tensor]:
    """``unet_common.prefixed_weights`` (``unet_common.py:99-104``)."""
    start = prefix + "."
    return {k[len(start):]: v for k, v in weights.items() if k.startswith(start)}


def per_level(value, n: int, name: str) -> tuple[int, ...]:
    """``unet_common.per_level`` (``unet_common.py:145-154``)."""
    if isinstance(value, int) and not isinstance(value, bool):
        return (int(value),) * n
    if isinstance(value, Sequence) and not isinstance(value, (str, bytes)):
        out = tuple(int(v) for v in value)
        if len(out) != n:
            raise ValueError(f"{name} length {len(out)} != num_channels {n}")
        return out
    raise ValueError(f"{name} must be int or sequence")


def _require_ncdhw(x, name: str) -> None:
    shape = x.shape
    if len(shape) != 5:
        raise ValueError(f"{name} must be NCDHW (5-D); got shape {tuple(shape)}")


def residual_block_ncdhw(x, emb: torch.Tensor, weights: Weights, *, num_groups: int, eps: float, up: bool = False,
                         down: bool = False) -> torch.Tensor:
    """``residual.residual_block_ncdhw`` validation (``residual.py:55-78``) then the fused block.

    ``emb`` may be a ``TimeBiasTable`` holding every block's projected embedding.
    """
    time_bias = None
    if isinstance(emb, A.TimeBiasTable):
        time_bias = emb.bias_for(weights)
        emb = emb.emb
    _require_ncdhw(x, "residual input")
    if emb.dim() != 2:
        raise ValueError(f"residual emb must be [N, temb]; got ndim={emb.dim()}")
    if up and down:
        raise ValueError("residual block cannot upsample and downsample together")
    missing = [k for k in _RES_KEYS if k not in weights]
    if missing:
        raise ValueError("residual weights missing: " + ", ".join(missing))
    if int(x.shape[1]) != int(weights["conv1.conv.weight"].shape[0]):
        skip_missing = [k for k in _SKIP_KEYS if k not in weights]
        if skip_missing:
            raise ValueError("residual skip weights missing: " + ", ".join(skip_missing))
    return A.residual_block_ncdhw(x, emb, weights, num_groups=num_groups, eps=eps, up=up, down=down,
                                  time_bias=time_bias)


def _silu_mlp(x: torch.Tensor, weights: Weights, prefix: str) -> torch.Tensor:
    h = A.silu(A.linear(x, required_weight(weights, f"{prefix}.0.weight"), required_weight(weights, f"{prefix}.0.bias")))
    return A.linear(h, required_weight(weights, f"{prefix}.2.weight"), required_weight(weights, f"{prefix}.2.bias"))


def condition_embedding(timesteps, class_labels, spacing, weights: Weights, constructor: Mapping,
                        with_spacing: bool = True) -> tuple[torch.Tensor, torch.Tensor]:
    """``unet._condition_embedding`` (``unet.py:190-271``) for the rflow networks, fp32."""
    t_emb = A.sinusoidal_timestep_embedding(timesteps, int(constructor["num_channels"][0]))
    emb = _silu_mlp(t_emb, weights, "time_embed")
    if constructor.get("num_class_embeds") is not None:
        if class_labels is None:
            raise ValueError("class_labels should be provided when num_class_embeds > 0")
        emb = emb + required_weight(weights, "class_embedding.weight").to(torch.float32)[class_labels.long()]
    if with_spacing and constructor.get("include_spacing_input"):
        if spacing is None:
            raise ValueError("spacing should be provided when include_spacing_input is true")
        if spacing.dim() != 2 or int(spacing.shape[-1]) != 3:
            raise ValueError(f"spacing must be [N, 3]; got shape={tuple(spacing.shape)}")
        emb = torch.cat([emb, _silu_mlp(spacing.to(torch.float32), weights, "spacing_layer")], dim=-1)
    return t_emb, emb


def _levels(constructor: Mapping):
    ch = [int(c) for c in constructor["num_channels"]]
    n = len(ch)
    return (ch, per_level(constructor["num_res_blocks"], n, "num_res_blocks"), list(constructor["attention_levels"]),
            per_level(constructor["num_head_channels"], n, "num_head_channels"), int(constructor["norm_num_groups"]),
            float(constructor["norm_eps"]), bool(constructor.get("include_fc", True)))


class Joined(list):
    """ControlNet residuals still being produced on ``stream``: the consumer's stream waits for
    that stream before it first reads them."""

    def __init__(self, items, stream: torch.cuda.Stream) -> None:
        super().__init__(items)
        self.stream = stream

    def join(self) -> None:
        torch.cuda.current_stream(self.stream.device).wait_stream(self.stream)


def apply_down_blocks(hidden, emb, weights: Weights, constructor: Mapping, down_block_additional_residuals=None):
    """``unet.apply_down_blocks`` (``unet.py:274-356``) with ``resblock_updown``."""
    ch, res, attn, heads, g, eps, fc = _levels(constructor)
    if not bool(constructor.get("resblock_updown", True)):
        raise ValueError("the B200 path implements the resblock_updown=True MAISI networks")
    skips = [hidden]
    for i in range(len(ch)):
        for r in range(res[i]):
            hidden = residual_block_ncdhw(hidden, emb, prefixed_weights(weights, f"down_blocks.{i}.resnets.{r}"),
                                          num_groups=g, eps=eps)
            if attn[i]:
                hidden = A.spatial_attention_ncdhw(hidden, prefixed_weights(weights, f"down_blocks.{i}.attentions.{r}"),
                                                   num_groups=g, eps=eps, num_head_channels=heads[i], include_fc=fc)
            skips.append(hidden)
        if i != len(ch) - 1:
            hidden = residual_block_ncdhw(hidden, emb, prefixed_weights(weights, f"down_blocks.{i}.downsampler"),
                                          num_groups=g, eps=eps, down=True)
            skips.append(hidden)
    if down_block_additional_residuals is not None:
        if isinstance(down_block_additional_residuals, Joined):
            down_block_additional_residuals.join()
        extras = list(down_block_additional_residuals)
        if len(extras) != len(skips):
            raise ValueError(f"ControlNet residuals length {len(extras)} != UNet skip count {len(skips)}")
        skips = [s + ops.to_ndhwc(r, s.dtype) for s, r in zip(skips, extras, strict=True)]
        hidden = skips[-1]
    return hidden, skips


def apply_mid_block(hidden, emb, weights: Weights, constructor: Mapping):
    """``unet.apply_mid_block`` (``unet.py:359-399``)."""
    _, _, _, heads, g, eps, fc = _levels(constructor)
    hidden = residual_block_ncdhw(hidden, emb, prefixed_weights(weights, "middle_block.resnet_1"), num_groups=g, eps=eps)
    hidden = A.spatial_attention_ncdhw(hidden, prefixed_weights(weights, "middle_block.attention"), num_groups=g,
                                       eps=eps, num_head_channels=heads[-1], include_fc=fc)
    return residual_block_ncdhw(hidden, emb, prefixed_weights(weights, "middle_block.resnet_2"), num_groups=g, eps=eps)


def apply_up_blocks(hidden, emb, skips: list, weights: Weights, constructor: Mapping):
    """``unet._apply_up_blocks`` (``unet.py:402-487``); the skip concat is never materialised."""
    ch, res, attn, heads, g, eps, fc = _levels(constructor)
    n = len(ch)
    res_r, attn_r, heads_r = list(reversed(res)), list(reversed(attn)), list(reversed(heads))
    remaining = list(skips)
    for i in range(n):
        k = res_r[i] + 1
        if len(remaining) < k:
            raise ValueError(f"UNet skip list too short: need {k} for up_blocks.{i}, have {len(remaining)}")
        samples, remaining = remaining[-k:], remaining[:-k]
        for r in range(k):
            skip = samples.pop()
            hidden = A.concat_channels_ncdhw(hidden, skip)
            hidden = residual_block_ncdhw(hidden, emb, prefixed_weights(weights, f"up_blocks.{i}.resnets.{r}"),
                                          num_groups=g, eps=eps)
            if attn_r[i]:
                hidden = A.spatial_attention_ncdhw(hidden, prefixed_weights(weights, f"up_blocks.{i}.attentions.{r}"),
                                                   num_groups=g, eps=eps, num_head_channels=heads_r[i], include_fc=fc)
        if i != n - 1:
            hidden = residual_block_ncdhw(hidden, emb, prefixed_weights(weights, f"up_blocks.{i}.upsampler"),
                                          num_groups=g, eps=eps, up=True)
    if remaining:
        raise ValueError(f"UNet skip list leftover after up blocks: {len(remaining)}")
    return hidden


def _refuse_unsupported(constructor: Mapping) -> None:
    """``unet._refuse_unsupported`` (``unet.py:490-504``)."""
    if int(constructor.get("spatial_dims", 3)) != 3:
        raise ValueError("MAISI UNet dest is 3D NCDHW")
    if bool(constructor.get("use_flash_attention")):
        raise ValueError("CUDA flash attention is not a destination here")
    if bool(constructor.get("with_conditioning")):
        raise ValueError("MAISI UNet dest has with_conditioning=false")
    if bool(constructor.get("use_combined_linear")):
        raise ValueError("MAISI UNet dest uses separate QKV projections")


def denoise_unet_ncdhw(x, timesteps, class_labels, spacing, weights: Weights, *, constructor: Mapping, mx=None,
                       down_block_additional_residuals=None, mid_block_additional_residual=None):
    """One denoiser pass; returns ``(t_emb, y)`` (``unet.py:42-187``)."""
    _require_ncdhw(x, "unet input")
    _refuse_unsupported(constructor)
    if int(x.shape[1]) != int(constructor["in_channels"]):
        raise ValueError(f"unet input channels {int(x.shape[1])} != in_channels {constructor['in_channels']}")
    if len(constructor["attention_levels"]) != len(constructor["num_channels"]):
        raise ValueError("attention_levels length must match num_channels")
    g, eps = int(constructor["norm_num_groups"]), float(constructor["norm_eps"])
    w_in, b_in = required_weight(weights, "conv_in.conv.weight"), required_weight(weights, "conv_in.conv.bias")
    side = None
    if A.SKIP_SIDE_STREAM and x.is_cuda and int(w_in.shape[2]) == 3:
        # conv_in runs on a side stream beside the condition embedding's small launches; its output
        # is allocated (and its weight packed) on the caller's stream, which joins before the blocks.
        xin = ops.to_ndhwc(x, A.activation_dtype())
        hidden = ops.empty_ndhwc(int(xin.shape[0]), int(w_in.shape[0]), *(int(n) for n in xin.shape[2:]),
                                 A.activation_dtype(), xin.device)
        packed_in = A._pack(w_in)
        with A.beside(xin.device) as side:
            ops.conv3d(xin, packed_in, b_in, out=hidden, stats=A._want_stats(xin, int(w_in.shape[0])))
    else:
        hidden = A.conv3d_ncdhw(ops.to_ndhwc(x), w_in, b_in, padding=1)
    t_emb, emb = condition_embedding(timesteps, class_labels, spacing, weights, constructor)
    emb = A.TimeBiasTable(emb, weights)  # every block's projected embedding in one GEMM
    if side is not None:
        torch.cuda.current_stream(side.device).wait_stream(side)
    hidden, skips = apply_down_blocks(hidden, emb, weights, constructor, down_block_additional_residuals)
    hidden = apply_mid_block(hidden, emb, weights, constructor)
    if mid_block_additional_residual is not None:
        hidden = hidden + ops.to_ndhwc(mid_block_additional_residual, hidden.dtype)
    hidden = apply_up_blocks(hidden, emb, skips, weights, constructor)
    y = A.norm_conv3d_ncdhw(hidden, required_weight(weights, "out.2.conv.weight"),
                            required_weight(weights, "out.2.conv.bias"),
                            norm=(required_weight(weights, "out.0.weight"), required_weight(weights, "out.0.bias")),
                            num_groups=g, eps=eps, apply_silu=True)
    return t_emb, y


# ---------------------------------------------------------------- ControlNet
def _cond_embed(cond, weights: Weights, channels: Sequence[int]) -> torch.Tensor:
    """``controlnet._cond_embed`` (``controlnet.py:197-255``): each SiLU after a conv runs in the next conv's prologue."""
    p = "controlnet_cond_embedding"
    w_in, b_in = required_weight(weights, f"{p}.conv_in.conv.weight"), required_weight(weights, f"{p}.conv_in.conv.bias")
    if isinstance(cond, ops.LabelBits):
        # The bit planes are formed in conv_in's operand pass from the int16 labels.
        h = ops.conv3d(cond, A._pack(w_in), b_in, out_dtype=A.activation_dtype())
    else:
        h = A.conv3d_ncdhw(ops.to_ndhwc(cond), w_in, b_in, padding=1)
    block = 0
    dtype = A.activation_dtype()
    for _ in range(len(channels) - 1):
        for stride in (1, 2):
            w = required_weight(weights, f"{p}.blocks.{block}.conv.weight")
            b = required_weight(weights, f"{p}.blocks.{block}.conv.bias")
            h = ops.conv3d(h, A._pack(w), b, silu=True, stride=stride, out_dtype=dtype)
            block += 1
    w = required_weight(weights, f"{p}.conv_out.conv.weight")
    return ops.conv3d(h, A._pack(w), required_weight(weights, f"{p}.conv_out.conv.bias"), silu=True, out_dtype=dtype)


def encode_controlnet_condition_ncdhw(cond, weights: Weights, *, constructor: Mapping, mx=None) -> torch.Tensor:
    """Encode the label condition once for all denoising steps (``controlnet.py:167-194``)."""
    _require_ncdhw(cond, "controlnet cond")
    channels = [int(c) for c in constructor["conditioning_embedding_num_channels"]]
    if int(cond.shape[1]) != int(constructor["conditioning_embedding_in_channels"]):
        raise ValueError(f"controlnet cond channels {int(cond.shape[1])} != "
                         f"{constructor['conditioning_embedding_in_channels']}")
    scale = 2 ** (len(channels) - 1)
    if any(int(s) % scale for s in cond.shape[2:]):
        raise ValueError(f"controlnet cond spatial sizes must be multiples of {scale}")
    return _cond_embed(cond, weights, channels)


def _zero_conv(h, weights: Weights, prefix: str) -> torch.Tensor:
    if f"{prefix}.conv.weight" in weights:
        w, b = weights[f"{prefix}.conv.weight"], required_weight(weights, f"{prefix}.conv.bias")
    elif f"{prefix}.weight" in weights:
        w, b = weights[f"{prefix}.weight"], required_weight(weights, f"{prefix}.bias")
    else:
        raise ValueError(f"ControlNet weights missing: {prefix}.conv.weight or {prefix}.weight")
    return A.conv3d_ncdhw(h, w, b, padding=0)


def controlnet_residuals_ncdhw(x, timesteps, class_labels, cond, weights: Weights, *, constructor: Mapping, mx=None,
                               conditioning_scale: float = 1.0, conditioning_embedding=None):
    """ControlNet down/mid residuals for the UNet (``controlnet.py:31-164``)."""
    _require_ncdhw(x, "controlnet latent")
    _refuse_unsupported(constructor)
    channels = [int(c) for c in constructor["num_channels"]]
    cond_channels = [int(c) for c in constructor["conditioning_embedding_num_channels"]]
    scale = 2 ** (len(cond_channels) - 1)
    if conditioning_embedding is None:
        _require_ncdhw(cond, "controlnet cond")
        expected = tuple(int(d) * scale for d in x.shape[2:])
        if tuple(int(d) for d in cond.shape[2:]) != expected:
            raise ValueError(f"controlnet cond spatial {tuple(cond.shape[2:])} must be {scale}x latent {tuple(x.shape[2:])}")
    else:
        expected = (int(x.shape[0]), channels[0], *(int(d) for d in x.shape[2:]))
        if tuple(conditioning_embedding.shape) != expected:
            raise ValueError(f"controlnet conditioning embedding shape {tuple(conditioning_embedding.shape)} "
                             f"must be {expected}")
    _, emb = condition_embedding(timesteps, class_labels, None, weights, constructor, with_spacing=False)
    embed = _cond_embed(cond, weights, cond_channels) if conditioning_embedding is None else conditioning_embedding
    # conv_in + the condition embedding, added in the conv epilogue.
    hidden = ops.conv3d(ops.to_ndhwc(x, A.activation_dtype()), A._pack(required_weight(weights, "conv_in.conv.weight")),
                        required_weight(weights, "conv_in.conv.bias"), residual=ops.to_ndhwc(embed),
                        out_dtype=A.activation_dtype())
    emb = A.TimeBiasTable(emb, weights)
    hidden, skips = apply_down_blocks(hidden, emb, weights, constructor)
    hidden = apply_mid_block(hidden, emb, weights, constructor)
    down = [_zero_conv(s, weights, f"controlnet_down_blocks.{i}") for i, s in enumerate(skips)]
    mid = _zero_conv(hidden, weights, "controlnet_mid_block")
    if conditioning_scale != 1.0:
        down = [d * conditioning_scale for d in down]
        mid = mid * conditioning_scale
    return down, mid


# ---------------------------------------------------------------- VAE decoder
def _vae_conv_weights(weights: Weights, prefix: str) -> tuple[torch.Tensor, torch.Tensor]:
    """``vae._conv_weights`` (``vae.py:527-537``)."""
    for key in (f"{prefix}.conv.conv", f"{prefix}.conv"):
        if f"{key}.weight" in weights:
            if f"{key}.bias" not in weights:
                raise ValueError(f"VAE weights missing: {key}.bias")
            return weights[f"{key}.weight"], weights[f"{key}.bias"]
    raise ValueError(f"VAE weights missing: {prefix}.conv.conv.weight or {prefix}.conv.weight")


def _need(weights: Weights, key: str) -> torch.Tensor:
    if key not in weights:
        raise ValueError(f"VAE weights missing: {key}")
    return weights[key]


def run_vae_decoder_ncdhw(array, weights: Weights, *, constructor: Mapping, mx=None) -> torch.Tensor:
    """Decoder of ``AutoencoderKlMaisi`` (``vae.py:273-379``, fast path)."""
    channels = [int(c) for c in constructor["num_channels"]]
    res_blocks = [int(c) for c in constructor["num_res_blocks"]]
    if any(bool(a) for a in constructor["attention_levels"]):
        raise ValueError("image VAE dest has no attention blocks")
    if bool(constructor.get("use_convtranspose")):
        raise ValueError("the B200 VAE decoder implements the trilinear upsampling path")
    g, eps = int(constructor["norm_num_groups"]), float(constructor["norm_eps"])
    hidden = A.conv3d_ncdhw(array, *_vae_conv_weights(weights, "decoder.blocks.0"), padding=1)
    index = 1
    rev_ch, rev_res = list(reversed(channels)), list(reversed(res_blocks))
    for level in range(len(rev_ch)):
        for _ in range(rev_res[level]):
            prefix = f"decoder.blocks.{index}"
            has_short = any(f"{prefix}.nin_shortcut.{k}.weight" in weights for k in ("conv.conv", "conv"))
            state = [hidden]
            del hidden
            hidden = A.vae_resblock_ncdhw(
                state, _vae_conv_weights(weights, f"{prefix}.conv1"), _vae_conv_weights(weights, f"{prefix}.conv2"),
                (_need(weights, f"{prefix}.norm1.weight"), _need(weights, f"{prefix}.norm1.bias")),
                (_need(weights, f"{prefix}.norm2.weight"), _need(weights, f"{prefix}.norm2.bias")),
                _vae_conv_weights(weights, f"{prefix}.nin_shortcut") if has_short else None,
                num_groups=g, eps=eps)
            index += 1
        if level != len(rev_ch) - 1:
            w = _need(weights, f"decoder.blocks.{index}.conv.conv.conv.weight")
            b = _need(weights, f"decoder.blocks.{index}.conv.conv.conv.bias")
            hidden = A.trilinear_conv3d_ncdhw(hidden, w, b)
            index += 1
    norm = (_need(weights, f"decoder.blocks.{index}.weight"), _need(weights, f"decoder.blocks.{index}.bias"))
    return A.norm_conv3d_ncdhw(hidden, *_vae_conv_weights(weights, f"decoder.blocks.{index + 1}"), norm=norm,
                               num_groups=g, eps=eps, apply_silu=False)


def decode_vae_ncdhw(latent, weights: Weights, *, constructor: Mapping, mx=None):
    """``post_quant_conv`` then the decoder; returns ``(post_quant, decoded)`` (``vae.py:29-62``)."""
    _require_ncdhw(latent, "vae latent")
    if bool(constructor.get("with_encoder_nonlocal_attn")) or bool(constructor.get("with_decoder_nonlocal_attn")):
        raise ValueError("image VAE dest has no nonlocal attention")
    x = ops.to_ndhwc(latent, A.activation_dtype())
    post = A.conv3d_ncdhw(x, *_vae_conv_weights(weights, "post_quant_conv"), padding=0)
    return post, run_vae_decoder_ncdhw(post, weights, constructor=constructor)
