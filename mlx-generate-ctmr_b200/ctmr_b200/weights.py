"""Parameter inventories of the MAISI networks and their random initialisation.

The shape builders walk each architecture the way its forward pass does (the
channel bookkeeping of the reference's ``unet.py:274-487``, ``controlnet.py``
and ``vae.py:273-379``) and list Torch-layout parameter names and shapes; a CPU
test checks them against the reference's production catalog and the recorded
fixtures' weight recipes. ``random_weights`` fills them the way a freshly
constructed torch module is (Kaiming-uniform with a = sqrt(5) for conv/linear
weights, U(+-1/sqrt(fan_in)) biases, GroupNorm gamma 1 / beta 0, N(0, 1)
embeddings), with ControlNet's zero convolutions at zero as MONAI creates them.
No checkpoint is needed; the benchmark runs on these.
"""

from __future__ import annotations

import math
from collections.abc import Mapping

import torch

Shapes = dict[str, tuple[int, ...]]


def _per_level(value, n: int) -> tuple[int, ...]:
    return tuple(int(v) for v in value) if isinstance(value, (list, tuple)) else (int(value),) * n


class _Builder:
    def __init__(self) -> None:
        self.shapes: Shapes = {}

    def conv(self, name: str, o: int, i: int, k: int) -> None:
        self.shapes[f"{name}.weight"] = (o, i, k, k, k)
        self.shapes[f"{name}.bias"] = (o,)

    def lin(self, name: str, o: int, i: int) -> None:
        self.shapes[f"{name}.weight"] = (o, i)
        self.shapes[f"{name}.bias"] = (o,)

    def norm(self, name: str, c: int) -> None:
        self.shapes[f"{name}.weight"] = (c,)
        self.shapes[f"{name}.bias"] = (c,)

    def resblock(self, name: str, cin: int, cout: int, emb_dim: int) -> None:
        self.norm(f"{name}.norm1", cin)
        self.conv(f"{name}.conv1.conv", cout, cin, 3)
        self.lin(f"{name}.time_emb_proj", cout, emb_dim)
        self.norm(f"{name}.norm2", cout)
        self.conv(f"{name}.conv2.conv", cout, cout, 3)
        if cin != cout:
            self.conv(f"{name}.skip_connection.conv", cout, cin, 1)

    def attention(self, name: str, c: int) -> None:
        self.norm(f"{name}.norm", c)
        for proj in ("to_q", "to_k", "to_v", "out_proj"):
            self.lin(f"{name}.attn.{proj}", c, c)


def _encoder(b: _Builder, ctor: Mapping, emb_dim: int) -> list[int]:
    """conv_in + down blocks + mid block; returns the skip channel list."""
    ch = [int(c) for c in ctor["num_channels"]]
    n = len(ch)
    res = _per_level(ctor["num_res_blocks"], n)
    attn = list(ctor["attention_levels"])
    b.conv("conv_in.conv", ch[0], int(ctor["in_channels"]), 3)
    skips = [ch[0]]
    cur = ch[0]
    for i in range(n):
        for r in range(res[i]):
            b.resblock(f"down_blocks.{i}.resnets.{r}", cur, ch[i], emb_dim)
            cur = ch[i]
            if attn[i]:
                b.attention(f"down_blocks.{i}.attentions.{r}", cur)
            skips.append(cur)
        if i != n - 1:
            b.resblock(f"down_blocks.{i}.downsampler", cur, cur, emb_dim)
            skips.append(cur)
    b.resblock("middle_block.resnet_1", cur, cur, emb_dim)
    b.attention("middle_block.attention", cur)
    b.resblock("middle_block.resnet_2", cur, cur, emb_dim)
    return skips


def _embeddings(b: _Builder, ctor: Mapping, spacing: bool) -> int:
    c0 = int(ctor["num_channels"][0])
    ted = 4 * c0
    b.lin("time_embed.0", ted, c0)
    b.lin("time_embed.2", ted, ted)
    if ctor.get("num_class_embeds") is not None:
        b.shapes["class_embedding.weight"] = (int(ctor["num_class_embeds"]), ted)
    if spacing and ctor.get("include_spacing_input"):
        b.lin("spacing_layer.0", ted, 3)
        b.lin("spacing_layer.2", ted, ted)
        return 2 * ted
    return ted


def unet_shapes(ctor: Mapping) -> Shapes:
    """``DiffusionModelUNetMaisi`` parameters (rflow, resblock_updown)."""
    b = _Builder()
    b.conv("conv_in.conv", int(ctor["num_channels"][0]), int(ctor["in_channels"]), 3)
    emb_dim = _embeddings(b, ctor, spacing=True)
    skips = _encoder(b, ctor, emb_dim)
    ch = [int(c) for c in ctor["num_channels"]]
    n = len(ch)
    res = _per_level(ctor["num_res_blocks"], n)
    attn = list(ctor["attention_levels"])
    cur = ch[-1]
    for i in range(n):
        lvl = n - 1 - i
        for r in range(res[lvl] + 1):
            s = skips.pop()
            b.resblock(f"up_blocks.{i}.resnets.{r}", cur + s, ch[lvl], emb_dim)
            cur = ch[lvl]
            if attn[lvl]:
                b.attention(f"up_blocks.{i}.attentions.{r}", cur)
        if i != n - 1:
            b.resblock(f"up_blocks.{i}.upsampler", cur, cur, emb_dim)
    b.norm("out.0", cur)
    b.conv("out.2.conv", int(ctor["out_channels"]), cur, 3)
    return b.shapes


def controlnet_shapes(ctor: Mapping) -> Shapes:
    """``ControlNetMaisi`` parameters."""
    b = _Builder()
    b.conv("conv_in.conv", int(ctor["num_channels"][0]), int(ctor["in_channels"]), 3)
    emb_dim = _embeddings(b, ctor, spacing=False)
    cc = [int(c) for c in ctor["conditioning_embedding_num_channels"]]
    p = "controlnet_cond_embedding"
    b.conv(f"{p}.conv_in.conv", cc[0], int(ctor["conditioning_embedding_in_channels"]), 3)
    for j in range(len(cc) - 1):
        b.conv(f"{p}.blocks.{2 * j}.conv", cc[j], cc[j], 3)
        b.conv(f"{p}.blocks.{2 * j + 1}.conv", cc[j + 1], cc[j], 3)
    b.conv(f"{p}.conv_out.conv", int(ctor["num_channels"][0]), cc[-1], 3)
    skips = _encoder(b, ctor, emb_dim)
    for k, s in enumerate(skips):
        b.conv(f"controlnet_down_blocks.{k}" + ("" if k == 0 else ".conv"), s, s, 1)
    last = int(ctor["num_channels"][-1])
    b.conv("controlnet_mid_block.conv", last, last, 1)
    return b.shapes


def vae_decoder_shapes(ctor: Mapping) -> Shapes:
    """``AutoencoderKlMaisi`` decode-path parameters (post_quant_conv + decoder)."""
    b = _Builder()
    latent = int(ctor["latent_channels"])
    ch = list(reversed([int(c) for c in ctor["num_channels"]]))
    res = list(reversed([int(c) for c in ctor["num_res_blocks"]]))
    b.conv("post_quant_conv.conv", latent, latent, 1)
    b.conv("decoder.blocks.0.conv.conv", ch[0], latent, 3)
    idx, cur = 1, ch[0]
    for level in range(len(ch)):
        for _ in range(res[level]):
            p = f"decoder.blocks.{idx}"
            b.norm(f"{p}.norm1", cur)
            b.conv(f"{p}.conv1.conv.conv", ch[level], cur, 3)
            b.norm(f"{p}.norm2", ch[level])
            b.conv(f"{p}.conv2.conv.conv", ch[level], ch[level], 3)
            if cur != ch[level]:
                b.conv(f"{p}.nin_shortcut.conv.conv", ch[level], cur, 1)
            cur = ch[level]
            idx += 1
        if level != len(ch) - 1:
            b.conv(f"decoder.blocks.{idx}.conv.conv.conv", cur, cur, 3)
            idx += 1
    b.norm(f"decoder.blocks.{idx}", cur)
    b.conv(f"decoder.blocks.{idx + 1}.conv.conv", int(ctor["out_channels"]), cur, 3)
    return b.shapes


def random_weights(shapes: Shapes, *, seed: int, device="cuda", zero_prefixes: tuple[str, ...] = ()
                   ) -> dict[str, torch.Tensor]:
    """Fresh-module initialisation of ``shapes`` (fp32, on ``device``), reproducible from ``seed``."""
    gen = torch.Generator(device="cpu").manual_seed(int(seed))
    out: dict[str, torch.Tensor] = {}
    for name, shape in shapes.items():
        if any(name.startswith(p) for p in zero_prefixes):
            t = torch.zeros(shape)
        elif name.endswith("embedding.weight"):
            t = torch.randn(shape, generator=gen)
        elif len(shape) == 1 and (".norm" in name or name.startswith("out.0") or _is_gn(name, shapes)):
            t = torch.ones(shape) if name.endswith("weight") else torch.zeros(shape)
        elif name.endswith("weight"):
            fan_in = math.prod(shape[1:])
            bound = 1.0 / math.sqrt(fan_in)  # kaiming_uniform(a=sqrt(5)) bound = sqrt(6 / ((1 + 5) fan_in))
            t = torch.empty(shape).uniform_(-bound, bound, generator=gen)
        else:
            wshape = shapes[name[: -len("bias")] + "weight"]
            bound = 1.0 / math.sqrt(math.prod(wshape[1:]))
            t = torch.empty(shape).uniform_(-bound, bound, generator=gen)
        out[name] = t.to(device)
    return out


def _is_gn(name: str, shapes: Shapes) -> bool:
    """A 1-D parameter whose layer has no 2-D+ weight is a GroupNorm affine (e.g. the VAE's final norm)."""
    stem = name.rsplit(".", 1)[0]
    w = shapes.get(f"{stem}.weight")
    return w is not None and len(w) == 1


# ---------------------------------------------------------------- released checkpoints
def disk_shape(torch_shape: tuple[int, ...]) -> tuple[int, ...]:
    """Stored shape of a parameter: convolution weights channels-last ``(O, k, k, k, I)``
    (the reference's ``LAYOUT_CONV3D_W``, ``maisi_mlx_weights.py:123-133``), everything else
    as in Torch."""
    if len(torch_shape) == 5:
        o, i, kd, kh, kw = torch_shape
        return (o, kd, kh, kw, i)
    return tuple(torch_shape)


def load_network_file(path, network: str, shapes: Shapes, *, device=None
                      ) -> tuple[dict[str, torch.Tensor], float | None]:
    """Load one network from a native ``.safetensors`` checkpoint (``weights.py:102-166``).

    ``shapes`` is the network's Torch-layout inventory (``unet_shapes``,
    ``controlnet_shapes``, ``vae_decoder_shapes``). A file named
    ``model.safetensors`` holds every network under ``<network>.``-prefixed keys;
    any other file holds one network unprefixed. Every tensor must be listed,
    finite float32 in its stored layout; the UNet file carries the latent
    ``scale_factor``, the others must not. Returns ``(weights, scale_factor)``:
    convolution weights are Torch-layout views ``(O, I, k, k, k)`` of the
    channels-last storage (no transposed copy; ``ops.pack_weight`` packs such a
    view from its storage), on ``device`` when given. Raises ``ValueError`` as the
    reference raises ``InvalidInputError``.
    """
    from pathlib import Path

    from safetensors import safe_open

    path = Path(path)
    if path.suffix != ".safetensors":
        raise ValueError(f"{path.name} must be a safetensors file")
    prefix = network + "." if path.name == "model.safetensors" else ""
    weights: dict[str, torch.Tensor] = {}
    scale_factor = None
    with safe_open(str(path), framework="pt") as f:
        selected = {k.removeprefix(prefix): k for k in f.keys() if k.startswith(prefix)}
        for name in selected:
            if name != "scale_factor" and name not in shapes:
                raise ValueError(f"{path.name} has unexpected tensor {name}")
        missing = [name for name in shapes if name not in selected]
        if missing:
            raise ValueError(f"{path.name} is missing {missing[0]}")
        if network == "unet":
            if "scale_factor" not in selected:
                raise ValueError(f"{path.name} is missing scale_factor")
            scale = f.get_tensor(selected["scale_factor"])
            if scale.numel() != 1 or not torch.isfinite(scale).all() or float(scale.reshape(())) <= 0.0:
                raise ValueError(f"{path.name} scale_factor must be one finite positive value")
            scale_factor = float(scale.reshape(()))
        elif "scale_factor" in selected:
            raise ValueError(f"{path.name} must not contain scale_factor")
        for name, stored in selected.items():
            if name == "scale_factor":
                continue
            t = f.get_tensor(stored)
            expected = disk_shape(shapes[name])
            if tuple(t.shape) != expected or t.dtype != torch.float32 or not torch.isfinite(t).all():
                raise ValueError(f"{path.name} tensor {name} must be finite float32 with shape {expected}; "
                                 f"got {t.dtype} {tuple(t.shape)}")
            if device is not None:
                t = t.to(device)
            weights[name] = t.permute(0, 4, 1, 2, 3) if t.dim() == 5 else t
    return weights, scale_factor


def save_network_file(path, network: str, weights: Mapping[str, torch.Tensor], *,
                      scale_factor: float | None = None) -> None:
    """Write Torch-layout ``weights`` as a native checkpoint (the inverse of
    ``load_network_file``): convolution weights channels-last, float32."""
    from pathlib import Path

    from safetensors.torch import save_file

    path = Path(path)
    prefix = network + "." if path.name == "model.safetensors" else ""
    out = {}
    for name, t in weights.items():
        t = t.detach().to("cpu", torch.float32)
        out[prefix + name] = (t.permute(0, 2, 3, 4, 1) if t.dim() == 5 else t).contiguous()
    if scale_factor is not None:
        out[prefix + "scale_factor"] = torch.tensor(float(scale_factor), dtype=torch.float32)
    save_file(out, str(path))
