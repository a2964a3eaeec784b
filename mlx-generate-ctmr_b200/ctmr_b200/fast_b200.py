"""Drop-in arithmetic module: the operator surface of the reference's ``fast_fp32``
(``fast_fp32.py:1-406``; protocols ``_types.py:216-286``) on torch CUDA tensors,
executed by ``libctmr_b200`` (sm_100a).

Tensors keep the reference's logical NCDHW shape and are stored channels-last
(``torch.channels_last_3d``, i.e. NDHWC rows), so no pack pass is needed: the
convolution's TMA loads read the activations in place and zero-fill padding.

Precision (request-scoped, like the reference's ``arithmetic_mode``):
  ``"fp32"`` (default) — convolutions in the split-fp16 "exact" mode (fp32
      accumulation, ~2^-22 relative product error), the reference's default
      arithmetic.
  ``"tf32"`` — TF32 tensor-core operands (fp32 range, 10 mantissa bits) with
      fp32 accumulation and epilogue, at half the 16-bit rate; dense ops in fp32.
  ``"bf16"`` / ``"fp16"`` — bf16 or fp16 tensor-core operands with fp32
      accumulation and fp32 epilogue additions (same tensor-core rate; fp16
      carries 3 more mantissa bits and needs |value| < 65504, like the split
      mode's hi plane). The small dense ops (attention, Q/K/V projections) run
      in the same 16-bit type with fp32 accumulation.
Activations between layers are stored in fp32 in both modes: the conv-input
preparation pass (which applies the group norm and SiLU anyway) writes the
bf16 or split-fp16 operand, so a bf16 operand costs no extra pass, and the
residual stream never accumulates bf16 storage rounding.

The fused entry points (``residual_block_ncdhw``, ``vae_resblock_ncdhw``,
``norm_conv3d_ncdhw``, ``trilinear_conv3d_ncdhw``) follow ``fast_fp32`` exactly in
where normalisation, SiLU, the time embedding, the skip and the upsampling
happen. There is no CPU or alternative backend: every convolution, group norm
and elementwise transform runs in the CUDA library, and the small dense ops the
reference also leaves to its framework (embedding MLPs, Q/K/V projections,
attention) run in torch's CUDA kernels.
"""

from __future__ import annotations

import contextlib
import math
import os
import weakref
from collections.abc import Generator, Iterable, Mapping
from contextvars import ContextVar
from dataclasses import dataclass

import torch
import torch.nn.functional as F

from . import _lib, ops

_precision: ContextVar[str] = ContextVar("ctmr_b200_precision", default="fp32")


@contextlib.contextmanager
def arithmetic_precision(precision: str) -> Generator[None]:
    """Select ``"fp32"``, ``"tf32"``, ``"bf16"`` or ``"fp16"`` for calls made inside the block (restored on exit)."""
    if precision not in ops.PRECISIONS:
        raise ValueError(f"precision must be one of {ops.PRECISIONS}; got {precision!r}")
    token = _precision.set(precision)
    try:
        yield
    finally:
        _precision.reset(token)


def active_precision() -> str:
    return _precision.get()


def activation_dtype() -> torch.dtype:
    """Storage dtype of activations between layers (fp32 in both precisions)."""
    return torch.float32


@dataclass(frozen=True)
class ChannelConcat:
    """``concat(first, second)`` along channels, never materialised.

    The UNet up path concatenates the running hidden state with a stored skip
    before every ResBlock (``unet.py:444``); the group-norm statistics, the
    input preparation and the 1x1x1 skip projection read both tensors directly.
    """

    first: torch.Tensor
    second: torch.Tensor

    @property
    def shape(self) -> tuple[int, ...]:
        b, c1, d, h, w = self.first.shape
        return (int(b), int(c1) + int(self.second.shape[1]), int(d), int(h), int(w))

    def materialize(self) -> torch.Tensor:
        return ops.transform(self.first, x2=self.second, out_dtype=self.first.dtype)


def concat_channels_ncdhw(first: torch.Tensor, second: torch.Tensor, mx=None) -> ChannelConcat:
    """Lazy channel concat (``medmlx_core.ops.concat_channels_ncdhw``'s role)."""
    if tuple(first.shape[2:]) != tuple(second.shape[2:]) or first.shape[0] != second.shape[0]:
        raise ValueError(f"cannot concat {tuple(first.shape)} and {tuple(second.shape)}")
    return ChannelConcat(ops.to_ndhwc(first, activation_dtype()), ops.to_ndhwc(second, activation_dtype()))


def _split(x) -> tuple[torch.Tensor, torch.Tensor | None]:
    if isinstance(x, ChannelConcat):
        return x.first, x.second
    return ops.to_ndhwc(x, activation_dtype()), None


# ---------------------------------------------------------------- packed weights
# Keyed by (id(weight), upsample, precision); the weak reference both validates
# that the id still names the same tensor and evicts on collection
# (``fast_fp32.py:70-90``).
_packed: dict[tuple[int, bool, str], tuple[weakref.ref, ops.PackedWeight]] = {}


NARROW_CHANNELS = 16


def conv_precision(weight: torch.Tensor) -> str:
    """Operand precision of one convolution under the active mode.

    In the bf16 mode the narrow input and output convolutions (at most 16
    channels on either side: the latent-facing conv_in / post_quant_conv and the
    4- or 1-channel output convs) keep the split-fp32 operands: with bf16's 8-bit
    significand the output conv otherwise dominates the decoded volume's error
    budget. fp16's 11-bit significand keeps them within it, so the fp16 mode runs
    them on the tensor cores like every other layer.
    """
    precision = _precision.get()
    if precision == "bf16" and min(int(weight.shape[0]), int(weight.shape[1])) <= NARROW_CHANNELS:
        return "fp32"
    return precision


_dense: dict[tuple[int, torch.dtype], tuple[weakref.ref, torch.Tensor]] = {}


def _dense_weight(weight: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """``weight`` in ``dtype``, cast once and cached like the packed conv weights."""
    if weight.dtype == dtype:
        return weight
    key = (id(weight), dtype)
    hit = _dense.get(key)
    if hit is not None and hit[0]() is weight:
        return hit[1]
    cast = weight.detach().to(dtype)
    _dense[key] = (weakref.ref(weight, lambda _: _dense.pop(key, None)), cast)
    return cast


# Whether a GroupNorm-feeding convolution reduces its output statistics in the epilogue
# (ops.conv3d(stats=True)) instead of the GroupNorm pass re-reading the tensor. By default
# only for outputs larger than L2 (the VAE decoder's full- and mid-resolution tensors), where
# that pass reads HBM; an L2-resident tensor (the UNet's) is read back cheaper than the
# epilogue reduction costs. CTMR_OUTPUT_STATS=1: every such convolution; 0: none.
OUTPUT_STATS = os.environ.get("CTMR_OUTPUT_STATS", "auto")
STATS_MIN_BYTES = 128 << 20


def _want_stats(x: torch.Tensor, out_channels: int, scale: float = 1.0) -> bool:
    """Epilogue statistics for a conv of ``x`` into ``out_channels`` on ``scale`` x its voxel count."""
    if OUTPUT_STATS in ("0", "1"):
        return OUTPUT_STATS == "1"
    b, _, d, h, w = (int(n) for n in x.shape)
    itemsize = torch.empty((), dtype=activation_dtype()).element_size()
    return b * d * h * w * scale * out_channels * itemsize > STATS_MIN_BYTES

_stacked: dict[tuple, tuple] = {}


def _stacked_dense(tensors: tuple[torch.Tensor, ...], dtype: torch.dtype) -> torch.Tensor:
    """``cat(tensors)`` in ``dtype`` (the Q/K/V projections as one), cached while the sources live."""
    key = (tuple(id(t) for t in tensors), dtype)
    hit = _stacked.get(key)
    if hit is not None and all(r() is t for r, t in zip(hit[0], tensors, strict=True)):
        return hit[1]
    out = torch.cat([t.detach().to(dtype) for t in tensors]).contiguous()
    _stacked[key] = (tuple(weakref.ref(t, lambda _: _stacked.pop(key, None)) for t in tensors), out)
    return out


def dense_dtype() -> torch.dtype:
    """Operand type of the dense (non-conv) tensor-core ops: fp32, or the 16-bit mode's type."""
    return {"fp32": torch.float32, "tf32": torch.float32, "bf16": torch.bfloat16,
            "fp16": torch.float16}[_precision.get()]


# At or above this many output voxels a <= 4-output-channel conv runs faster on the
# direct fp32 kernel than as an N = 16 tensor-core GEMM (measured: the VAE decoder's
# 64 -> 1 conv on 96 x 256 x 128 voxels, 0.71 ms vs 1.24 ms with its operand pass;
# the UNet's 64 -> 4 on 2 x 64 x 64 x 32 voxels prefers the GEMM, 0.11 vs 0.22 ms).
NARROW_DIRECT_VOXELS = 1 << 21


def _pack(weight: torch.Tensor, *, upsample: bool = False, out_voxels: int = 0) -> ops.PackedWeight:
    precision = conv_precision(weight)
    if precision in ("fp16", "tf32") and int(weight.shape[0]) <= 4 and out_voxels >= NARROW_DIRECT_VOXELS:
        precision = "fp32"
    key = (id(weight), upsample, precision)
    hit = _packed.get(key)
    if hit is not None and hit[0]() is weight:
        return hit[1]
    packed = ops.pack_weight(weight, precision, upsample=upsample)
    _packed[key] = (weakref.ref(weight, lambda _: _packed.pop(key, None)), packed)
    return packed


def drop_packed_weights(weights: Iterable[torch.Tensor]) -> None:
    """Forget the packed copies of ``weights``; a later use packs them again."""
    ids = {id(w) for w in weights}
    for key in [k for k in _packed if k[0] in ids]:
        del _packed[key]
    for key in [k for k in _dense if k[0] in ids]:
        del _dense[key]


# ---------------------------------------------------------------- elementwise surface
def silu(array, mx=None) -> torch.Tensor:
    """SiLU ``y / (1 + exp(-y))`` on activations, or torch's on small dense tensors."""
    if isinstance(array, torch.Tensor) and array.dim() != 5:
        return F.silu(array)
    x, x2 = _split(array)
    return ops.transform(x, x2=x2, silu=True, out_dtype=activation_dtype())


def linear(array: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None, mx=None) -> torch.Tensor:
    """Dense projection of small tensors (embeddings, attention tokens) in fp32 or the activation dtype."""
    dtype = array.dtype if array.dtype in (torch.float32, torch.bfloat16) else torch.float32
    return F.linear(array.to(dtype), weight.to(dtype), None if bias is None else bias.to(dtype))


def group_norm_ncdhw(array, weight, bias, *, num_groups: int, eps: float, mx=None, apply_silu: bool = False,
                     out_dtype: torch.dtype | None = None):
    """Group norm with fp32 statistics and an optional fused SiLU (``fast_fp32.py:102-118``).

    ``out_dtype`` (default: the activation dtype) may also be fp16, for a result that
    only feeds 16-bit dense operands (the attention tokens)."""
    x, x2 = _split(array)
    affine = ops.group_norm_affine(x, weight, bias, groups=num_groups, eps=eps, x2=x2)
    return ops.transform(x, x2=x2, affine=affine, silu=apply_silu, out_dtype=out_dtype or activation_dtype())


def avg_pool3d_ncdhw(array, *, mx=None) -> torch.Tensor:
    x, x2 = _split(array)
    return ops.transform(x, x2=x2, mode=_lib.TRANSFORM_AVGPOOL, out_dtype=activation_dtype())


def upsample_nearest_ncdhw(array, *, mx=None) -> torch.Tensor:
    x, _ = _split(array)
    return x.repeat_interleave(2, 2).repeat_interleave(2, 3).repeat_interleave(2, 4).contiguous(
        memory_format=torch.channels_last_3d)


def upsample_trilinear_ncdhw(array, *, mx=None, scale: int = 2) -> torch.Tensor:
    """Half-pixel trilinear 2x (``source_vae.py:95-111``)."""
    if scale != 2:
        raise ValueError("NV-Generate VAE trilinear upsampling requires scale=2")
    x, x2 = _split(array)
    return ops.transform(x, x2=x2, mode=_lib.TRANSFORM_TRILINEAR, out_dtype=activation_dtype())


def sinusoidal_timestep_embedding(timesteps: torch.Tensor, embedding_dim: int, *, mx=None,
                                  max_period: int = 10000) -> torch.Tensor:
    """``[cos, sin]`` timestep features (``embed.py:15-42``), fp32."""
    if timesteps.dim() != 1:
        raise ValueError("Timesteps should be a 1d-array")
    half = embedding_dim // 2
    exponent = -math.log(max_period) * torch.arange(half, dtype=torch.float32, device=timesteps.device)
    freqs = torch.exp(exponent / half)
    args = timesteps.to(torch.float32).reshape(-1, 1) * freqs.reshape(1, -1)
    emb = torch.cat([torch.cos(args), torch.sin(args)], dim=-1)
    if embedding_dim % 2 == 1:
        emb = F.pad(emb, (0, 1))
    return emb


# ---------------------------------------------------------------- convolutions
def _norm_args(x, x2, weight, bias, *, groups: int, eps: float) -> dict:
    """Keyword arguments that GroupNorm ``x ++ x2`` for the conv consuming it.

    From the producing convolutions' epilogue statistics when they are attached
    (the opt-in path), else inside the conv call itself (``norm=``): one fused
    kernel for small tensors, the statistics pass + operand pass for large ones.
    """
    if ops.output_stats(x) is not None and (x2 is None or ops.output_stats(x2) is not None):
        return {"affine": ops.group_norm_affine(x, weight, bias, groups=groups, eps=eps, x2=x2)}
    return {"norm": (weight, bias, groups, eps)}


def _bias(weight: torch.Tensor, bias: torch.Tensor | None) -> torch.Tensor:
    return torch.zeros(int(weight.shape[0]), dtype=torch.float32, device=weight.device) if bias is None else bias


def pointwise_conv_ncdhw(array, weight: torch.Tensor, bias: torch.Tensor | None, *, mx=None) -> torch.Tensor:
    """1x1x1 convolution as an implicit GEMM with one tap (``fast_fp32.py:121-130``)."""
    x, x2 = _split(array)
    return ops.conv3d(x, _pack(weight), bias, x2=x2, out_dtype=activation_dtype())


def conv3d_ncdhw(array, weight: torch.Tensor, bias: torch.Tensor | None, *, padding: int, mx=None,
                 stride: int = 1) -> torch.Tensor:
    """NCDHW convolution with a Torch ``(O, C, K, K, K)`` weight (``fast_fp32.py:133-154``)."""
    k = int(weight.shape[2])
    if k == 1 and padding == 0 and stride == 1:
        return pointwise_conv_ncdhw(array, weight, bias)
    if k != 3 or padding != 1 or stride not in (1, 2):
        raise ValueError(f"unsupported convolution: kernel {k}, padding {padding}, stride {stride}")
    x, x2 = _split(array)
    return ops.conv3d(x, _pack(weight), bias, x2=x2, stride=stride, out_dtype=activation_dtype(),
                      stats=_want_stats(x, int(weight.shape[0]), 1.0 / 8 if stride == 2 else 1.0))


def norm_conv3d_ncdhw(array, weight: torch.Tensor, bias: torch.Tensor, *, norm, num_groups: int, eps: float,
                      apply_silu: bool, mx=None, upsample: bool = False, residual=None,
                      residual_upsampled: bool = False, avgpool: bool = False) -> torch.Tensor:
    """``conv(upsample?(silu?(norm?(x)))) + bias (+ residual)`` for padding-1 3x3x3 kernels (``fast_fp32.py:162-211``).

    ``bias`` is ``(O,)`` or per batch item ``(B, O)``. ``residual_upsampled`` reads
    the residual on the half-resolution grid (nearest 2x), ``avgpool`` convolves
    the 2x2x2 mean of the prepared input; both are this module's fusions of the
    surrounding ops in ``fast_fp32.residual_block_ncdhw``.
    """
    x, x2 = _split(array)
    nargs = {}
    if norm is not None:
        nargs = _norm_args(x, x2, norm[0], norm[1], groups=num_groups, eps=eps)
    res = None
    if residual is not None:
        res = residual if isinstance(residual, torch.Tensor) else residual.materialize()
        res = ops.to_ndhwc(res)
    b, _, d, h, w = (int(n) for n in x.shape)
    scale = 8 if upsample else 1
    voxels = b * d * h * w * scale // (8 if avgpool else 1)
    return ops.conv3d(x, _pack(weight, upsample=upsample, out_voxels=voxels), bias, x2=x2, **nargs,
                      silu=apply_silu,
                      avgpool=avgpool, residual=res, residual_upsampled=residual_upsampled,
                      out_dtype=activation_dtype(),
                      stats=_want_stats(x, int(weight.shape[0]), (8.0 if upsample else 1.0) / (8 if avgpool else 1)))


def trilinear_conv3d_ncdhw(array, weight: torch.Tensor, bias: torch.Tensor, *, mx=None) -> torch.Tensor:
    """Padding-1 3x3x3 conv of the half-pixel trilinear 2x upsampling, computed while preparing the operand."""
    x, x2 = _split(array)
    if x2 is not None:
        x = ChannelConcat(x, x2).materialize()
    return ops.conv3d(x, _pack(weight), bias, trilinear=True, out_dtype=activation_dtype(),
                      stats=_want_stats(x, int(weight.shape[0]), 8.0))


_TIME_TABLES: dict[tuple, tuple[torch.Tensor, torch.Tensor, torch.Tensor, list[tuple[int, int, int]]]] = {}


class TimeBiasTable:
    """Every residual block's ``conv1`` bias + time-embedding projection for one network pass.

    The reference projects ``silu(emb)`` once per block (``residual.py:75``, one
    small GEMV each); here all blocks' ``time_emb_proj`` weights are stacked
    (once per weight set) and projected with one GEMM, and each block takes its
    column slice. ``bias_for(block_weights)`` finds the slice by the block's
    projection tensor. The stacked copy assumes the weights are not modified in
    place, as the packed convolution weights do.
    """

    def __init__(self, emb: torch.Tensor, weights: Mapping[str, torch.Tensor]) -> None:
        names = sorted(k[: -len("time_emb_proj.weight")] for k in weights if k.endswith("time_emb_proj.weight"))
        key = tuple(weights[n + "time_emb_proj.weight"].data_ptr() for n in names)
        if key not in _TIME_TABLES:
            ws = [weights[n + "time_emb_proj.weight"].to(torch.float32) for n in names]
            bs = [weights[n + "time_emb_proj.bias"].to(torch.float32) for n in names]
            cs = [weights[n + "conv1.conv.bias"].to(torch.float32) for n in names]
            spans, start = [], 0
            for n, w in zip(names, ws, strict=True):
                spans.append((weights[n + "time_emb_proj.weight"].data_ptr(), start, start + int(w.shape[0])))
                start += int(w.shape[0])
            _TIME_TABLES[key] = (torch.cat(ws).contiguous(), torch.cat(bs).contiguous(),
                                 torch.cat(cs).reshape(1, -1).contiguous(), spans)
        w_all, b_all, c_all, spans = _TIME_TABLES[key]
        self.emb = emb
        bias = c_all + F.linear(F.silu(emb.to(torch.float32)), w_all, b_all)
        self._by_ptr = {ptr: bias[:, a:b] for ptr, a, b in spans}

    def bias_for(self, weights: Mapping[str, torch.Tensor]) -> torch.Tensor | None:
        w = weights.get("time_emb_proj.weight")
        return None if w is None else self._by_ptr.get(w.data_ptr())


# The UNet ResBlock's skip projection (a 1x1x1 conv of the block input, independent of conv1)
# runs on a second stream beside norm1 -> conv1 -> norm2, joining before conv2 reads it: on the
# deep levels, whose launches each fill a fraction of the SMs, the two chains overlap.
# CTMR_SKIP_SIDE_STREAM=0 keeps it on the caller's stream.
SKIP_SIDE_STREAM = os.environ.get("CTMR_SKIP_SIDE_STREAM", "1") != "0"
# One side stream per (device, parent stream): chains forked from different streams (the UNet's and
# a concurrently running ControlNet's) do not queue behind each other.
_SIDE_STREAMS: dict[tuple[int, int], torch.cuda.Stream] = {}


def side_stream(device: torch.device, parent: torch.cuda.Stream | None = None) -> torch.cuda.Stream:
    """The side stream forked from ``parent`` (default: the current stream) on ``device``."""
    index = device.index if device.index is not None else torch.cuda.current_device()
    parent = parent if parent is not None else torch.cuda.current_stream(index)
    key = (index, int(parent.cuda_stream))
    if key not in _SIDE_STREAMS:
        _SIDE_STREAMS[key] = torch.cuda.Stream(device=index)
    return _SIDE_STREAMS[key]


@contextlib.contextmanager
def beside(device: torch.device) -> Generator[torch.cuda.Stream, None, None]:
    """Runs the enclosed launches on the current stream's side stream, ordered after everything
    queued so far on the current stream; the caller joins with
    ``torch.cuda.current_stream().wait_stream(side)``."""
    parent = torch.cuda.current_stream(device)
    side = side_stream(device, parent)
    side.wait_stream(parent)
    with torch.cuda.stream(side):
        yield side


def residual_block_ncdhw(x, emb: torch.Tensor, weights: Mapping[str, torch.Tensor], *, num_groups: int, eps: float,
                         mx=None, up: bool = False, down: bool = False,
                         time_bias: torch.Tensor | None = None) -> torch.Tensor:
    """Fused UNet ResBlock (``fast_fp32.py:214-291``).

    The time-embedding projection joins conv1's bias per batch item; the skip
    (after its optional 1x1x1 projection, on the small grid) joins conv2's
    accumulator. ``down``: conv1 reads the 2x2x2 mean of ``silu(norm1(x))``
    (pooling after the activation, as the reference). ``up``: conv1 reads the
    nearest-2x upsampling through the folded weights, and the skip stays on the
    small grid and is upsampled by index in conv2's epilogue. ``time_bias``: the
    block's ``conv1`` bias + projected embedding when already computed.
    """
    xa, xb = _split(x)
    if time_bias is not None:  # precomputed by a TimeBiasTable
        bias1 = time_bias
    else:
        temb = linear(F.silu(emb.to(torch.float32)), weights["time_emb_proj.weight"], weights["time_emb_proj.bias"])
        bias1 = weights["conv1.conv.bias"].to(torch.float32).reshape(1, -1) + temb
    norm1 = (weights["norm1.weight"], weights["norm1.bias"])
    cin = int(xa.shape[1]) + (int(xb.shape[1]) if xb is not None else 0)
    project = cin != int(weights["conv1.conv.weight"].shape[0])
    dtype = activation_dtype()
    n1 = _norm_args(xa, xb, *norm1, groups=num_groups, eps=eps)
    side = project and SKIP_SIDE_STREAM and xa.is_cuda
    if project:
        # The projection's output is allocated on the caller's stream (so its lifetime follows that
        # stream) and written on the side stream; its packed weights are made here, not there.
        skip_w = _pack(weights["skip_connection.conv.weight"])
        b_, o_ = int(xa.shape[0]), int(skip_w.out_channels)
        grid = [int(n) // (2 if down else 1) for n in xa.shape[2:]]
        skip = ops.empty_ndhwc(b_, o_, *grid, dtype, xa.device)
        with beside(xa.device) if side else contextlib.nullcontext():
            ops.conv3d(xa, skip_w, weights["skip_connection.conv.bias"], x2=xb, avgpool=down, out=skip)
    if down:
        if not project:
            skip = ops.transform(xa, x2=xb, mode=_lib.TRANSFORM_AVGPOOL, out_dtype=dtype)
        hidden = ops.conv3d(xa, _pack(weights["conv1.conv.weight"]), bias1, x2=xb, **n1, silu=True,
                            avgpool=True, out_dtype=dtype,
                            stats=_want_stats(xa, int(weights["conv1.conv.weight"].shape[0]), 1.0 / 8))
    else:
        if not project:
            skip = xa if xb is None else ChannelConcat(xa, xb).materialize()
        hidden = ops.conv3d(xa, _pack(weights["conv1.conv.weight"], upsample=up), bias1, x2=xb, **n1,
                            silu=True, out_dtype=dtype,
                            stats=_want_stats(xa, int(weights["conv1.conv.weight"].shape[0]), 8.0 if up else 1.0))
    if side:
        torch.cuda.current_stream(xa.device).wait_stream(side_stream(xa.device))
    n2 = _norm_args(hidden, None, weights["norm2.weight"], weights["norm2.bias"], groups=num_groups, eps=eps)
    return ops.conv3d(hidden, _pack(weights["conv2.conv.weight"]), weights["conv2.conv.bias"], **n2,
                      silu=True, residual=skip, residual_upsampled=up, out_dtype=dtype,
                      stats=_want_stats(hidden, int(weights["conv2.conv.weight"].shape[0])))


def vae_resblock_ncdhw(state: list, conv1, conv2, norm1, norm2, shortcut, *, num_groups: int, eps: float,
                       mx=None) -> torch.Tensor:
    """Fused ``MaisiResBlock`` (``fast_fp32.py:294-336``); consumes ``state`` so the input can be freed early."""
    array = state.pop()
    x, x2 = _split(array)
    del array
    dtype = activation_dtype()
    n1 = _norm_args(x, x2, norm1[0], norm1[1], groups=num_groups, eps=eps)
    hidden = ops.conv3d(x, _pack(conv1[0]), conv1[1], x2=x2, **n1, silu=True, out_dtype=dtype,
                        stats=_want_stats(x, int(conv1[0].shape[0])))
    if shortcut is None:
        skip = x if x2 is None else ChannelConcat(x, x2).materialize()
    else:
        skip = ops.conv3d(x, _pack(shortcut[0]), shortcut[1], x2=x2, out_dtype=dtype)
    del x, x2
    n2 = _norm_args(hidden, None, norm2[0], norm2[1], groups=num_groups, eps=eps)
    out = ops.conv3d(hidden, _pack(conv2[0]), conv2[1], **n2, silu=True, residual=skip, out_dtype=dtype,
                     stats=_want_stats(hidden, int(conv2[0].shape[0])))
    return out


# ---------------------------------------------------------------- attention
def attention(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor, *, scale: float, mx=None) -> torch.Tensor:
    """``softmax(Q K^T * scale) V`` on ``(B, H, L, D)`` heads."""
    return F.scaled_dot_product_attention(query, key, value, scale=scale)


def attention_projection(array: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, mx=None) -> torch.Tensor:
    return linear(array, weight, bias)


# Head-size-32 attention on this library's tensor-core kernel (CTMR_TORCH_ATTENTION=1: torch SDPA)
# up to this many tokens. Measured on B200 (fp16, batch 2): 256 tokens x 16 heads 5.8 µs against
# cuDNN SDPA's 6.2 µs; 2048 tokens x 8 heads 34.7 µs against 25.1 µs. At head size 32 the pass is
# bound by the softmax exponentials (16 per clock per SM), where cuDNN's pipeline gets closer.
USE_TCGEN05_ATTENTION = os.environ.get("CTMR_TORCH_ATTENTION") is None
TCGEN05_ATTENTION_MAX_TOKENS = 512


def self_attention_tokens(tokens: torch.Tensor, weights: Mapping[str, torch.Tensor], *, heads: int, scale: float,
                          include_fc: bool, mx=None, prefix: str = "attn", qkv_bias: bool = True) -> torch.Tensor:
    """Q/K/V projections, multi-head self-attention and optional ``out_proj`` on ``(B, L, C)`` (``fast_fp32.py:352-396``)."""
    dt = dense_dtype()
    tokens = tokens.to(dt)
    # One projection GEMM with the Q, K and V weights stacked (same products as three).
    names = ("q", "k", "v")
    w_qkv = _stacked_dense(tuple(weights[f"{prefix}.to_{n}.weight"] for n in names), dt)
    b_qkv = _stacked_dense(tuple(weights[f"{prefix}.to_{n}.bias"] for n in names), dt) if qkv_bias else None
    qkv = F.linear(tokens, w_qkv, b_qkv)
    b, length, c3 = qkv.shape
    c = c3 // 3
    if (dt != torch.float32 and c == 32 * heads and length % 128 == 0 and USE_TCGEN05_ATTENTION
            and length <= TCGEN05_ATTENTION_MAX_TOKENS):
        # Head size 32: the tensor-core flash-attention kernel reads the fused projection directly.
        merged = ops.attention_d32(qkv.contiguous(), heads, scale)
    else:
        q, k, v = qkv.chunk(3, dim=-1)

        def split(a):
            return a.reshape(b, length, heads, c // heads).transpose(1, 2)

        att = F.scaled_dot_product_attention(split(q), split(k), split(v), scale=scale)
        merged = att.transpose(1, 2).reshape(b, length, c)
    if include_fc:
        merged = F.linear(merged, _dense_weight(weights[f"{prefix}.out_proj.weight"], dt),
                          _dense_weight(weights[f"{prefix}.out_proj.bias"], dt))
    return merged


def spatial_attention_ncdhw(x: torch.Tensor, weights: Mapping[str, torch.Tensor], *, num_groups: int, eps: float,
                            num_head_channels: int, include_fc: bool, mx=None) -> torch.Tensor:
    """Residual self-attention over all voxels (``attention.py:92-160`` fast path).

    With channels-last storage the tokens ``(B, D*H*W, C)`` are a view of the
    normalised tensor, and the merged result viewed back is again channels-last.
    """
    x = ops.to_ndhwc(x, activation_dtype())
    b, c, d, h, w = (int(n) for n in x.shape)
    if c % num_head_channels:
        raise ValueError("num_channels must be divisible by num_head_channels")
    heads, scale = c // num_head_channels, float(num_head_channels) ** -0.5
    # The normalised tokens feed only the Q/K/V projection: written directly in its operand dtype.
    normed = group_norm_ncdhw(x, weights["norm.weight"], weights["norm.bias"], num_groups=num_groups, eps=eps,
                              out_dtype=dense_dtype())
    tokens = normed.permute(0, 2, 3, 4, 1).reshape(b, d * h * w, c)
    merged = self_attention_tokens(tokens, weights, heads=heads, scale=scale, include_fc=include_fc)
    out = merged.reshape(b, d, h, w, c).permute(0, 4, 1, 2, 3)
    return torch.add(x, out)  # promotes a 16-bit projection to x's dtype in the same kernel
