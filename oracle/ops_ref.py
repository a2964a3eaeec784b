"""Kernel-level oracle: float64/float32 CPU restatements of the reference's operators.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``). Each function cites the
reference code it restates (paths relative to the reference project root).
"""

from __future__ import annotations

import math

import numpy as np
import torch
import torch.nn.functional as F


def conv3d_ref(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None = None, *, stride: int = 1,
               padding: int | None = None) -> torch.Tensor:
    """Padding-1 (or 0 for 1x1x1) 3-D convolution of NCDHW ``x`` with a Torch-layout weight.

    Restates the float64 reference of ``tests/test_fast_fp32.py:21-38`` (there an
    einsum per tap; here ``F.conv3d`` in the input's dtype, float64 when the
    caller passes float64). ``bias`` may be ``(O,)`` or per batch item ``(B, O)``.
    """
    k = int(w.shape[2])
    pad = (k // 2) if padding is None else padding
    out = F.conv3d(x, w.to(x.dtype), None, stride=stride, padding=pad)
    if bias is not None:
        bias = bias.to(x.dtype)
        out = out + (bias[:, :, None, None, None] if bias.dim() == 2 else bias[None, :, None, None, None])
    return out


def group_norm_ref(x: torch.Tensor, weight: torch.Tensor | None, bias: torch.Tensor | None, groups: int,
                   eps: float) -> torch.Tensor:
    """GroupNorm with biased variance (``tests/test_fast_fp32.py:41-48`` without the SiLU)."""
    b = x.shape[0]
    g = x.reshape(b, groups, -1)
    mean = g.mean(-1, keepdim=True)
    var = ((g - mean) ** 2).mean(-1, keepdim=True)
    y = ((g - mean) / torch.sqrt(var + eps)).reshape(x.shape)
    if weight is not None:
        y = y * weight.to(x.dtype)[None, :, None, None, None]
    if bias is not None:
        y = y + bias.to(x.dtype)[None, :, None, None, None]
    return y


def silu_ref(x: torch.Tensor) -> torch.Tensor:
    """``y / (1 + exp(-y))`` (``_nax_conv.py:177``, ``tests/test_fast_fp32.py:48``)."""
    return x / (1 + torch.exp(-x))


def group_norm_silu_ref(x, weight, bias, groups, eps=1e-6):
    """``tests/test_fast_fp32.py:41-48``."""
    return silu_ref(group_norm_ref(x, weight, bias, groups, eps))


def group_norm_affine_ref(x: torch.Tensor, weight, bias, groups: int, eps: float) -> torch.Tensor:
    """(B, C, 2) (scale, offset) pairs whose affine equals GroupNorm (``_nax_conv.py:174-176`` operand)."""
    b, c = x.shape[:2]
    g = x.double().reshape(b, groups, -1)
    mean = g.mean(-1)
    var = ((g - mean[..., None]) ** 2).mean(-1)
    rstd = 1.0 / torch.sqrt(var + eps)
    per_c = c // groups
    mean_c = mean.repeat_interleave(per_c, dim=1)
    rstd_c = rstd.repeat_interleave(per_c, dim=1)
    gam = weight.double()[None] if weight is not None else torch.ones(1, c, dtype=torch.float64)
    bet = bias.double()[None] if bias is not None else torch.zeros(1, c, dtype=torch.float64)
    scale = gam * rstd_c
    offset = bet - mean_c * scale
    return torch.stack([scale, offset], dim=-1)


def upsample_nearest_ref(x: torch.Tensor) -> torch.Tensor:
    """Nearest 2x on every spatial axis (``tests/test_fast_fp32.py:120-121``)."""
    return x.repeat_interleave(2, 2).repeat_interleave(2, 3).repeat_interleave(2, 4)


def upsample_trilinear_ref(x: torch.Tensor) -> torch.Tensor:
    """Half-pixel trilinear 2x, align_corners=False (``source_vae.py:95-111``; equal to
    ``F.interpolate(..., mode="trilinear")`` per ``tests/test_maisi_mlx_blocks.py:40-47``)."""
    return F.interpolate(x, scale_factor=2, mode="trilinear", align_corners=False)


def avg_pool_ref(x: torch.Tensor) -> torch.Tensor:
    """2x2x2 mean pooling (``medmlx_core.ops.avg_pool3d_ncdhw`` as used at ``fast_fp32.py:250-255``)."""
    return F.avg_pool3d(x, kernel_size=2, stride=2)


def split_fp16_ref(v: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """fp16 hi/lo operand split of ``_nax_conv.py:384-388``: hi = half(v), lo = half((v - hi) * 2^11)."""
    v = np.asarray(v, dtype=np.float32)
    hi = v.astype(np.float16)
    lo = ((v - hi.astype(np.float32)) * np.float32(2048.0)).astype(np.float16)
    return hi, lo


def fold_upsample_weight_ref(w: torch.Tensor) -> torch.Tensor:
    """Nearest-2x fold of a 3x3x3 weight into 8 parities x 2x2x2 taps (``_nax_conv.py:407-445``).

    Returns float64 ``(8, 8, O, C)``: parity ``pd*4+ph*2+pw``, tap ``td*4+th*2+tw``.
    """
    w = w.double()
    sets = {(0, 0): [0], (0, 1): [1, 2], (1, 0): [0, 1], (1, 1): [2]}
    out = torch.zeros(8, 8, w.shape[0], w.shape[1], dtype=torch.float64)
    for par in range(8):
        pd, ph, pw = par >> 2, (par >> 1) & 1, par & 1
        for tap in range(8):
            td, th, tw = tap >> 2, (tap >> 1) & 1, tap & 1
            for kd in sets[(pd, td)]:
                for kh in sets[(ph, th)]:
                    for kw in sets[(pw, tw)]:
                        out[par, tap] += w[:, :, kd, kh, kw]
    return out


def gaussian_1d_ref(length: int, sigma_scale: float = 0.125) -> np.ndarray:
    """One axis of ``decode.gaussian_importance_ncdhw`` (``decode.py:88-112``), float32."""
    half = (length - 1) / 2.0
    x = np.arange(-half, half + 1.0, dtype=np.float32)
    sigma = float(sigma_scale) * float(length)
    return np.exp((x * x) / np.float32(-2.0 * sigma * sigma)).astype(np.float32)


def conv_flops(batch: int, out_vox: int, cout: int, cin: int, taps: int) -> float:
    """Algorithmic FLOPs of one convolution: 2 B V_out C_out C_in T."""
    return 2.0 * batch * out_vox * cout * cin * taps


def rel_l2(a: torch.Tensor, b: torch.Tensor) -> float:
    """||a - b|| / ||b|| in float64."""
    a = a.double()
    b = b.double()
    den = torch.linalg.vector_norm(b).item()
    return torch.linalg.vector_norm(a - b).item() / (den if den > 0 else 1.0)


__all__ = [name for name in dir() if not name.startswith("_") and name not in ("math", "np", "torch", "F")]
