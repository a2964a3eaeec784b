"""Torch-tensor entry points over the C ABI.

Activations are torch tensors with the reference's logical NCDHW shape stored
channels-last (``torch.channels_last_3d``), i.e. physically NDHWC rows; a
channel slice of such a tensor is also accepted (its rows keep the parent's
stride). Every function launches on the current torch CUDA stream and
allocates its outputs and workspaces through torch's caching allocator, so the
calls can be captured in CUDA graphs.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _lib
from ._lib import LIB, check

F32 = torch.float32
BF16 = torch.bfloat16
PRECISIONS = ("fp32", "bf16", "fp16", "tf32")

# Instrumentation: LAUNCHES counts the library's kernel launches issued from
# Python; when PROFILE is a list, conv3d and group_norm_affine append one record
# per stage ({"kind": "prepare" | "gemm" | "gn", "start", "end", "flops", "what"},
# CUDA events on the current stream) around their launches.
LAUNCHES = [0]
PROFILE: list | None = None


def _count(n: int) -> None:
    LAUNCHES[0] += n


class _profiled:
    """Append a PROFILE record bracketing the enclosed launches with CUDA events."""

    def __init__(self, kind: str, flops: float, what: str) -> None:
        self.rec = {"kind": kind, "flops": flops, "what": what,
                    "start": torch.cuda.Event(enable_timing=True), "end": torch.cuda.Event(enable_timing=True)}

    def __enter__(self):
        self.rec["start"].record()
        return self

    def __exit__(self, *exc) -> None:
        self.rec["end"].record()
        PROFILE.append(self.rec)


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _dtype_code(dtype: torch.dtype, *, allow_f16: bool = False) -> int:
    if dtype == F32:
        return _lib.DTYPE_F32
    if dtype == BF16:
        return _lib.DTYPE_BF16
    if allow_f16 and dtype == torch.float16:
        return _lib.DTYPE_F16
    raise ValueError(f"ctmr_b200 activations must be float32 or bfloat16, got {dtype}")


def _precision_code(precision: str) -> int:
    if precision == "fp32":
        return _lib.PRECISION_FP32
    if precision == "bf16":
        return _lib.PRECISION_BF16
    if precision == "fp16":
        return _lib.PRECISION_FP16
    if precision == "tf32":
        return _lib.PRECISION_TF32
    raise ValueError(f"precision must be one of {PRECISIONS}; got {precision!r}")


def rows_stride(x: torch.Tensor) -> int:
    """Elements between voxel rows of an NDHWC-stored NCDHW tensor; raises if not so stored."""
    if x.dim() != 5:
        raise ValueError(f"expected an NCDHW tensor, got shape {tuple(x.shape)}")
    b, c, d, h, w = (int(n) for n in x.shape)
    if w > 1:
        cs = x.stride(4)
    elif h > 1:
        cs = x.stride(3)
    elif d > 1:
        cs = x.stride(2)
    elif b > 1:
        cs = x.stride(0)
    else:
        cs = c
    ok = cs >= c and (c == 1 or x.stride(1) == 1)
    ok = ok and (w == 1 or x.stride(4) == cs) and (h == 1 or x.stride(3) == w * cs)
    ok = ok and (d == 1 or x.stride(2) == h * w * cs) and (b == 1 or x.stride(0) == d * h * w * cs)
    if not ok:
        raise ValueError(
            f"tensor of shape {tuple(x.shape)} and strides {x.stride()} is not channels-last (NDHWC rows)"
        )
    return int(cs)


class LabelBits:
    """An int16 label volume ``(N, 1, D, H, W)`` that ``conv3d`` reads as its 8 bit-plane
    channels (channel k = bit k of the id, 0.0 or 1.0), formed in the conv's operand pass
    (``CTMR_DTYPE_LABEL8``) instead of as a materialised fp32 condition: the ControlNet
    condition of ``condition.binarize_labels_ncdhw`` (``condition.py:20-43``)."""

    def __init__(self, label: torch.Tensor) -> None:
        if label.dim() != 5 or int(label.shape[1]) != 1 or not label.is_cuda:
            raise ValueError(f"label must be a CUDA (N, 1, D, H, W) tensor; got {tuple(label.shape)}")
        if label.dtype not in (torch.int16, torch.int32, torch.int64, torch.uint8):
            raise ValueError(f"label must be integer; got {label.dtype}")
        self.label = label.to(torch.int16).contiguous()
        self.shape = torch.Size((int(label.shape[0]), 8, *(int(s) for s in label.shape[2:])))
        self.device = label.device
        self.dtype = torch.int16

    def dim(self) -> int:
        return 5


def view(x) -> _lib.Tensor:
    """``ctmr_tensor`` for an NDHWC-stored tensor, a ``LabelBits`` volume, or an absent one."""
    if x is None:
        return _lib.Tensor(None, 0, 0, 0)
    if isinstance(x, LabelBits):
        return _lib.Tensor(x.label.data_ptr(), _lib.DTYPE_LABEL8, 8, 1)
    if not x.is_cuda:
        raise ValueError("ctmr_b200 tensors must live on a CUDA device")
    return _lib.Tensor(x.data_ptr(), _dtype_code(x.dtype), int(x.shape[1]), rows_stride(x))


def empty_ndhwc(b: int, c: int, d: int, h: int, w: int, dtype: torch.dtype, device) -> torch.Tensor:
    """Uninitialised NCDHW tensor with channels-last storage."""
    return torch.empty((b, c, d, h, w), dtype=dtype, device=device, memory_format=torch.channels_last_3d)


def to_ndhwc(x: torch.Tensor, dtype: torch.dtype | None = None) -> torch.Tensor:
    """Channels-last copy of an NCDHW tensor (via the library's transpose kernel when contiguous NCDHW)."""
    dtype = dtype or x.dtype
    try:
        rows_stride(x)
        return x if x.dtype == dtype else transform(x, out_dtype=dtype)
    except ValueError:
        pass
    x = x.contiguous()
    b, c, d, h, w = x.shape
    out = empty_ndhwc(b, c, d, h, w, dtype, x.device)
    _count(1)
    check(
        LIB.ctmr_ncdhw_to_ndhwc(
            x.data_ptr(), _dtype_code(x.dtype), out.data_ptr(), _dtype_code(dtype), b, c, d * h * w, _stream()
        ),
        "ncdhw_to_ndhwc",
    )
    return out


def to_ncdhw(x: torch.Tensor, dtype: torch.dtype = F32) -> torch.Tensor:
    """Contiguous NCDHW copy of a channels-last tensor (library transpose kernel)."""
    cs = rows_stride(x)
    b, c, d, h, w = x.shape
    if cs != c:
        x = transform(x, out_dtype=x.dtype)
    out = torch.empty((b, c, d, h, w), dtype=dtype, device=x.device)
    _count(1)
    check(
        LIB.ctmr_ndhwc_to_ncdhw(
            x.data_ptr(), _dtype_code(x.dtype), out.data_ptr(), _dtype_code(dtype), b, c, d * h * w, _stream()
        ),
        "ndhwc_to_ncdhw",
    )
    return out


@dataclass(frozen=True)
class PackedWeight:
    """Convolution weight packed for the tensor cores (``ctmr_pack_weight``)."""

    hi: torch.Tensor
    lo: torch.Tensor | None
    out_channels: int
    in_channels: int
    kernel_size: int
    upsample: bool
    precision: str


def pack_weight(weight: torch.Tensor, precision: str, *, upsample: bool = False) -> PackedWeight:
    """Pack a Torch ``(O, C, k, k, k)`` weight; the nearest-2x fold with ``upsample``.

    Counterpart of ``pack_weight`` / ``pack_upsample_weight`` (``_nax_conv.py:391-445``).
    A weight whose storage is channels-last ``(O, k, k, k, C)`` — the Torch-layout view
    ``weights.load_network_file`` returns for a released checkpoint — is packed from
    that storage directly (``ctmr_pack_weight_channels_last``), without a transposed copy.
    """
    if weight.dim() != 5 or weight.shape[2] != weight.shape[3] or weight.shape[3] != weight.shape[4]:
        raise ValueError(f"conv weight must be (O, C, k, k, k); got {tuple(weight.shape)}")
    o, c, k = int(weight.shape[0]), int(weight.shape[1]), int(weight.shape[2])
    code = _precision_code(precision)
    w = weight.detach()
    channels_last = (w.dtype == F32 and c > 1 and k > 1 and
                     w.is_contiguous(memory_format=torch.channels_last_3d))
    if not channels_last:
        w = w.to(dtype=F32).contiguous()
    entry = LIB.ctmr_pack_weight_channels_last if channels_last else LIB.ctmr_pack_weight
    n = int(LIB.ctmr_packed_weight_elems(o, c, k, int(upsample)))
    if n == 0:
        raise ValueError(f"unsupported conv weight shape {tuple(weight.shape)}")
    if precision == "fp32":
        hi = torch.empty(n, dtype=torch.float16, device=w.device)
        lo = torch.empty(n, dtype=torch.float16, device=w.device)
    elif precision == "tf32":  # TF32-rounded fp32 rows of round8(C) values
        hi = torch.empty(int(LIB.ctmr_packed_weight_bytes(o, c, k, int(upsample), code)) // 4, dtype=F32,
                         device=w.device)
        lo = None
    else:
        hi = torch.empty(n, dtype=BF16 if precision == "bf16" else torch.float16, device=w.device)
        lo = None
    _count(1)
    check(
        entry(
            w.data_ptr(), o, c, k, int(upsample), code, hi.data_ptr(), lo.data_ptr() if lo is not None else None,
            _stream(),
        ),
        "pack_weight",
    )
    return PackedWeight(hi, lo, o, c, k, upsample, precision)


def conv3d(
    x: torch.Tensor,
    packed: PackedWeight,
    bias: torch.Tensor | None = None,
    *,
    x2: torch.Tensor | None = None,
    affine: torch.Tensor | None = None,
    silu: bool = False,
    stride: int = 1,
    trilinear: bool = False,
    avgpool: bool = False,
    residual: torch.Tensor | None = None,
    residual_upsampled: bool = False,
    out: torch.Tensor | None = None,
    out_dtype: torch.dtype | None = None,
    stats: bool = False,
    workspace: torch.Tensor | None = None,
    stages: int | None = None,
    norm: tuple | None = None,
) -> torch.Tensor:
    """``conv(prepare(x ++ x2)) + bias (+ residual)`` in one call (``ctmr_conv3d``).

    Mirrors ``nax_conv3d`` (``_nax_conv.py:475-487``): ``bias`` is ``(O,)`` or per
    batch item ``(B, O)``; ``affine`` is the ``(B, C, 2)`` group-norm scale/offset;
    ``silu`` follows it; ``packed.upsample`` convolves the nearest-2x upsampling,
    ``trilinear`` the half-pixel trilinear-2x upsampling and ``avgpool`` the 2x2x2
    mean of the prepared input; the residual (on the output grid, or the half grid
    when ``residual_upsampled``) is added before the single rounding.
    """
    b, cx, d, h, w = (int(n) for n in x.shape)
    cin = cx + (int(x2.shape[1]) if x2 is not None else 0)
    if x2 is not None and tuple(x2.shape[2:]) != (d, h, w):
        raise ValueError(f"concat inputs differ in grid: {tuple(x.shape)} vs {tuple(x2.shape)}")
    if cin != packed.in_channels:
        raise ValueError(f"packed weight has {packed.in_channels} input channels, input has {cin}")
    k = packed.kernel_size
    if packed.upsample:
        od, oh, ow = 2 * d, 2 * h, 2 * w
    elif trilinear:
        od, oh, ow = 2 * d, 2 * h, 2 * w
    elif avgpool:
        od, oh, ow = d // 2, h // 2, w // 2
    elif stride == 2:
        od, oh, ow = (d - 1) // 2 + 1, (h - 1) // 2 + 1, (w - 1) // 2 + 1
    else:
        od, oh, ow = d, h, w
    o = packed.out_channels
    bias_rows = 0
    if bias is not None:
        if not (bias.shape == (o,) or bias.shape == (b, o)):
            raise ValueError(f"bias shape {tuple(bias.shape)} must be ({o},) or ({b}, {o})")
        if bias.dim() == 2 and bias.dtype == F32 and bias.stride(1) == 1 and bias.stride(0) >= o:
            bias_rows = int(bias.stride(0))  # a column slice of a wider table: read in place
        else:
            bias = bias.to(dtype=F32).contiguous()
    if affine is not None:
        affine = affine.to(dtype=F32).contiguous()
        if affine.numel() != b * cin * 2:
            raise ValueError(f"affine must hold (B, C, 2) = ({b}, {cin}, 2) values")
    if residual is not None:
        expect = (b, o, od // 2, oh // 2, ow // 2) if residual_upsampled else (b, o, od, oh, ow)
        if tuple(residual.shape) != expect:
            raise ValueError(f"residual shape {tuple(residual.shape)} != output {expect}")
    if out is None:
        dtype = out_dtype or F32
        out = empty_ndhwc(b, o, od, oh, ow, dtype, x.device)
    elif tuple(out.shape) != (b, o, od, oh, ow):
        raise ValueError(f"out shape {tuple(out.shape)} != {(b, o, od, oh, ow)}")
    ycs = rows_stride(out)
    desc = _lib.Conv3dDesc()
    desc.batch, desc.depth, desc.height, desc.width = b, d, h, w
    desc.x = view(x)
    desc.x2 = view(x2)
    desc.out_channels = o
    desc.kernel_size = k
    desc.stride = stride
    desc.upsample = int(packed.upsample)
    desc.trilinear = int(trilinear)
    desc.avgpool = int(avgpool)
    desc.precision = _precision_code(packed.precision)
    desc.weight = packed.hi.data_ptr()
    desc.weight_lo = packed.lo.data_ptr() if packed.lo is not None else None
    desc.affine = affine.data_ptr() if affine is not None else None
    desc.silu = int(silu)
    desc.bias = bias.data_ptr() if bias is not None else None
    desc.bias_per_batch = int(bias is not None and bias.dim() == 2)
    desc.bias_row_stride = bias_rows
    desc.residual = view(residual)
    desc.residual_upsampled = int(residual_upsampled)
    desc.y = out.data_ptr()  # a channel slice's pointer already includes its first channel
    desc.y_dtype = _dtype_code(out.dtype)
    desc.y_cstride = ycs
    desc.y_coffset = 0
    keep = []
    if norm is not None:  # (gamma, beta, groups, eps): the input's GroupNorm computed inside the call
        gamma, beta, groups, eps = norm
        gamma = gamma.to(dtype=F32).contiguous() if gamma is not None else None
        beta = beta.to(dtype=F32).contiguous() if beta is not None else None
        keep = [gamma, beta]
        desc.gn_gamma = gamma.data_ptr() if gamma is not None else None
        desc.gn_beta = beta.data_ptr() if beta is not None else None
        desc.gn_groups = int(groups)
        desc.gn_eps = float(eps)
    stats_buf = None
    if stats:  # GroupNorm moments of the output from the conv epilogue, when its kernel can produce them
        slots = int(LIB.ctmr_conv3d_stats_slots(ctypes.byref(desc)))
        if slots > 0:
            stats_buf = torch.empty((b, slots, o, 3), dtype=F32, device=x.device)
            desc.stats = stats_buf.data_ptr()
            desc.stats_slots = slots
    ws_bytes = int(LIB.ctmr_conv3d_workspace_size(ctypes.byref(desc)))
    if workspace is not None:  # caller-held workspace (e.g. to time the GEMM stage alone)
        if workspace.numel() < ws_bytes:
            raise WorkspaceTooSmall(ws_bytes, workspace.numel())
        ws = workspace
    else:
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=x.device) if ws_bytes else None
    ws_ptr = ws.data_ptr() if ws is not None else None
    if stages is not None:  # one or both stages (_lib.CONV_PREPARE | _lib.CONV_GEMM)
        _count(int(LIB.ctmr_conv3d_launch_count(ctypes.byref(desc))))
        check(LIB.ctmr_conv3d_stages(ctypes.byref(desc), ws_ptr, ws_bytes, int(stages), _stream()), "conv3d stages")
        return out
    _count(int(LIB.ctmr_conv3d_launch_count(ctypes.byref(desc))))
    if PROFILE is None:
        check(LIB.ctmr_conv3d(ctypes.byref(desc), ws_ptr, ws_bytes, _stream()), "conv3d")
    else:
        taps = 8 if packed.upsample else k ** 3
        what = (f"{b}x{cin}->{o} out {od}x{oh}x{ow} k{k} s{stride} up{int(packed.upsample)} tri{int(trilinear)} "
                f"pool{int(avgpool)} norm{int(affine is not None or norm is not None)} res{int(residual is not None)} "
                f"{packed.precision}")
        if ws_bytes:
            with _profiled("prepare", 0.0, what):
                check(LIB.ctmr_conv3d_stages(ctypes.byref(desc), ws_ptr, ws_bytes, _lib.CONV_PREPARE, _stream()),
                      "conv3d prepare")
        with _profiled("gemm", 2.0 * b * od * oh * ow * o * cin * taps, what):
            check(LIB.ctmr_conv3d_stages(ctypes.byref(desc), ws_ptr, ws_bytes, _lib.CONV_GEMM, _stream()),
                  "conv3d gemm")
    if stats_buf is not None:
        out._ctmr_stats = OutputStats(stats_buf, int(desc.stats_slots), o)
    del keep
    return out


class WorkspaceTooSmall(ValueError):
    """A caller-held conv3d workspace is smaller than the call needs (``needed`` bytes)."""

    def __init__(self, needed: int, given: int) -> None:
        super().__init__(f"conv3d workspace holds {given} bytes, needs {needed}")
        self.needed = needed


class OutputStats:
    """Per-(batch item, slot, channel) moments a convolution wrote for its output tensor."""

    __slots__ = ("buffer", "slots", "channels")

    def __init__(self, buffer: torch.Tensor, slots: int, channels: int) -> None:
        self.buffer, self.slots, self.channels = buffer, slots, channels


def output_stats(t: torch.Tensor | None) -> OutputStats | None:
    """The statistics attached to ``t`` by the convolution that produced it, if any."""
    return getattr(t, "_ctmr_stats", None) if t is not None else None


def group_norm_affine(
    x: torch.Tensor,
    weight: torch.Tensor | None,
    bias: torch.Tensor | None,
    *,
    groups: int,
    eps: float,
    x2: torch.Tensor | None = None,
) -> torch.Tensor:
    """GroupNorm statistics of ``x ++ x2`` as ``(B, C, 2)`` (scale, offset) pairs (``ctmr_group_norm_affine``)."""
    b, c, d, h, w = (int(n) for n in x.shape)
    ctot = c + (int(x2.shape[1]) if x2 is not None else 0)
    voxels = d * h * w
    if ctot % groups:
        raise ValueError("group_norm channels must be divisible by num_groups")
    gamma = weight.to(dtype=F32).contiguous() if weight is not None else None
    beta = bias.to(dtype=F32).contiguous() if bias is not None else None
    affine = torch.empty((b, ctot, 2), dtype=F32, device=x.device)
    sa, sb = output_stats(x), output_stats(x2)
    if (sa is not None and sa.channels == c and (x2 is None or (sb is not None and sb.slots == sa.slots and
                                                                sb.channels == ctot - c))):
        # The producing convolutions already reduced the moments: merge them only.
        _count(1)

        def from_stats() -> None:
            check(LIB.ctmr_group_norm_affine_from_stats(
                sa.buffer.data_ptr(), c, sb.buffer.data_ptr() if sb is not None else None, ctot - c if sb else 0,
                sa.slots, b, gamma.data_ptr() if gamma is not None else None,
                beta.data_ptr() if beta is not None else None, groups, float(eps), affine.data_ptr(), _stream()),
                "group_norm_affine_from_stats")

        if PROFILE is None:
            from_stats()
        else:
            with _profiled("gn", 0.0, f"{b}x{ctot} {d}x{h}x{w} g{groups} from-stats"):
                from_stats()
        return affine
    _count(int(LIB.ctmr_group_norm_launch_count(voxels, ctot, groups)))
    ws_bytes = int(LIB.ctmr_group_norm_workspace_size(b, voxels, groups))
    ws = torch.empty(max(ws_bytes, 4), dtype=torch.uint8, device=x.device)
    def launch() -> None:
        check(
            LIB.ctmr_group_norm_affine(
                view(x), view(x2), b, voxels,
                gamma.data_ptr() if gamma is not None else None,
                beta.data_ptr() if beta is not None else None,
                groups, float(eps), affine.data_ptr(), ws.data_ptr(), ws_bytes, _stream(),
            ),
            "group_norm_affine",
        )

    if PROFILE is None:
        launch()
    else:
        with _profiled("gn", 0.0, f"{b}x{ctot} {d}x{h}x{w} g{groups}"):
            launch()
    return affine


def group_norm_moments(x: torch.Tensor, *, groups: int, x2: torch.Tensor | None = None,
                       out: torch.Tensor | None = None) -> torch.Tensor:
    """Merged ``(count, mean, M2)`` per (batch item, group) of ``x ++ x2`` as ``(B, groups, 3)`` fp32
    (``ctmr_group_norm_moments``): the statistics of ``group_norm_affine`` before the affine, for
    tensors split across devices. ``out`` may be a view into a larger (exchange) buffer."""
    b, c, d, h, w = (int(n) for n in x.shape)
    ctot = c + (int(x2.shape[1]) if x2 is not None else 0)
    if ctot % groups:
        raise ValueError("group_norm channels must be divisible by num_groups")
    if out is None:
        out = torch.empty((b, groups, 3), dtype=F32, device=x.device)
    elif out.dtype != F32 or out.numel() != b * groups * 3 or not out.is_contiguous():
        raise ValueError(f"moments output must be {b * groups * 3} contiguous float32 values")
    voxels = d * h * w
    ws_bytes = int(LIB.ctmr_group_norm_workspace_size(b, voxels, groups))
    ws = torch.empty(max(ws_bytes, 4), dtype=torch.uint8, device=x.device)
    _count(2)
    check(LIB.ctmr_group_norm_moments(view(x), view(x2), b, voxels, groups, out.data_ptr(), ws.data_ptr(), ws_bytes,
                                      _stream()), "group_norm_moments")
    return out


def group_norm_affine_from_moments(moments: torch.Tensor, weight: torch.Tensor | None, bias: torch.Tensor | None, *,
                                   channels: int, groups: int, eps: float) -> torch.Tensor:
    """``(B, C, 2)`` affine from the moments ``(parts, B, groups, 3)`` of the parts of one tensor
    (``ctmr_group_norm_affine_from_moments``; merged in part order)."""
    if moments.dim() != 4 or int(moments.shape[2]) != groups or int(moments.shape[3]) != 3:
        raise ValueError(f"moments must be (parts, B, {groups}, 3); got {tuple(moments.shape)}")
    moments = moments.to(dtype=F32).contiguous()
    parts, b = int(moments.shape[0]), int(moments.shape[1])
    gamma = weight.to(dtype=F32).contiguous() if weight is not None else None
    beta = bias.to(dtype=F32).contiguous() if bias is not None else None
    affine = torch.empty((b, channels, 2), dtype=F32, device=moments.device)
    _count(1)
    check(LIB.ctmr_group_norm_affine_from_moments(
        moments.data_ptr(), parts, b, int(channels), gamma.data_ptr() if gamma is not None else None,
        beta.data_ptr() if beta is not None else None, int(groups), float(eps), affine.data_ptr(), _stream()),
        "group_norm_affine_from_moments")
    return affine


def attention_d32(qkv: torch.Tensor, heads: int, scale: float) -> torch.Tensor:
    """``softmax(Q K^T * scale) V`` per head for head size 32 (``ctmr_attention_d32``).

    ``qkv`` is the fused projection ``(B, L, 3 * heads * 32)`` in fp16 or bf16 with
    ``L`` a multiple of 128; returns ``(B, L, heads * 32)`` in the same type. The
    counterpart of the reference's ``flash_attention`` (``_flash_attention.py:320-360``).
    """
    if qkv.dim() != 3 or qkv.dtype not in (torch.float16, BF16) or not qkv.is_contiguous():
        raise ValueError("qkv must be a contiguous (B, L, 3C) fp16/bf16 tensor")
    b, length, c3 = (int(n) for n in qkv.shape)
    if c3 != 3 * heads * 32 or length % 128:
        raise ValueError(f"qkv {tuple(qkv.shape)} does not hold {heads} heads of 32 over a multiple of 128 tokens")
    out = torch.empty((b, length, heads * 32), dtype=qkv.dtype, device=qkv.device)
    _count(1)
    check(LIB.ctmr_attention_d32(qkv.data_ptr(), _lib.DTYPE_BF16 if qkv.dtype == BF16 else _lib.DTYPE_F16, b, length,
                                 heads, float(scale), out.data_ptr(), _stream()), "attention")
    return out


def transform(
    x: torch.Tensor,
    *,
    x2: torch.Tensor | None = None,
    mode: int = _lib.TRANSFORM_COPY,
    affine: torch.Tensor | None = None,
    silu: bool = False,
    out_dtype: torch.dtype | None = None,
    out_channels: int | None = None,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """Materialise ``mode(silu?(affine?(x ++ x2)))`` channels-last (``ctmr_transform``)."""
    b, c, d, h, w = (int(n) for n in x.shape)
    ctot = c + (int(x2.shape[1]) if x2 is not None else 0)
    if mode == _lib.TRANSFORM_TRILINEAR:
        od, oh, ow = 2 * d, 2 * h, 2 * w
    elif mode == _lib.TRANSFORM_AVGPOOL:
        od, oh, ow = d // 2, h // 2, w // 2
    else:
        od, oh, ow = d, h, w
    cout = out_channels or ctot
    if out is None:
        out = empty_ndhwc(b, cout, od, oh, ow, out_dtype or x.dtype, x.device)
    if affine is not None:
        affine = affine.to(dtype=F32).contiguous()
    desc = _lib.TransformDesc()
    desc.batch, desc.depth, desc.height, desc.width = b, d, h, w
    desc.x = view(x)
    desc.x2 = view(x2)
    desc.mode = mode
    desc.affine = affine.data_ptr() if affine is not None else None
    desc.silu = int(silu)
    desc.y = out.data_ptr()
    desc.y_dtype = _dtype_code(out.dtype, allow_f16=True)  # fp16 is a transform-only output (dense operands)
    desc.y_channels = int(out.shape[1])
    desc.y_cstride = rows_stride(out)
    _count(1)
    check(LIB.ctmr_transform(ctypes.byref(desc), _stream()), "transform")
    return out


def rflow_step(z: torch.Tensor, velocity: torch.Tensor, *, guidance: float | None, dt: float | torch.Tensor,
               out: torch.Tensor | None = None) -> torch.Tensor:
    """Guided Euler update ``z + dt * (u + s (c - u))`` (``ctmr_rflow_step``).

    ``z`` and ``velocity`` are fp32 and share one memory layout (``velocity`` holds
    the [cond, uncond] batch when guided); ``dt`` may be a device scalar tensor,
    read at execution time; ``out`` may be ``z``.
    """
    if z.dtype != F32 or velocity.dtype != F32:
        raise ValueError("rflow_step takes float32 tensors")
    # (a batch-1 tensor's batch stride is immaterial: e.g. the inner planes of a depth shard)
    first = 1 if int(z.shape[0]) == 1 else 0
    if z.stride()[first:] != velocity[: z.shape[0]].stride()[first:] or not (z.is_contiguous() or z.is_contiguous(
            memory_format=torch.channels_last_3d)):
        raise ValueError("z and velocity must be dense with the same memory layout")
    n = z.numel()
    guided = guidance is not None
    if velocity.numel() != (2 * n if guided else n):
        raise ValueError("velocity must hold the [cond, uncond] batch when guided")
    out = out if out is not None else torch.empty_like(z)
    dt_dev = dt.data_ptr() if isinstance(dt, torch.Tensor) else None
    _count(1)
    check(
        LIB.ctmr_rflow_step(z.data_ptr(), velocity.data_ptr(), n, float(guidance or 0.0), int(guided),
                            0.0 if dt_dev is not None else float(dt), dt_dev, out.data_ptr(), _stream()),
        "rflow_step",
    )
    return out


def window_accumulate(pred: torch.Tensor, acc: torch.Tensor, wsum: torch.Tensor, *, origin: tuple[int, int, int],
                      tables: list[torch.Tensor], scale: int, floor: float) -> None:
    """Add one decoded window, Gaussian-weighted, into the blend (``ctmr_window_accumulate``).

    ``pred`` is the channels-last window ``(B, C, wd, wh, ww)``; ``acc`` is the
    fp32 NDHWC accumulator ``(B, OD, OH, OW, C)`` and ``wsum`` the fp32 weight
    sum ``(OD, OH, OW)``; ``tables`` are the per-axis 1-D Gaussians over the
    latent ROI, resized by ``scale`` with nearest indexing.
    """
    b, c, wd, wh, ww = (int(n) for n in pred.shape)
    od, oh, ow = (int(n) for n in acc.shape[1:4])
    if acc.dtype != F32 or wsum.dtype != F32 or not acc.is_contiguous() or not wsum.is_contiguous():
        raise ValueError("window accumulators must be contiguous float32")
    gz, gy, gx = (t.to(F32).contiguous() for t in tables)
    _count(1)
    check(
        LIB.ctmr_window_accumulate(view(pred), b, wd, wh, ww, int(origin[0]), int(origin[1]), int(origin[2]), od, oh,
                                   ow, gz.data_ptr(), gy.data_ptr(), gx.data_ptr(), int(scale), float(floor),
                                   acc.data_ptr(), wsum.data_ptr(), _stream()),
        "window_accumulate",
    )


def window_finalize(acc: torch.Tensor, wsum: torch.Tensor, *, origin: tuple[int, int, int],
                    extent: tuple[int, int, int]) -> torch.Tensor:
    """``acc / wsum`` over the crop at ``origin`` as a contiguous NCDHW fp32 tensor (``ctmr_window_finalize``)."""
    b, od, oh, ow, c = (int(n) for n in acc.shape)
    out = torch.empty((b, c, *(int(e) for e in extent)), dtype=F32, device=acc.device)
    _count(1)
    check(
        LIB.ctmr_window_finalize(acc.data_ptr(), wsum.data_ptr(), out.data_ptr(), b, c, od, oh, ow, int(origin[0]),
                                 int(origin[1]), int(origin[2]), int(extent[0]), int(extent[1]), int(extent[2]),
                                 _stream()),
        "window_finalize",
    )
    return out
