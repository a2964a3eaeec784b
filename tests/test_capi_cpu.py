"""The C-ABI library loads on a CPU host, exports every declared symbol, and validates arguments
(status codes, no CUDA call) exactly as the header documents."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from ctmr_b200 import _lib

HEADER = Path(__file__).resolve().parents[1] / "include" / "ctmr_b200.h"


def test_header_symbols_are_exported():
    declared = set(re.findall(r"CTMR_API\s+[\w\s\*]+?\b(ctmr_\w+)\s*\(", HEADER.read_text()))
    assert declared == set(_lib.EXPORTED_SYMBOLS)
    for name in declared:
        assert hasattr(_lib.LIB, name), name


def test_packed_weight_elems():
    assert _lib.LIB.ctmr_packed_weight_elems(64, 64, 3, 0) == 27 * 64 * 64
    assert _lib.LIB.ctmr_packed_weight_elems(4, 4, 3, 0) == 27 * 16 * 16
    assert _lib.LIB.ctmr_packed_weight_elems(32, 24, 3, 1) == 64 * 32 * 32
    assert _lib.LIB.ctmr_packed_weight_elems(1, 64, 1, 0) == 16 * 64
    assert _lib.LIB.ctmr_packed_weight_elems(4, 4, 5, 0) == 0


def _desc(**kw) -> _lib.Conv3dDesc:
    d = _lib.Conv3dDesc()
    d.batch, d.depth, d.height, d.width = 1, 4, 4, 4
    d.x = _lib.Tensor(0x10000, _lib.DTYPE_F32, 32, 32)
    d.out_channels, d.kernel_size, d.stride = 32, 3, 1
    d.precision = _lib.PRECISION_FP32
    d.weight, d.weight_lo = 0x20000, 0x30000
    d.y, d.y_dtype, d.y_cstride = 0x40000, _lib.DTYPE_F32, 32
    for k, v in kw.items():
        setattr(d, k, v)
    return d


def _status(desc) -> int:
    return _lib.LIB.ctmr_conv3d(ctypes.byref(desc), None, 0, None)


def test_workspace_size_reports_prepared_operand():
    # fp32 split mode on a grid large enough to fill the GPU: hi + lo fp16 planes of
    # B * D * H * W * round16(C) elements, nothing else.
    big = _desc(depth=64, height=64, width=64)
    assert _lib.LIB.ctmr_conv3d_workspace_size(ctypes.byref(big)) == 2 * 64 ** 3 * 32 * 2
    # trilinear input doubles every axis before the conv
    assert _lib.LIB.ctmr_conv3d_workspace_size(ctypes.byref(_desc(depth=32, height=32, width=32, trilinear=1))) == (
        2 * 64 ** 3 * 32 * 2)
    # a tiny grid splits K across CTAs: the fp32 partial planes come on top of the operand
    assert _lib.LIB.ctmr_conv3d_workspace_size(ctypes.byref(_desc())) > 2 * 64 * 32 * 2


@pytest.mark.parametrize(("overrides", "status"), [
    ({"batch": 0}, _lib.CTMR_ERR_INVALID),
    ({"kernel_size": 5}, _lib.CTMR_ERR_UNSUPPORTED),
    ({"stride": 3}, _lib.CTMR_ERR_UNSUPPORTED),
    ({"upsample": 1, "trilinear": 1}, _lib.CTMR_ERR_UNSUPPORTED),
    ({"avgpool": 1, "depth": 3}, _lib.CTMR_ERR_INVALID),
    ({"y_cstride": 16}, _lib.CTMR_ERR_INVALID),
    ({"weight_lo": None}, _lib.CTMR_ERR_INVALID),
    ({"precision": 7}, _lib.CTMR_ERR_INVALID),
    ({"trilinear": 1, "silu": 1}, _lib.CTMR_ERR_UNSUPPORTED),
    ({"stride": 2, "width": 1}, _lib.CTMR_ERR_UNSUPPORTED),
    # label volumes (int16 ids read as 8 bit planes): 8 channels, only as the plain conv input
    ({"x": _lib.Tensor(0x10000, _lib.DTYPE_LABEL8, 4, 1)}, _lib.CTMR_ERR_INVALID),
    ({"residual": _lib.Tensor(0x50000, _lib.DTYPE_LABEL8, 8, 1)}, _lib.CTMR_ERR_INVALID),
    ({"x": _lib.Tensor(0x10000, _lib.DTYPE_LABEL8, 8, 1), "stride": 2}, _lib.CTMR_ERR_UNSUPPORTED),
    ({"x": _lib.Tensor(0x10000, _lib.DTYPE_LABEL8, 8, 1), "trilinear": 1}, _lib.CTMR_ERR_UNSUPPORTED),
    ({"x": _lib.Tensor(0x10000, _lib.DTYPE_LABEL8, 8, 1), "x2": _lib.Tensor(0x50000, _lib.DTYPE_F32, 8, 8)},
     _lib.CTMR_ERR_UNSUPPORTED),
    ({"x": _lib.Tensor(0x10000, _lib.DTYPE_LABEL8, 8, 1), "gn_groups": 8}, _lib.CTMR_ERR_UNSUPPORTED),
    # per-batch bias rows: 0 (rows of out_channels) or a stride of at least out_channels
    ({"bias_row_stride": 16}, _lib.CTMR_ERR_INVALID),
    ({"bias_row_stride": 1 << 31}, _lib.CTMR_ERR_INVALID),
])
def test_conv_argument_validation(overrides, status):
    assert _status(_desc(**overrides)) == status
    assert _lib.LIB.ctmr_last_error()


def test_conv_workspace_too_small():
    assert _status(_desc()) == _lib.CTMR_ERR_WORKSPACE


def test_check_maps_status_to_exceptions():
    with pytest.raises(ValueError):
        _lib.check(_lib.CTMR_ERR_INVALID, "x")
    with pytest.raises(_lib.CtmrError):
        _lib.check(_lib.CTMR_ERR_CUDA, "x")
    _lib.check(_lib.CTMR_OK, "x")


def test_group_norm_validation():
    t = _lib.Tensor(0x10000, _lib.DTYPE_F32, 30, 30)
    none = _lib.Tensor(None, 0, 0, 0)
    st = _lib.LIB.ctmr_group_norm_affine(t, none, 1, 64, None, None, 32, 1e-6, 0x2000, 0x3000, 1 << 20, None)
    assert st == _lib.CTMR_ERR_INVALID  # 30 channels are not divisible by 32 groups


def test_group_norm_launch_count(monkeypatch):
    """One launch for groups that 1024 threads read with at most eight loads each (four channels per
    load when the group's channel count allows, at most 64 channels), two otherwise;
    CTMR_DISABLE_GN_DIRECT keeps the two-pass path everywhere; invalid extents count nothing."""
    count = _lib.LIB.ctmr_group_norm_launch_count
    monkeypatch.delenv("CTMR_DISABLE_GN_DIRECT", raising=False)
    assert count(8 * 8 * 4, 512, 32) == 1          # the UNet's deepest level: one load per thread
    assert count(16 * 16 * 8, 512, 32) == 1        # level 2 concat, 16 channels per group: eight loads
    assert count(16 * 16 * 8, 768, 32) == 2        # 24 channels per group: thirteen loads
    assert count(8192, 128, 32) == 1               # 8,192 voxels x 4 channels: eight loads
    assert count(8193, 128, 32) == 2               # one voxel more: a ninth load
    assert count(32 * 32 * 16, 128, 32) == 2       # level 1
    assert count(64 * 64 * 32, 64, 32) == 2        # the UNet's level 0
    assert count(16, 65 * 2, 2) == 2               # 65 channels per group
    assert count(100, 30, 4) == 0                  # channels not divisible by groups
    monkeypatch.setenv("CTMR_DISABLE_GN_DIRECT", "1")
    assert count(8 * 8 * 4, 512, 32) == 2


@pytest.mark.parametrize(("args", "status"), [
    ((None, _lib.DTYPE_F16, 1, 128, 1, 0x2000), _lib.CTMR_ERR_INVALID),        # no Q/K/V
    ((0x1000, _lib.DTYPE_F32, 1, 128, 1, 0x2000), _lib.CTMR_ERR_INVALID),      # fp32 operands
    ((0x1000, _lib.DTYPE_BF16, 0, 128, 1, 0x2000), _lib.CTMR_ERR_INVALID),     # empty batch
    ((0x1000, _lib.DTYPE_F16, 1, 200, 1, 0x2000), _lib.CTMR_ERR_UNSUPPORTED),  # tokens not a multiple of 128
    ((0x1008, _lib.DTYPE_F16, 1, 128, 1, 0x2000), _lib.CTMR_ERR_INVALID),      # Q/K/V not 16-byte aligned
])
def test_attention_validation(args, status):
    qkv, dtype, batch, tokens, heads, out = args
    assert _lib.LIB.ctmr_attention_d32(qkv, dtype, batch, tokens, heads, 1.0, out, None) == status
    assert _lib.LIB.ctmr_last_error()


@pytest.mark.parametrize("scale", [0.0, -0.5, float("nan")])
def test_attention_scale_must_be_positive(scale):
    """The kernel takes each row's maximum of the raw logits and scales it afterwards, which is the
    maximum of the scaled logits only for a positive scale: anything else is refused, nothing launched."""
    st = _lib.LIB.ctmr_attention_d32(0x1000, _lib.DTYPE_F16, 1, 128, 1, scale, 0x2000, None)
    assert st == _lib.CTMR_ERR_INVALID
    assert b"scale" in _lib.LIB.ctmr_last_error()


def _tdesc(**kw) -> _lib.TransformDesc:
    d = _lib.TransformDesc()
    d.batch, d.depth, d.height, d.width = 1, 4, 4, 4
    d.x = _lib.Tensor(0x10000, _lib.DTYPE_F32, 32, 32)
    d.y, d.y_dtype, d.y_channels, d.y_cstride = 0x40000, _lib.DTYPE_F32, 32, 32
    for k, v in kw.items():
        setattr(d, k, v)
    return d


@pytest.mark.parametrize(("overrides", "status"), [
    ({"x": _lib.Tensor(0x10000, _lib.DTYPE_LABEL8, 8, 1)}, _lib.CTMR_ERR_INVALID),  # labels only feed a conv
    ({"y": None}, _lib.CTMR_ERR_INVALID),
    ({"y_dtype": _lib.DTYPE_LABEL8}, _lib.CTMR_ERR_INVALID),
    ({"y_channels": 16, "y_cstride": 16}, _lib.CTMR_ERR_INVALID),                    # narrower than the input
    ({"depth": 0}, _lib.CTMR_ERR_INVALID),
    ({"mode": _lib.TRANSFORM_TRILINEAR, "silu": 1}, _lib.CTMR_ERR_UNSUPPORTED),
    ({"mode": _lib.TRANSFORM_AVGPOOL, "width": 3}, _lib.CTMR_ERR_INVALID),
])
def test_transform_validation(overrides, status):
    assert _lib.LIB.ctmr_transform(ctypes.byref(_tdesc(**overrides)), None) == status
    assert _lib.LIB.ctmr_last_error()


def _fuse_desc(**kw) -> _lib.Conv3dDesc:
    """A 16-bit 64 -> 64 3x3x3 conv with an input affine + SiLU: a kh-concatenated-kernel call."""
    d = _lib.Conv3dDesc()
    d.batch, d.depth, d.height, d.width = 2, 8, 32, 32
    d.x = _lib.Tensor(0x10000000, _lib.DTYPE_F32, 64, 64)
    d.out_channels, d.kernel_size, d.stride = 64, 3, 1
    d.precision = _lib.PRECISION_FP16
    d.weight = 0x20000000
    d.y, d.y_dtype, d.y_cstride = 0x40000000, _lib.DTYPE_F32, 64
    d.affine, d.silu = 0x30000000, 1
    for k, v in kw.items():
        setattr(d, k, v)
    return d


def test_converter_warp_route_skips_the_operand_pass(monkeypatch):
    """With CTMR_KHCAT_FUSE=1 the kh-concatenated kernel converts its own operand: the call makes
    one launch (the conv) instead of two (operand pass + conv). The route is taken only where the
    converter warps can read the sources directly; everywhere else the operand pass stays."""
    count = lambda d: _lib.LIB.ctmr_conv3d_launch_count(ctypes.byref(d))  # noqa: E731
    monkeypatch.setenv("CTMR_KHCAT_FUSE", "0")
    assert count(_fuse_desc()) == 2
    monkeypatch.setenv("CTMR_KHCAT_FUSE", "1")
    assert count(_fuse_desc()) == 1
    assert count(_fuse_desc(affine=None, silu=0)) == 1  # a plain cast is folded as well
    # two sources split at a 64-channel boundary (the up path's virtual concat)
    assert count(_fuse_desc(x2=_lib.Tensor(0x50000000, _lib.DTYPE_F32, 64, 64), out_channels=48)) == 1
    kept = [
        _fuse_desc(y=0x10000000 + 64 * 4),                                   # output overlaps the source
        _fuse_desc(x=_lib.Tensor(0x10000004, _lib.DTYPE_F32, 64, 64)),        # source rows not 16-byte aligned
        _fuse_desc(affine=0x30000008),                                       # affine not 16-byte aligned
        _fuse_desc(x=_lib.Tensor(0x10000000, _lib.DTYPE_F32, 32, 32)),        # 32-channel blocks
        _fuse_desc(x2=_lib.Tensor(0x50000000, _lib.DTYPE_F32, 32, 32)),       # concat split inside a block
        _fuse_desc(x=_lib.Tensor(0x10000000, _lib.DTYPE_BF16, 64, 64)),       # bf16 source
        _fuse_desc(precision=_lib.PRECISION_FP32, weight_lo=0x50000000),     # split-fp32 operands
        _fuse_desc(precision=_lib.PRECISION_TF32),                           # TF32 operands
        _fuse_desc(trilinear=1, depth=4, height=16, width=16, affine=None, silu=0),  # resampled input
    ]
    for d in kept:
        assert count(d) == 2
