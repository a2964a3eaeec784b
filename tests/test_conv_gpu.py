"""Implicit-GEMM conv3d on the GPU against the float64 oracle.

Mirrors the reference's kernel tests (``tests/test_fast_fp32.py:59-150``): the
same five shapes (one per tiling branch there), seeds, weight scaling and the
reference's bar for the fp32 mode, ``atol = 2e-6 * max|ref|`` elementwise
(``tests/test_fast_fp32.py:18, 51-56``).

The bf16 mode rounds both operands to bf16 (relative rounding error RMS about
2^-9 each), which alone puts a single convolution's rel-L2 near 2e-3; a lone
conv is therefore held to 4e-3, while whole blocks (where the fp32 residual
dominates) are held to the stated 2e-3 in the block tests. fp16 operands carry
3 more mantissa bits: 6e-4 per conv; TF32 operands (10 mantissa bits, fp32 range) are held
to the fp16 bar.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import ops_ref

pytestmark = pytest.mark.gpu

RELATIVE = 2e-6
BF16_CONV_REL_L2 = 4e-3
FP16_CONV_REL_L2 = 6e-4

SHAPES = [
    ((2, 64, 8, 16, 16), 64, 1),
    ((2, 512, 4, 8, 8), 512, 1),
    ((2, 256, 8, 16, 16), 128, 1),
    ((1, 4, 8, 8, 8), 4, 1),
    ((1, 32, 8, 12, 16), 64, 2),
]


def _close_fp32(actual: torch.Tensor, expected: torch.Tensor) -> None:
    host = actual.detach().double().cpu()
    assert host.shape == expected.shape
    assert torch.isfinite(host).all()
    atol = RELATIVE * expected.abs().max().item()
    err = (host - expected).abs().max().item()
    assert err <= atol, f"max abs err {err:.3e} > {atol:.3e}"


def _inputs(shape, out_channels, seed=3):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal(shape).astype(np.float32)
    w = (rng.standard_normal((out_channels, shape[1], 3, 3, 3)) / np.sqrt(27 * shape[1])).astype(np.float32)
    b = rng.standard_normal(out_channels).astype(np.float32)
    return torch.from_numpy(x), torch.from_numpy(w), torch.from_numpy(b)


@pytest.mark.parametrize(("shape", "out_channels", "stride"), SHAPES)
def test_conv_fp32_matches_float64(cuda, shape, out_channels, stride):
    from ctmr_b200 import ops

    x, w, b = _inputs(shape, out_channels)
    packed = ops.pack_weight(w.to(cuda), "fp32")
    y = ops.conv3d(ops.to_ndhwc(x.to(cuda)), packed, b.to(cuda), stride=stride)
    torch.cuda.synchronize()
    expected = ops_ref.conv3d_ref(x.double(), w.double(), b.double(), stride=stride)
    _close_fp32(y, expected)


# Grids with at least half as many persistent tiles (8 h x 16 w of one depth, per N tile) as SMs: the
# fp32 mode runs on the atom-shifted kernel's split-precision variant there (3x3x3 with one and two N
# tiles, 1x1x1, the nearest-2x fold), held to the reference's bar like the per-tap kernel.
PERSISTENT_EXACT = [
    ((2, 64, 16, 32, 32), 64, 3, False),
    ((1, 96, 12, 32, 32), 128, 3, False),
    ((1, 32, 8, 32, 32), 256, 3, False),
    ((2, 64, 16, 32, 32), 48, 1, False),
    ((1, 64, 8, 16, 16), 64, 3, True),
]


@pytest.mark.parametrize(("shape", "out_channels", "k", "upsample"), PERSISTENT_EXACT)
def test_conv_fp32_persistent_kernel_matches_float64(cuda, shape, out_channels, k, upsample):
    from ctmr_b200 import ops

    rng = np.random.default_rng(11)
    x = torch.from_numpy(rng.standard_normal(shape).astype(np.float32))
    c = shape[1]
    w = torch.from_numpy((rng.standard_normal((out_channels, c, k, k, k)) / np.sqrt(k ** 3 * c)).astype(np.float32))
    b = torch.from_numpy(rng.standard_normal(out_channels).astype(np.float32))
    packed = ops.pack_weight(w.to(cuda), "fp32", upsample=upsample)
    y = ops.conv3d(ops.to_ndhwc(x.to(cuda)), packed, b.to(cuda))
    torch.cuda.synchronize()
    xin = ops_ref.upsample_nearest_ref(x.double()) if upsample else x.double()
    _close_fp32(y, ops_ref.conv3d_ref(xin, w.double(), b.double()))


@pytest.mark.parametrize("precision", ["bf16", "fp16", "tf32"])
@pytest.mark.parametrize(("shape", "out_channels", "stride"), SHAPES)
def test_conv_16bit_matches_float64(cuda, shape, out_channels, stride, precision):
    from ctmr_b200 import ops

    x, w, b = _inputs(shape, out_channels)
    packed = ops.pack_weight(w.to(cuda), precision)
    y = ops.conv3d(ops.to_ndhwc(x.to(cuda)), packed, b.to(cuda), stride=stride, out_dtype=torch.float32)
    torch.cuda.synchronize()
    expected = ops_ref.conv3d_ref(x.double(), w.double(), b.double(), stride=stride)
    err = ops_ref.rel_l2(y.cpu(), expected)
    assert err <= (BF16_CONV_REL_L2 if precision == "bf16" else FP16_CONV_REL_L2), f"{precision} rel-L2 {err:.3e}"


@pytest.mark.parametrize("upsample", [False, True])
def test_fused_norm_conv_matches_float64(cuda, upsample):
    """``tests/test_fast_fp32.py:91-127``: GN + SiLU (+ nearest 2x) + conv + per-batch bias + residual."""
    from ctmr_b200 import ops

    rng = np.random.default_rng(5)
    batch, channels, out_channels, groups = 2, 64, 32, 8
    x = (3 * rng.standard_normal((batch, channels, 4, 8, 8)) + 1).astype(np.float32)
    w = (rng.standard_normal((out_channels, channels, 3, 3, 3)) / np.sqrt(27 * channels)).astype(np.float32)
    batch_bias = rng.standard_normal((batch, out_channels)).astype(np.float32)
    norm_w = (1 + 0.1 * rng.standard_normal(channels)).astype(np.float32)
    norm_b = (0.1 * rng.standard_normal(channels)).astype(np.float32)
    scale = 2 if upsample else 1
    residual = rng.standard_normal((batch, out_channels, 4 * scale, 8 * scale, 8 * scale)).astype(np.float32)
    xt, wt = torch.from_numpy(x), torch.from_numpy(w)
    xg = ops.to_ndhwc(xt.to(cuda))
    affine = ops.group_norm_affine(xg, torch.from_numpy(norm_w).to(cuda), torch.from_numpy(norm_b).to(cuda),
                                   groups=groups, eps=1e-6)
    packed = ops.pack_weight(wt.to(cuda), "fp32", upsample=upsample)
    y = ops.conv3d(xg, packed, torch.from_numpy(batch_bias).to(cuda), affine=affine, silu=True,
                   residual=ops.to_ndhwc(torch.from_numpy(residual).to(cuda)))
    torch.cuda.synchronize()
    prepared = ops_ref.group_norm_silu_ref(xt.double(), torch.from_numpy(norm_w).double(),
                                           torch.from_numpy(norm_b).double(), groups)
    if upsample:
        prepared = ops_ref.upsample_nearest_ref(prepared)
    expected = ops_ref.conv3d_ref(prepared, wt.double())
    expected = expected + torch.from_numpy(batch_bias).double()[:, :, None, None, None] + torch.from_numpy(residual).double()
    _close_fp32(y, expected)


@pytest.mark.parametrize("shape", [(2, 24, 3, 5, 6), (1, 24, 1, 4, 4), (1, 24, 2, 3, 5), (1, 64, 5, 6, 8)])
def test_trilinear_conv_matches_materialized_upsampling(cuda, shape):
    """``tests/test_fast_fp32.py:130-150``: fused trilinear conv equals materialised trilinear + conv bitwise;
    one and two source depths exercise the depth walk's first and last outputs."""
    from ctmr_b200 import ops, _lib

    rng = np.random.default_rng(7)
    x = torch.from_numpy(rng.standard_normal(shape).astype(np.float32))
    c = shape[1]
    w = torch.from_numpy((rng.standard_normal((32, c, 3, 3, 3)) / np.sqrt(27 * c)).astype(np.float32))
    b = torch.from_numpy(rng.standard_normal(32).astype(np.float32))
    xg = ops.to_ndhwc(x.to(cuda))
    packed = ops.pack_weight(w.to(cuda), "fp32")
    fused = ops.conv3d(xg, packed, b.to(cuda), trilinear=True)
    up = ops.transform(xg, mode=_lib.TRANSFORM_TRILINEAR)
    materialized = ops.conv3d(up, packed, b.to(cuda))
    torch.cuda.synchronize()
    assert tuple(fused.shape) == (shape[0], 32, 2 * shape[2], 2 * shape[3], 2 * shape[4])
    assert torch.equal(fused.cpu(), materialized.cpu())
    # and the upsampling itself matches the oracle's half-pixel trilinear
    ref_up = ops_ref.upsample_trilinear_ref(x.double())
    assert (up.cpu().double() - ref_up).abs().max().item() < 1e-5
    expected = ops_ref.conv3d_ref(ref_up, w.double(), b.double())
    _close_fp32(fused, expected)


def test_no_device_wait_timed_out(cuda):
    from ctmr_b200 import _lib

    assert _lib.device_error(clear=True) == 0


V2_SHAPES = [
    ((2, 64, 3, 12, 24), 64, False),   # partial w, h and depth-pair tiles
    ((1, 32, 5, 16, 32), 48, False),   # 32-channel blocks, N = 48
    ((1, 128, 4, 8, 16), 256, False),  # two N tiles
    ((2, 64, 3, 8, 16), 32, True),     # nearest-2x fold (two taps along w per parity)
    ((1, 16, 2, 8, 16), 16, False),    # 16-channel blocks
]


@pytest.mark.parametrize("precision", ["fp16", "bf16", "tf32"])
@pytest.mark.parametrize(("shape", "out_channels", "upsample"), V2_SHAPES)
def test_persistent_kernel_shapes(cuda, shape, out_channels, upsample, precision):
    """16-bit stride-1 convs on grids with W >= 16 and H >= 8 run a persistent kernel (the
    kh-concatenated one for <= 64 output channels, else the atom-shifted one); bias per batch
    item and a residual exercise its epilogue."""
    from ctmr_b200 import ops

    rng = np.random.default_rng(13)
    x = torch.from_numpy(rng.standard_normal(shape).astype(np.float32))
    w = torch.from_numpy((rng.standard_normal((out_channels, shape[1], 3, 3, 3)) / np.sqrt(27 * shape[1]))
                         .astype(np.float32))
    bias = torch.from_numpy(rng.standard_normal((shape[0], out_channels)).astype(np.float32))
    scale = 2 if upsample else 1
    out_sp = tuple(scale * n for n in shape[2:])
    res = torch.from_numpy(rng.standard_normal((shape[0], out_channels, *out_sp)).astype(np.float32))
    packed = ops.pack_weight(w.to(cuda), precision, upsample=upsample)
    y = ops.conv3d(ops.to_ndhwc(x.to(cuda)), packed, bias.to(cuda), residual=ops.to_ndhwc(res.to(cuda)))
    torch.cuda.synchronize()
    xin = ops_ref.upsample_nearest_ref(x.double()) if upsample else x.double()
    expected = ops_ref.conv3d_ref(xin, w.double(), bias.double()) + res.double()
    err = ops_ref.rel_l2(y.cpu(), expected)
    assert err <= (FP16_CONV_REL_L2 if precision in ("fp16", "tf32") else BF16_CONV_REL_L2), f"{precision} rel-L2 {err:.3e}"


KHCAT_SHAPES = [
    ((2, 64, 3, 30, 20), 64),    # partial h (14 + 14 + 2 rows), w (8 + 8 + 4) and depth-pair tiles
    ((1, 128, 4, 16, 16), 48),   # two channel blocks, N = 3 x 48
    ((1, 32, 2, 8, 8), 16),      # 32-channel blocks, N = 3 x 16, smallest grid
    ((2, 192, 2, 14, 24), 64),   # three channel blocks, H = one tile
    ((2, 32, 4, 20, 24), 32),    # 32 outputs (4-lane transposed stores), partial h tile
]


@pytest.mark.parametrize("depths", ["1", "2"])
@pytest.mark.parametrize("precision", ["fp16", "bf16", "tf32"])
@pytest.mark.parametrize(("shape", "out_channels"), KHCAT_SHAPES)
def test_kh_concatenated_kernel(cuda, shape, out_channels, precision, depths, monkeypatch):
    """16-bit stride-1 3x3x3 convs with <= 64 output channels run the kh-concatenated kernel (the
    three taps along h side by side in one N = 3 x C_out MMA, row-shifted sums in the epilogue):
    per-batch bias, a residual and a bf16 output written into a channel slice exercise it, against
    the float64 oracle and against the atom-shifted kernel (CTMR_DISABLE_KHCAT) on the same inputs."""
    from ctmr_b200 import ops

    rng = np.random.default_rng(57)
    b, c = shape[:2]
    x = torch.from_numpy(rng.standard_normal(shape).astype(np.float32))
    w = torch.from_numpy((rng.standard_normal((out_channels, c, 3, 3, 3)) / np.sqrt(27 * c)).astype(np.float32))
    bias = torch.from_numpy(rng.standard_normal((b, out_channels)).astype(np.float32))
    res = torch.from_numpy(rng.standard_normal((b, out_channels, *shape[2:])).astype(np.float32))
    xc, bc, rc = ops.to_ndhwc(x.to(cuda)), bias.to(cuda), ops.to_ndhwc(res.to(cuda))
    packed = ops.pack_weight(w.to(cuda), precision)
    monkeypatch.delenv("CTMR_DISABLE_KHCAT", raising=False)
    monkeypatch.setenv("CTMR_KHCAT_MT", depths)  # depth tiles per weight box (1: two accumulator buffers)
    y = ops.conv3d(xc, packed, bc, residual=rc)
    plain = ops.conv3d(xc, packed, bc)
    wide = ops.empty_ndhwc(b, out_channels + 32, *shape[2:], torch.bfloat16, xc.device).zero_()
    ops.conv3d(xc, packed, bc, out=wide[:, 16:16 + out_channels])
    monkeypatch.setenv("CTMR_DISABLE_KHCAT", "1")
    y_v2 = ops.conv3d(xc, packed, bc, residual=rc)
    monkeypatch.delenv("CTMR_DISABLE_KHCAT")
    torch.cuda.synchronize()
    expected = ops_ref.conv3d_ref(x.double(), w.double(), bias.double()) + res.double()
    err = ops_ref.rel_l2(y.cpu(), expected)
    assert err <= (FP16_CONV_REL_L2 if precision in ("fp16", "tf32") else BF16_CONV_REL_L2), f"{precision} rel-L2 {err:.3e}"
    # Same rounded operands, fp32 sums in another order: the two kernels agree to fp32 rounding,
    # and do not agree bitwise (which would mean the route switch changed nothing).
    diff = ops_ref.rel_l2(y.cpu(), y_v2.cpu().double())
    assert diff <= 1e-5, f"kh-concatenated vs atom-shifted rel-L2 {diff:.3e}"
    assert not torch.equal(y, y_v2)
    # bf16 output into a channel slice: the fp32 result rounded once; the other channels untouched.
    torch.testing.assert_close(wide[:, 16:16 + out_channels].float(), plain.to(torch.bfloat16).float(),
                               rtol=0, atol=0)
    assert not wide[:, :16].any() and not wide[:, 16 + out_channels:].any()


KHCAT_PAIR_SHAPES = [
    (2, 64, 3, 30, 20),    # 36 tiles: partial h, w and depth-pair tiles
    (1, 64, 2, 14, 24),    # 3 tiles: the last pair's second CTA repeats a tile and stores nothing
    (2, 192, 2, 14, 24),   # three channel blocks
    (1, 128, 6, 44, 40),   # 60 tiles, two channel blocks
    (1, 64, 8, 128, 64),   # 320 tiles: each CTA pair walks several pair tiles
]


def _kernel_names(fn) -> list[str]:
    """Names of the CUDA kernels `fn` launches (torch's profiler, CUDA activity)."""
    from torch.profiler import ProfilerActivity, profile

    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        fn()
        torch.cuda.synchronize()
    return [e.name for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA]


@pytest.mark.parametrize("precision", ["fp16", "bf16"])
@pytest.mark.parametrize("shape", KHCAT_PAIR_SHAPES)
def test_kh_concatenated_pair_kernel(cuda, shape, precision, monkeypatch):
    """With CTMR_KHCAT_PAIR=1, 64 -> 64 convs in 64-channel blocks run the CTA-pair kernel
    (tcgen05.mma.cta_group::2, M = 256: two tiles per product, each SM holding half of every weight
    box): it is the kernel launched, it meets the float64 oracle at the 16-bit bar, and it agrees with
    the one-SM kernel (the default) on the same rounded operands, with a bias, a residual and a bf16
    output into a channel slice."""
    from ctmr_b200 import ops

    rng = np.random.default_rng(64)
    b, c = shape[:2]
    x = torch.from_numpy(rng.standard_normal(shape).astype(np.float32))
    w = torch.from_numpy((rng.standard_normal((64, c, 3, 3, 3)) / np.sqrt(27 * c)).astype(np.float32))
    bias = torch.from_numpy(rng.standard_normal(64).astype(np.float32))
    res = torch.from_numpy(rng.standard_normal((b, 64, *shape[2:])).astype(np.float32))
    xc, bc, rc = ops.to_ndhwc(x.to(cuda)), bias.to(cuda), ops.to_ndhwc(res.to(cuda))
    packed = ops.pack_weight(w.to(cuda), precision)
    monkeypatch.delenv("CTMR_DISABLE_KHCAT", raising=False)
    monkeypatch.delenv("CTMR_KHCAT_MT", raising=False)
    monkeypatch.setenv("CTMR_KHCAT_PAIR", "1")
    out = {}
    names = _kernel_names(lambda: out.setdefault("y", ops.conv3d(xc, packed, bc, residual=rc)))
    assert any("khcat_pair" in n for n in names), names
    y = out["y"]
    wide = ops.empty_ndhwc(b, 96, *shape[2:], torch.bfloat16, xc.device).zero_()
    ops.conv3d(xc, packed, bc, out=wide[:, 16:80])
    monkeypatch.delenv("CTMR_KHCAT_PAIR")
    names_one = _kernel_names(lambda: out.setdefault("y_one", ops.conv3d(xc, packed, bc, residual=rc)))
    assert not any("khcat_pair" in n for n in names_one) and any("khcat_kernel" in n for n in names_one), names_one
    y_one = out["y_one"]
    plain_one = ops.conv3d(xc, packed, bc)
    torch.cuda.synchronize()
    expected = ops_ref.conv3d_ref(x.double(), w.double(), bias.double()) + res.double()
    err = ops_ref.rel_l2(y.cpu(), expected)
    assert err <= (FP16_CONV_REL_L2 if precision == "fp16" else BF16_CONV_REL_L2), f"{precision} rel-L2 {err:.3e}"
    diff = ops_ref.rel_l2(y.cpu(), y_one.cpu().double())
    assert diff <= 1e-6, f"pair vs one-SM kernel rel-L2 {diff:.3e}"
    torch.testing.assert_close(wide[:, 16:80].float(), plain_one.to(torch.bfloat16).float(), rtol=8e-3, atol=1e-3)
    assert not wide[:, :16].any() and not wide[:, 80:].any()


@pytest.mark.parametrize("out_channels", [64, 48])
def test_kh_concatenated_residual_forms(cuda, out_channels, monkeypatch):
    """The kh-concatenated kernel's two store paths (64 outputs: 8-lane transposed; fewer: per
    voxel) with a bf16 residual and with a residual on the half-resolution grid (nearest-upsampled
    in the epilogue): each against the float64 oracle and against the atom-shifted kernel."""
    from ctmr_b200 import ops

    rng = np.random.default_rng(91)
    shape = (2, 64, 4, 18, 16)
    b, c = shape[:2]
    x = torch.from_numpy(rng.standard_normal(shape).astype(np.float32))
    w = torch.from_numpy((rng.standard_normal((out_channels, c, 3, 3, 3)) / np.sqrt(27 * c)).astype(np.float32))
    bias = torch.from_numpy(rng.standard_normal(out_channels).astype(np.float32))
    res_full = torch.from_numpy(rng.standard_normal((b, out_channels, *shape[2:])).astype(np.float32))
    res_half = torch.from_numpy(rng.standard_normal((b, out_channels, 2, 9, 8)).astype(np.float32))
    xc = ops.to_ndhwc(x.to(cuda))
    packed = ops.pack_weight(w.to(cuda), "fp16")
    res_bf16 = ops.to_ndhwc(res_full.to(cuda)).to(torch.bfloat16)
    res_half_dev = ops.to_ndhwc(res_half.to(cuda))
    conv = ops_ref.conv3d_ref(x.double(), w.double(), bias.double())
    cases = [
        (dict(residual=res_bf16), conv + res_bf16.double().cpu()),
        (dict(residual=res_half_dev, residual_upsampled=True), conv + ops_ref.upsample_nearest_ref(res_half.double())),
    ]
    for kw, expected in cases:
        monkeypatch.delenv("CTMR_DISABLE_KHCAT", raising=False)
        y = ops.conv3d(xc, packed, bias.to(cuda), **kw)
        monkeypatch.setenv("CTMR_DISABLE_KHCAT", "1")
        y_v2 = ops.conv3d(xc, packed, bias.to(cuda), **kw)
        monkeypatch.delenv("CTMR_DISABLE_KHCAT")
        torch.cuda.synchronize()
        err = ops_ref.rel_l2(y.cpu(), expected)
        assert err <= FP16_CONV_REL_L2, f"{sorted(kw)} rel-L2 {err:.3e}"
        diff = ops_ref.rel_l2(y.cpu(), y_v2.cpu().double())
        assert diff <= 1e-5, f"{sorted(kw)} kh-concatenated vs atom-shifted rel-L2 {diff:.3e}"
        assert not torch.equal(y, y_v2)


@pytest.mark.parametrize("precision", ["fp16", "bf16", "tf32"])
@pytest.mark.parametrize(("shape", "x2_channels", "out_channels"), [
    ((2, 64, 3, 12, 24), 128, 64),   # skip 1x1 over cat(hidden, skip): partial tiles, two sources
    ((1, 128, 4, 16, 32), 0, 64),    # VAE shortcut class
    ((1, 32, 2, 8, 16), 0, 256),     # two N tiles
])
def test_persistent_pointwise_conv(cuda, shape, x2_channels, out_channels, precision):
    """16-bit 1x1x1 convs on grids with W >= 16 and H >= 8 run the persistent kernel (one box per
    channel block); a virtual concat input, per-batch bias and a residual exercise its paths."""
    from ctmr_b200 import ops

    rng = np.random.default_rng(31)
    b, c = shape[:2]
    x = torch.from_numpy(rng.standard_normal(shape).astype(np.float32))
    x2 = torch.from_numpy(rng.standard_normal((b, x2_channels, *shape[2:])).astype(np.float32)) if x2_channels else None
    cin = c + x2_channels
    w = torch.from_numpy((rng.standard_normal((out_channels, cin, 1, 1, 1)) / np.sqrt(cin)).astype(np.float32))
    bias = torch.from_numpy(rng.standard_normal((b, out_channels)).astype(np.float32))
    res = torch.from_numpy(rng.standard_normal((b, out_channels, *shape[2:])).astype(np.float32))
    y = ops.conv3d(ops.to_ndhwc(x.to(cuda)), ops.pack_weight(w.to(cuda), precision), bias.to(cuda),
                   x2=ops.to_ndhwc(x2.to(cuda)) if x2 is not None else None, residual=ops.to_ndhwc(res.to(cuda)))
    torch.cuda.synchronize()
    xin = torch.cat([x, x2], dim=1) if x2 is not None else x
    expected = ops_ref.conv3d_ref(xin.double(), w.double(), bias.double(), padding=0) + res.double()
    err = ops_ref.rel_l2(y.cpu(), expected)
    assert err <= (FP16_CONV_REL_L2 if precision in ("fp16", "tf32") else BF16_CONV_REL_L2), f"{precision} rel-L2 {err:.3e}"


@pytest.mark.parametrize("precision", ["fp32", "fp16"])
@pytest.mark.parametrize(("shape", "out_channels", "norm"), [
    ((2, 4, 8, 16, 12), 64, False),   # the UNet / ControlNet conv_in class
    ((1, 4, 5, 7, 9), 256, False),    # the VAE decoder conv_in class, two N tiles, odd extents
    ((1, 3, 4, 6, 8), 32, True),      # 3 channels with group-norm affine + SiLU
    ((1, 1, 3, 5, 4), 16, False),     # one channel
])
def test_tiny_input_im2col(cuda, shape, out_channels, norm, precision):
    """3x3x3 convs of <= 4 input channels: the fp32 mode runs the direct FMA kernel, the 16-bit
    modes a 1x1x1 GEMM over im2col rows of 27 * C columns."""
    from ctmr_b200 import ops

    rng = np.random.default_rng(37)
    b, c = shape[:2]
    x = torch.from_numpy(rng.standard_normal(shape).astype(np.float32))
    w = torch.from_numpy((rng.standard_normal((out_channels, c, 3, 3, 3)) / np.sqrt(27 * c)).astype(np.float32))
    bias = torch.from_numpy(rng.standard_normal(out_channels).astype(np.float32))
    res = torch.from_numpy(rng.standard_normal((b, out_channels, *shape[2:])).astype(np.float32))
    kw = {}
    xin = x.double()
    if norm:
        affine = torch.from_numpy(np.stack([1 + 0.2 * rng.standard_normal((b, c)), 0.3 * rng.standard_normal((b, c))],
                                           axis=-1).astype(np.float32))
        kw = {"affine": affine.to(cuda), "silu": True}
        a = affine.double()
        xin = ops_ref.silu_ref(xin * a[..., 0][..., None, None, None] + a[..., 1][..., None, None, None])
    y = ops.conv3d(ops.to_ndhwc(x.to(cuda)), ops.pack_weight(w.to(cuda), precision), bias.to(cuda),
                   residual=ops.to_ndhwc(res.to(cuda)), **kw)
    torch.cuda.synchronize()
    expected = ops_ref.conv3d_ref(xin, w.double(), bias.double()) + res.double()
    if precision == "fp32":
        _close_fp32(y, expected)
    else:
        assert ops_ref.rel_l2(y.cpu(), expected) <= FP16_CONV_REL_L2


@pytest.mark.parametrize("precision", ["fp32", "fp16", "tf32"])
def test_splitk_reduction_epilogue(cuda, precision):
    """A deep, small grid (2 x 256 x 4^3) splits K across CTAs; the reduction adds the
    per-batch bias and the residual before the single rounding."""
    from ctmr_b200 import ops

    rng = np.random.default_rng(17)
    x = torch.from_numpy(rng.standard_normal((2, 256, 4, 4, 4)).astype(np.float32))
    w = torch.from_numpy((rng.standard_normal((256, 256, 3, 3, 3)) / np.sqrt(27 * 256)).astype(np.float32))
    bias = torch.from_numpy(rng.standard_normal((2, 256)).astype(np.float32))
    res = torch.from_numpy(rng.standard_normal((2, 256, 4, 4, 4)).astype(np.float32))
    y = ops.conv3d(ops.to_ndhwc(x.to(cuda)), ops.pack_weight(w.to(cuda), precision), bias.to(cuda),
                   residual=ops.to_ndhwc(res.to(cuda)))
    torch.cuda.synchronize()
    expected = ops_ref.conv3d_ref(x.double(), w.double(), bias.double()) + res.double()
    if precision == "fp32":
        _close_fp32(y, expected)
    else:
        assert ops_ref.rel_l2(y.cpu(), expected) <= FP16_CONV_REL_L2


@pytest.mark.parametrize(("shape", "out_channels", "silu"), [
    ((2, 64, 5, 12, 40), 4, True),   # UNet out.2 shape class, partial blocks on every axis
    ((1, 64, 8, 16, 16), 1, False),  # VAE decoder output conv
    ((1, 24, 3, 9, 7), 3, True),     # fewer channels than one 32-channel staging slice
    ((1, 64, 21, 34, 70), 1, True),  # several h / w columns and depth chunks, one output channel
    ((1, 30, 6, 17, 33), 2, True),   # channels not a multiple of 4 (scalar staging), two outputs
    ((2, 72, 7, 16, 32), 1, False),  # two staging slices plus a partial one
])
def test_narrow_output_conv(cuda, shape, out_channels, silu):
    """<= 4 output channels run the direct fp32 kernel (GN affine + SiLU applied while staging);
    held to the reference's fp32 bar."""
    from ctmr_b200 import ops

    rng = np.random.default_rng(19)
    b, c = shape[:2]
    x = torch.from_numpy((2 * rng.standard_normal(shape) + 0.5).astype(np.float32))
    w = torch.from_numpy((rng.standard_normal((out_channels, c, 3, 3, 3)) / np.sqrt(27 * c)).astype(np.float32))
    bias = torch.from_numpy(rng.standard_normal((b, out_channels)).astype(np.float32))
    res = torch.from_numpy(rng.standard_normal((b, out_channels, *shape[2:])).astype(np.float32))
    norm_w = torch.from_numpy((1 + 0.1 * rng.standard_normal(c)).astype(np.float32))
    norm_b = torch.from_numpy((0.1 * rng.standard_normal(c)).astype(np.float32))
    groups = 8 if c % 8 == 0 else 2
    xg = ops.to_ndhwc(x.to(cuda))
    affine = ops.group_norm_affine(xg, norm_w.to(cuda), norm_b.to(cuda), groups=groups, eps=1e-6)
    y = ops.conv3d(xg, ops.pack_weight(w.to(cuda), "fp32"), bias.to(cuda), affine=affine, silu=silu,
                   residual=ops.to_ndhwc(res.to(cuda)))
    torch.cuda.synchronize()
    prepared = ops_ref.group_norm_ref(x.double(), norm_w.double(), norm_b.double(), groups, 1e-6)
    if silu:
        prepared = ops_ref.silu_ref(prepared)
    expected = ops_ref.conv3d_ref(prepared, w.double(), bias.double()) + res.double()
    _close_fp32(y, expected)


@pytest.mark.parametrize("mode", ["trilinear", "avgpool"])
def test_narrow_output_with_resampled_input(cuda, mode):
    """A <= 4-channel conv of a trilinear-upsampled or pooled input still prepares the operand."""
    from ctmr_b200 import ops

    rng = np.random.default_rng(23)
    x = torch.from_numpy(rng.standard_normal((1, 8, 4, 6, 8)).astype(np.float32))
    w = torch.from_numpy((rng.standard_normal((4, 8, 3, 3, 3)) / np.sqrt(27 * 8)).astype(np.float32))
    xg = ops.to_ndhwc(x.to(cuda))
    y = ops.conv3d(xg, ops.pack_weight(w.to(cuda), "fp32"), None, **{mode: True})
    torch.cuda.synchronize()
    xin = ops_ref.upsample_trilinear_ref(x.double()) if mode == "trilinear" else ops_ref.avg_pool_ref(x.double())
    _close_fp32(y, ops_ref.conv3d_ref(xin, w.double()))


def test_narrow_output_with_half_grid_residual(cuda):
    """The UNet up-block conv2 adds its skip from the half-resolution grid (nearest 2x by index)."""
    from ctmr_b200 import ops

    rng = np.random.default_rng(29)
    x = torch.from_numpy(rng.standard_normal((2, 8, 4, 6, 8)).astype(np.float32))
    w = torch.from_numpy((rng.standard_normal((4, 8, 3, 3, 3)) / np.sqrt(27 * 8)).astype(np.float32))
    res = torch.from_numpy(rng.standard_normal((2, 4, 2, 3, 4)).astype(np.float32))
    y = ops.conv3d(ops.to_ndhwc(x.to(cuda)), ops.pack_weight(w.to(cuda), "fp32"), None,
                   residual=ops.to_ndhwc(res.to(cuda)), residual_upsampled=True)
    torch.cuda.synchronize()
    expected = ops_ref.conv3d_ref(x.double(), w.double()) + ops_ref.upsample_nearest_ref(res.double())
    _close_fp32(y, expected)


@pytest.mark.parametrize("precision", ["fp16", "bf16"])
@pytest.mark.parametrize(("shape", "out_channels", "upsample", "k"), [
    ((2, 64, 3, 12, 24), 128, False, 3),  # partial tiles, batch 2
    ((1, 32, 2, 8, 16), 192, False, 3),   # 192 channels: N tiles of 128 + 64
    ((2, 64, 3, 8, 16), 128, True, 3),    # nearest-2x fold: every parity writes its voxels
    ((1, 128, 4, 16, 32), 256, False, 1), # 1x1x1, two N tiles
    ((2, 64, 3, 30, 20), 64, False, 3),   # kh-concatenated kernel (four slots per CTA), partial tiles
    ((2, 64, 2, 14, 24), 64, False, 3),   # ... six tiles: CTAs that see one batch item zero the other's slots
    ((2, 64, 8, 64, 64), 64, False, 3),   # ... 320 tiles: CTAs walk several tiles across the batch change
    ((1, 128, 6, 44, 40), 64, False, 3),  # ... two input channel blocks
])
def test_output_statistics_match_a_pass(cuda, shape, out_channels, upsample, k, precision):
    """GroupNorm moments reduced in the persistent kernel's epilogue give the affine of a separate
    statistics pass over the stored output (and over a virtual concat of two such outputs)."""
    from ctmr_b200 import ops

    rng = np.random.default_rng(41)
    b, c = shape[:2]
    x = ops.to_ndhwc(torch.from_numpy(rng.standard_normal(shape).astype(np.float32)).to(cuda))
    w = torch.from_numpy((rng.standard_normal((out_channels, c, k, k, k)) / np.sqrt(c * k ** 3)).astype(np.float32))
    bias = torch.from_numpy(rng.standard_normal((b, out_channels)).astype(np.float32) + 3.0).to(cuda)
    packed = ops.pack_weight(w.to(cuda), precision, upsample=upsample)
    y = ops.conv3d(x, packed, bias, stats=True)
    assert ops.output_stats(y) is not None, "the persistent kernel should produce statistics here"
    gamma = torch.from_numpy(rng.standard_normal(out_channels).astype(np.float32)).to(cuda)
    beta = torch.from_numpy(rng.standard_normal(out_channels).astype(np.float32)).to(cuda)
    fused = ops.group_norm_affine(y, gamma, beta, groups=16, eps=1e-6)
    plain = ops.group_norm_affine(y.clone(), gamma, beta, groups=16, eps=1e-6)  # no statistics attached
    torch.cuda.synchronize()
    torch.testing.assert_close(fused, plain, rtol=2e-5, atol=1e-6)
    # Concat of two outputs (the UNet up path's cat(hidden, skip)), groups spanning the boundary.
    y2 = ops.conv3d(x, packed, bias * 0.5, stats=True)
    g2 = 2 * out_channels // 8 if (2 * out_channels) % 8 == 0 else 2
    cat_gamma = torch.cat([gamma, gamma])
    fused = ops.group_norm_affine(y, cat_gamma, None, groups=g2, eps=1e-6, x2=y2)
    plain = ops.group_norm_affine(y.clone(), cat_gamma, None, groups=g2, eps=1e-6, x2=y2.clone())
    torch.cuda.synchronize()
    torch.testing.assert_close(fused, plain, rtol=2e-5, atol=1e-6)


def test_output_statistics_refused_where_unsupported(cuda):
    """A conv that does not run the persistent kernel reports no slots and attaches nothing."""
    from ctmr_b200 import ops

    x = ops.to_ndhwc(torch.randn((1, 64, 4, 8, 8), device=cuda))
    w = torch.randn((4, 64, 3, 3, 3), device=cuda) / 40
    y = ops.conv3d(x, ops.pack_weight(w, "fp32"), None, stats=True)  # narrow fp32 kernel
    assert ops.output_stats(y) is None
    w = torch.randn((48, 64, 3, 3, 3), device=cuda) / 40
    y = ops.conv3d(ops.to_ndhwc(torch.randn((1, 64, 4, 8, 16), device=cuda)), ops.pack_weight(w, "fp16"), None,
                   stats=True)  # 48 outputs: the kh-concatenated kernel's per-voxel stores keep none
    assert ops.output_stats(y) is None
    w = torch.randn((64, 64, 3, 3, 3), device=cuda) / 40
    y = ops.conv3d(ops.to_ndhwc(torch.randn((1, 64, 4, 8, 16), device=cuda)), ops.pack_weight(w, "tf32"), None,
                   stats=True)  # TF32 operands: the kh-concatenated kernel keeps none
    assert ops.output_stats(y) is None


def test_output_statistics_after_residual_and_norm(cuda):
    """The kh-concatenated kernel's statistics describe the stored output: GroupNorm affine + SiLU on
    the input, bias and a residual added in the epilogue (the VAE residual block's conv2), against a
    statistics pass over the output; a second conv then consumes the affine from those statistics."""
    from ctmr_b200 import ops

    rng = np.random.default_rng(43)
    shape = (1, 64, 6, 40, 48)
    x = ops.to_ndhwc(torch.from_numpy((rng.standard_normal(shape) * 1.5 + 0.4).astype(np.float32)).to(cuda))
    res = ops.to_ndhwc(torch.from_numpy(rng.standard_normal(shape).astype(np.float32)).to(cuda))
    w = torch.from_numpy((rng.standard_normal((64, 64, 3, 3, 3)) / np.sqrt(27 * 64)).astype(np.float32)).to(cuda)
    gamma = torch.from_numpy((1 + 0.2 * rng.standard_normal(64)).astype(np.float32)).to(cuda)
    beta = torch.from_numpy((0.3 * rng.standard_normal(64)).astype(np.float32)).to(cuda)
    bias = torch.from_numpy(rng.standard_normal(64).astype(np.float32)).to(cuda)
    packed = ops.pack_weight(w, "fp16")
    y = ops.conv3d(x, packed, bias, norm=(gamma, beta, 32, 1e-6), silu=True, residual=res, stats=True)
    assert ops.output_stats(y) is not None
    fused = ops.group_norm_affine(y, gamma, beta, groups=32, eps=1e-6)
    plain = ops.group_norm_affine(y.clone(), gamma, beta, groups=32, eps=1e-6)
    z_fused = ops.conv3d(y, packed, bias, affine=fused, silu=True)
    z_plain = ops.conv3d(y, packed, bias, affine=plain, silu=True)
    torch.cuda.synchronize()
    torch.testing.assert_close(fused, plain, rtol=2e-5, atol=1e-6)
    assert ops_ref.rel_l2(z_fused.cpu(), z_plain.cpu().double()) <= 1e-5


@pytest.mark.parametrize(("shape", "x2_channels", "out_channels", "precision", "groups"), [
    ((2, 512, 4, 8, 8), 0, 512, "fp16", 32),      # deep level (fused small-tensor kernel if enabled)
    ((2, 256, 4, 8, 8), 256, 256, "fp16", 32),    # concat input
    ((1, 64, 16, 32, 64), 0, 64, "fp16", 32),     # large: statistics pass + operand pass
    ((1, 64, 16, 32, 64), 32, 64, "bf16", 32),    # large with concat
    ((2, 24, 3, 5, 7), 0, 32, "fp32", 8),         # split-fp32 operand, padded channels 24..31 zeroed
    ((1, 64, 5, 12, 40), 0, 4, "fp32", 32),       # narrow fp32 kernel takes the affine from the workspace
])
@pytest.mark.parametrize("fused", [False, True])
def test_groupnorm_inside_the_conv_call(cuda, shape, x2_channels, out_channels, precision, groups, fused,
                                        monkeypatch):
    """``conv3d(norm=...)`` (statistics computed inside the call, also through the opt-in fused
    small-tensor kernel) equals ``conv3d(affine=...)`` with the affine of ``ctmr_group_norm_affine``."""
    from ctmr_b200 import ops

    if fused:
        monkeypatch.setenv("CTMR_GN_FUSED", "1")
    else:
        monkeypatch.delenv("CTMR_GN_FUSED", raising=False)

    rng = np.random.default_rng(47)
    b, c = shape[:2]
    x = ops.to_ndhwc(torch.from_numpy((rng.standard_normal(shape) * 2 + 0.7).astype(np.float32)).to(cuda))
    x2 = None
    if x2_channels:
        x2 = ops.to_ndhwc(torch.from_numpy(rng.standard_normal((b, x2_channels, *shape[2:])).astype(np.float32))
                          .to(cuda))
    cin = c + x2_channels
    w = torch.from_numpy((rng.standard_normal((out_channels, cin, 3, 3, 3)) / np.sqrt(27 * cin)).astype(np.float32))
    gamma = torch.from_numpy((1 + 0.2 * rng.standard_normal(cin)).astype(np.float32)).to(cuda)
    beta = torch.from_numpy((0.3 * rng.standard_normal(cin)).astype(np.float32)).to(cuda)
    bias = torch.from_numpy(rng.standard_normal(out_channels).astype(np.float32)).to(cuda)
    packed = ops.pack_weight(w.to(cuda), precision)
    affine = ops.group_norm_affine(x, gamma, beta, groups=groups, eps=1e-6, x2=x2)
    ref = ops.conv3d(x, packed, bias, x2=x2, affine=affine, silu=True)
    got = ops.conv3d(x, packed, bias, x2=x2, norm=(gamma, beta, groups, 1e-6), silu=True)
    torch.cuda.synchronize()
    err = ops_ref.rel_l2(got.cpu(), ref.cpu().double())
    assert err <= (1e-6 if precision == "fp32" else 1e-3), f"{precision} rel-L2 {err:.3e}"


GN_DIRECT_CASES = [
    ((2, 512, 4, 8, 8), 0, 32),       # 16 channels per group: shuffle-xor tree
    ((2, 256, 8, 16, 16), 128, 32),   # virtual concat, 12 channels per group: lane-ordered sums
    ((1, 128, 8, 32, 32), 0, 32),     # 4 channels per group over 8,192 voxels: eight 16-byte loads
    ((2, 64, 8, 16, 32), 0, 32),      # 2 channels per group: eight 4-byte loads
    ((2, 1024, 4, 8, 8), 512, 32),    # 48 channels per group
    ((1, 24, 3, 5, 7), 0, 8),         # 3 channels per group, 85 lanes, odd extents
]


@pytest.mark.parametrize(("shape", "x2_channels", "groups"), GN_DIRECT_CASES)
def test_group_norm_small_tensor_kernel(cuda, shape, x2_channels, groups, monkeypatch):
    """Small GroupNorms (a group that 1024 threads read with at most eight loads each) run one kernel,
    one block per group and batch item: it is the kernel launched, its affine matches float64 and the
    two-pass path (CTMR_DISABLE_GN_DIRECT), and it is bitwise reproducible."""
    from ctmr_b200 import _lib, ops

    rng = np.random.default_rng(73)
    b, c = shape[:2]
    xh = (rng.standard_normal(shape) * 2 + 0.7).astype(np.float32)
    x2h = rng.standard_normal((b, x2_channels, *shape[2:])).astype(np.float32) if x2_channels else None
    x = ops.to_ndhwc(torch.from_numpy(xh).to(cuda))
    x2 = ops.to_ndhwc(torch.from_numpy(x2h).to(cuda)) if x2_channels else None
    ctot = c + x2_channels
    gamma = torch.from_numpy((1 + 0.2 * rng.standard_normal(ctot)).astype(np.float32)).to(cuda)
    beta = torch.from_numpy((0.3 * rng.standard_normal(ctot)).astype(np.float32)).to(cuda)
    voxels = int(np.prod(shape[2:]))
    monkeypatch.delenv("CTMR_DISABLE_GN_DIRECT", raising=False)
    assert _lib.LIB.ctmr_group_norm_launch_count(voxels, ctot, groups) == 1
    out = {}
    names = _kernel_names(lambda: out.setdefault(
        "direct", ops.group_norm_affine(x, gamma, beta, groups=groups, eps=1e-6, x2=x2)))
    assert any("gn_direct" in n for n in names) and not any("gn_partial" in n for n in names), names
    direct = out["direct"]
    again = ops.group_norm_affine(x, gamma, beta, groups=groups, eps=1e-6, x2=x2)
    monkeypatch.setenv("CTMR_DISABLE_GN_DIRECT", "1")
    assert _lib.LIB.ctmr_group_norm_launch_count(voxels, ctot, groups) == 2
    two_pass = ops.group_norm_affine(x, gamma, beta, groups=groups, eps=1e-6, x2=x2)
    monkeypatch.delenv("CTMR_DISABLE_GN_DIRECT")
    torch.cuda.synchronize()
    assert torch.equal(direct, again)
    full = np.concatenate([xh, x2h], axis=1) if x2_channels else xh
    xg = full.astype(np.float64).reshape(b, groups, -1)
    cpg = ctot // groups
    mean = np.repeat(xg.mean(axis=2), cpg, axis=1)
    rstd = np.repeat(1.0 / np.sqrt(xg.var(axis=2) + 1e-6), cpg, axis=1)
    scale = gamma.double().cpu().numpy()[None, :] * rstd
    offset = beta.double().cpu().numpy()[None, :] - mean * scale
    expected = torch.from_numpy(np.stack([scale, offset], axis=-1))
    torch.testing.assert_close(direct.cpu().double(), expected, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(direct, two_pass, rtol=2e-6, atol=2e-6)


@pytest.mark.parametrize("shape", [(2, 64, 3, 16, 16), (2, 32, 2, 8, 16)])
def test_bias_rows_read_in_place(cuda, shape):
    """A per-batch bias that is a column slice of a wider table (bias_row_stride) gives the same
    output, bitwise, as the same bias made contiguous."""
    from ctmr_b200 import ops

    rng = np.random.default_rng(61)
    b, c = shape[:2]
    o = 48
    x = ops.to_ndhwc(torch.from_numpy(rng.standard_normal(shape).astype(np.float32)).to(cuda))
    w = torch.from_numpy((rng.standard_normal((o, c, 3, 3, 3)) / np.sqrt(27 * c)).astype(np.float32)).to(cuda)
    table = torch.from_numpy(rng.standard_normal((b, 200)).astype(np.float32)).to(cuda)
    sliced = table[:, 37:37 + o]
    assert not sliced.is_contiguous()
    packed = ops.pack_weight(w, "fp16")
    y_slice = ops.conv3d(x, packed, sliced)
    y_dense = ops.conv3d(x, packed, sliced.contiguous())
    torch.cuda.synchronize()
    assert torch.equal(y_slice, y_dense)


def test_transform_fp16_output(cuda):
    """GroupNorm transform written in fp16 equals the fp32 transform rounded once (attention tokens)."""
    from ctmr_b200 import ops

    rng = np.random.default_rng(67)
    x = ops.to_ndhwc(torch.from_numpy(rng.standard_normal((2, 64, 4, 8, 8)).astype(np.float32)).to(cuda))
    gamma = torch.from_numpy(rng.standard_normal(64).astype(np.float32)).to(cuda)
    beta = torch.from_numpy(rng.standard_normal(64).astype(np.float32)).to(cuda)
    affine = ops.group_norm_affine(x, gamma, beta, groups=32, eps=1e-6)
    y32 = ops.transform(x, affine=affine, out_dtype=torch.float32)
    y16 = ops.transform(x, affine=affine, out_dtype=torch.float16)
    torch.cuda.synchronize()
    assert y16.dtype == torch.float16
    assert torch.equal(y16, y32.to(torch.float16))


@pytest.mark.parametrize("precision", ["fp32", "bf16", "fp16", "tf32"])
@pytest.mark.parametrize(("o", "c", "k", "upsample"), [(48, 64, 3, False), (32, 16, 3, True), (20, 24, 3, False)])
def test_channels_last_weight_packs_identically(cuda, o, c, k, upsample, precision):
    """A weight stored channels-last (O, k, k, k, C) — a released checkpoint's layout, seen through
    a Torch-layout view — packs to the same bits as the Torch-layout weight."""
    from ctmr_b200 import ops

    g = torch.Generator().manual_seed(71)
    w = torch.randn(o, c, k, k, k, generator=g)
    view = w.permute(0, 2, 3, 4, 1).contiguous().permute(0, 4, 1, 2, 3).to(cuda)
    assert view.is_contiguous(memory_format=torch.channels_last_3d) and not view.is_contiguous()
    a = ops.pack_weight(w.to(cuda), precision, upsample=upsample)
    b = ops.pack_weight(view, precision, upsample=upsample)
    torch.cuda.synchronize()
    assert torch.equal(a.hi, b.hi)
    assert (a.lo is None and b.lo is None) or torch.equal(a.lo, b.lo)


def _round_tf32_host(a: np.ndarray) -> np.ndarray:
    """fp32 -> TF32 (10 mantissa bits), nearest with ties away from zero, as fp32 bits."""
    u = a.astype(np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x1000) & 0xFFFFE000).astype(np.uint32).view(np.float32)


def test_tf32_weights_and_operands(cuda):
    """TF32 mode: the packed weights are the fp32 weights rounded to TF32 at the K-major
    [tap][O16][C8] positions, and a conv whose 20 input channels fill no whole 16-value row
    (8-value TF32 rows, zero padded) meets the fp16 bar against float64."""
    from ctmr_b200 import ops

    rng = np.random.default_rng(23)
    w = (rng.standard_normal((24, 20, 3, 3, 3)) / np.sqrt(27 * 20)).astype(np.float32)
    packed = ops.pack_weight(torch.from_numpy(w).to(cuda), "tf32")
    torch.cuda.synchronize()
    assert packed.hi.dtype == torch.float32 and packed.hi.numel() == 27 * 32 * 24
    got = packed.hi.cpu().numpy().reshape(27, 32, 24)
    want = np.zeros((27, 32, 24), dtype=np.float32)
    want[:, :24, :20] = _round_tf32_host(w.reshape(24, 20, 27).transpose(2, 0, 1))
    np.testing.assert_array_equal(got, want)
    x = rng.standard_normal((2, 20, 6, 12, 16)).astype(np.float32)
    b = rng.standard_normal(24).astype(np.float32)
    y = ops.conv3d(ops.to_ndhwc(torch.from_numpy(x).to(cuda)), packed, torch.from_numpy(b).to(cuda))
    torch.cuda.synchronize()
    expected = ops_ref.conv3d_ref(torch.from_numpy(x).double(), torch.from_numpy(w).double(),
                                  torch.from_numpy(b).double())
    err = ops_ref.rel_l2(y.cpu(), expected)
    assert err <= FP16_CONV_REL_L2, f"tf32 rel-L2 {err:.3e}"


def test_decoder_from_a_native_checkpoint(cuda, tmp_path):
    """The production VAE decoder run on weights loaded from a native checkpoint (channels-last
    conv weights, packed from that storage) gives the same volume, bitwise, as on the weights it
    was written from."""
    from ctmr_b200 import fast_b200, networks, pipeline as P, weights as W

    shapes = W.vae_decoder_shapes(P.PRODUCTION_VAE)
    w = W.random_weights(shapes, seed=9, device="cpu")
    W.save_network_file(tmp_path / "vae.safetensors", "vae", w)
    loaded, scale = W.load_network_file(tmp_path / "vae.safetensors", "vae", shapes, device=cuda)
    assert scale is None
    w_dev = {k: t.to(cuda) for k, t in w.items()}
    latent = torch.randn(1, 4, 8, 8, 8, generator=torch.Generator().manual_seed(3)).to(cuda)
    with fast_b200.arithmetic_precision("fp16"):
        a = networks.decode_vae_ncdhw(latent, w_dev, constructor=P.PRODUCTION_VAE)
        b = networks.decode_vae_ncdhw(latent, loaded, constructor=P.PRODUCTION_VAE)
    torch.cuda.synchronize()
    assert all(torch.equal(x, y) for x, y in zip(a, b, strict=True))


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize(("b", "length", "heads"), [(2, 2048, 8), (2, 256, 16), (1, 128, 1), (1, 384, 2)])
def test_attention_d32_matches_sdpa(cuda, b, length, heads, dtype):
    """The tensor-core head-size-32 attention against fp32 SDPA on the same 16-bit Q/K/V (the
    MAISI UNet's level-2 and level-3 token counts and smaller ones): P is rounded to the operand
    type once per key tile, so the bar is 2e-3 rel-L2 for fp16 and 1e-2 for bf16."""
    from ctmr_b200 import ops

    g = torch.Generator().manual_seed(73)
    c = heads * 32
    qkv = (torch.randn(b, length, 3 * c, generator=g) * 1.5).to(cuda, dtype)
    scale = 32 ** -0.5
    out = ops.attention_d32(qkv, heads, scale)
    q, k, v = qkv.float().chunk(3, dim=-1)

    def split(a):
        return a.reshape(b, length, heads, 32).transpose(1, 2)

    ref = torch.nn.functional.scaled_dot_product_attention(split(q), split(k), split(v), scale=scale)
    ref = ref.transpose(1, 2).reshape(b, length, c)
    torch.cuda.synchronize()
    assert out.shape == ref.shape and out.dtype == dtype
    err = ((out.float() - ref).norm() / ref.norm()).item()
    assert err <= (2e-3 if dtype == torch.float16 else 1e-2), f"rel-L2 {err:.3e}"


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("ramp", [(0.25, 4.0), (4.0, 0.25)])
def test_attention_d32_row_maximum_growing_and_shrinking(cuda, ramp, dtype):
    """Keys scaled by a ramp along the sequence: rising, each row's maximum grows by many powers
    of two from key tile to key tile, so the online softmax rescales its running output and sum on
    every tile; falling, the first tile holds the maximum and every later tile's exponentials are
    far below one."""
    from ctmr_b200 import ops

    b, length, heads = 1, 1024, 4
    g = torch.Generator().manual_seed(5)
    c = heads * 32
    qkv = torch.randn(b, length, 3 * c, generator=g) * 1.5
    qkv[:, :, c:2 * c] *= torch.linspace(*ramp, length)[None, :, None]
    qkv = qkv.to(cuda, dtype)
    scale = 32 ** -0.5
    out = ops.attention_d32(qkv, heads, scale)
    q, k, v = qkv.float().chunk(3, dim=-1)

    def split(a):
        return a.reshape(b, length, heads, 32).transpose(1, 2)

    ref = torch.nn.functional.scaled_dot_product_attention(split(q), split(k), split(v), scale=scale)
    ref = ref.transpose(1, 2).reshape(b, length, c)
    torch.cuda.synchronize()
    err = ((out.float() - ref).norm() / ref.norm()).item()
    assert err <= (2e-3 if dtype == torch.float16 else 1e-2), f"rel-L2 {err:.3e}"
