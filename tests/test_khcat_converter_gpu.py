"""The kh-concatenated conv kernel converting its own operand, against the operand-pass route.

With ``CTMR_KHCAT_FUSE=1`` a 16-bit stride-1 3x3x3 conv over fp32 inputs of whole 64-channel
blocks runs ``conv3d_khcat_kernel`` with four converter warps: they read the fp32 NDHWC rows,
apply the GroupNorm affine and SiLU (the reference's ``_PACK`` transform, ``_nax_conv.py:144-197``,
as ``fast_fp32.norm_conv3d_ncdhw`` uses it, ``fast_fp32.py:162-211``) and store the rounded
16-bit operand straight into the kernel's swizzled shared-memory ring. The operand pass
(``prepare_copy_kernel``) is then not launched: the call makes one launch fewer. The transform
is the same expression and the rounding the same round-to-nearest as that pass's, and the
products run in the same order, so the two routes must agree bit for bit; the float64 oracle
checks one of them at the 16-bit bar.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import ops_ref

pytestmark = pytest.mark.gpu

FP16_CONV_REL_L2 = 6e-4
BF16_CONV_REL_L2 = 4e-3

# (shape of x, channels of x2, output channels, depth tiles per weight box)
CASES = [
    ((2, 64, 3, 30, 20), 0, 64, "2"),    # partial h (14 + 14 + 2), w (8 + 8 + 4) and depth-pair tiles
    ((1, 64, 4, 16, 16), 64, 48, "2"),   # virtual concat of two sources, N = 3 x 48
    ((2, 128, 2, 14, 24), 0, 64, "1"),   # two channel blocks, one depth per tile
    ((1, 64, 5, 9, 13), 0, 32, "1"),     # odd extents, 32 outputs (per-voxel stores)
    ((1, 64, 8, 128, 64), 0, 64, "2"),   # 320 tiles: every CTA walks several tiles and ring laps
]


def _launches(fn) -> tuple[torch.Tensor, int]:
    """``fn()``'s result and the number of library kernels it launched (the C ABI's own count of
    the launches of each call, ``ctmr_conv3d_launch_count``, summed by ``ops``)."""
    from ctmr_b200 import ops

    before = ops.LAUNCHES[0]
    y = fn()
    return y, ops.LAUNCHES[0] - before


@pytest.mark.parametrize("precision", ["fp16", "bf16"])
@pytest.mark.parametrize("transform", ["norm", "affine", "plain"])
@pytest.mark.parametrize(("shape", "x2_channels", "out_channels", "depths"), CASES)
def test_converter_warps_match_the_operand_pass(cuda, shape, x2_channels, out_channels, depths, transform,
                                                precision, monkeypatch):
    from ctmr_b200 import ops

    rng = np.random.default_rng(73)
    b, c = shape[:2]
    x = ops.to_ndhwc(torch.from_numpy((rng.standard_normal(shape) * 1.5 + 0.4).astype(np.float32)).to(cuda))
    x2 = None
    if x2_channels:
        x2 = ops.to_ndhwc(torch.from_numpy(rng.standard_normal((b, x2_channels, *shape[2:])).astype(np.float32))
                          .to(cuda))
    cin = c + x2_channels
    w = torch.from_numpy((rng.standard_normal((out_channels, cin, 3, 3, 3)) / np.sqrt(27 * cin)).astype(np.float32))
    bias = torch.from_numpy(rng.standard_normal((b, out_channels)).astype(np.float32)).to(cuda)
    res = ops.to_ndhwc(torch.from_numpy(rng.standard_normal((b, out_channels, *shape[2:])).astype(np.float32))
                       .to(cuda))
    gamma = torch.from_numpy((1 + 0.2 * rng.standard_normal(cin)).astype(np.float32)).to(cuda)
    beta = torch.from_numpy((0.3 * rng.standard_normal(cin)).astype(np.float32)).to(cuda)
    packed = ops.pack_weight(w.to(cuda), precision)
    kw = dict(x2=x2, residual=res)
    if transform == "norm":
        kw.update(norm=(gamma, beta, 32, 1e-6), silu=True)
    elif transform == "affine":
        kw.update(affine=ops.group_norm_affine(x, gamma, beta, groups=32, eps=1e-6, x2=x2), silu=True)
    monkeypatch.delenv("CTMR_DISABLE_KHCAT", raising=False)
    monkeypatch.setenv("CTMR_KHCAT_MT", depths)
    out = {}
    monkeypatch.setenv("CTMR_KHCAT_FUSE", "0")
    out["pass"], n_pass = _launches(lambda: ops.conv3d(x, packed, bias, **kw))
    monkeypatch.setenv("CTMR_KHCAT_FUSE", "1")
    out["fused"], n_fused = _launches(lambda: ops.conv3d(x, packed, bias, **kw))
    assert n_fused == n_pass - 1, f"the operand pass should be the one launch saved ({n_pass} -> {n_fused})"
    torch.cuda.synchronize()
    assert torch.equal(out["fused"], out["pass"]), (
        f"rel-L2 {ops_ref.rel_l2(out['fused'].cpu(), out['pass'].cpu().double()):.3e}")
    if transform == "plain" and x2 is None:
        xin = ops.to_ncdhw(x).double().cpu()
        expected = (ops_ref.conv3d_ref(xin, w.double(), None) + bias.double().cpu()[:, :, None, None, None]
                    + ops.to_ncdhw(res).double().cpu())
        err = ops_ref.rel_l2(ops.to_ncdhw(out["fused"]).cpu(), expected)
        assert err <= (FP16_CONV_REL_L2 if precision == "fp16" else BF16_CONV_REL_L2), f"rel-L2 {err:.3e}"


@pytest.mark.parametrize("shape", [(2, 64, 3, 30, 20), (2, 64, 8, 64, 64), (1, 128, 6, 44, 40)])
def test_converter_warps_with_output_statistics(cuda, shape, monkeypatch):
    """The converter-warp kernel with the epilogue's GroupNorm moments: the same output and the
    same moments as the operand-pass route."""
    from ctmr_b200 import ops

    rng = np.random.default_rng(29)
    b, c = shape[:2]
    x = ops.to_ndhwc(torch.from_numpy(rng.standard_normal(shape).astype(np.float32)).to(cuda))
    w = torch.from_numpy((rng.standard_normal((64, c, 3, 3, 3)) / np.sqrt(27 * c)).astype(np.float32))
    bias = torch.from_numpy(rng.standard_normal(64).astype(np.float32) + 2.0).to(cuda)
    gamma = torch.from_numpy((1 + 0.2 * rng.standard_normal(c)).astype(np.float32)).to(cuda)
    beta = torch.from_numpy((0.3 * rng.standard_normal(c)).astype(np.float32)).to(cuda)
    packed = ops.pack_weight(w.to(cuda), "fp16")
    monkeypatch.delenv("CTMR_DISABLE_KHCAT", raising=False)
    monkeypatch.delenv("CTMR_KHCAT_MT", raising=False)
    results = {}
    for fuse in ("0", "1"):
        monkeypatch.setenv("CTMR_KHCAT_FUSE", fuse)
        y = ops.conv3d(x, packed, bias, norm=(gamma, beta, 32, 1e-6), silu=True, stats=True)
        assert ops.output_stats(y) is not None
        g2 = torch.ones(64, device=cuda)
        results[fuse] = (y, ops.group_norm_affine(y, g2, None, groups=16, eps=1e-6))
    torch.cuda.synchronize()
    assert torch.equal(results["1"][0], results["0"][0])
    torch.testing.assert_close(results["1"][1], results["0"][1], rtol=0, atol=0)
