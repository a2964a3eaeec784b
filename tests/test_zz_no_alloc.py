"""ctmr_conv3d_noalloc: the convolution for callers that cannot allocate device memory.

Plugins that live inside another framework's memory pool, and real-time or
safety-constrained callers whose allocations are all made up front, cannot
call cudaMalloc for the workspace ``ctmr_conv3d`` needs. The no-allocation
entry point takes that scratch from one static device array instead. These
tests call it through the C ABI and check that two calls in a row (the second
reusing the scratch the first left behind) return exactly what the
workspace-taking ``ctmr_conv3d`` returns for the same inputs, and that a
convolution too large for the static scratch is refused without a launch.
This file is collected last so that a failure here cannot hide other results.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from oracle import ops_ref

pytestmark = pytest.mark.gpu

RELATIVE = 2e-6  # the fp32-mode bar of the conv tests (reference tests/test_fast_fp32.py:18)


def _case(seed: int, dev):
    from ctmr_b200 import ops

    rng = np.random.default_rng(seed)
    batch, channels, out_channels, groups = 2, 64, 48, 8
    x = torch.from_numpy((3 * rng.standard_normal((batch, channels, 8, 16, 16)) + 1).astype(np.float32))
    w = torch.from_numpy((rng.standard_normal((out_channels, channels, 3, 3, 3)) / np.sqrt(27 * channels))
                         .astype(np.float32))
    bias = torch.from_numpy(rng.standard_normal((batch, out_channels)).astype(np.float32))
    norm_w = torch.from_numpy((1 + 0.1 * rng.standard_normal(channels)).astype(np.float32))
    norm_b = torch.from_numpy((0.1 * rng.standard_normal(channels)).astype(np.float32))
    res = torch.from_numpy(rng.standard_normal((batch, out_channels, 8, 16, 16)).astype(np.float32))
    xg = ops.to_ndhwc(x.to(dev))
    affine = ops.group_norm_affine(xg, norm_w.to(dev), norm_b.to(dev), groups=groups, eps=1e-6)
    packed = ops.pack_weight(w.to(dev), "fp32")
    host = dict(x=x, w=w, bias=bias, norm_w=norm_w, norm_b=norm_b, res=res, groups=groups)
    return xg, affine, packed, bias.to(dev).contiguous(), ops.to_ndhwc(res.to(dev)), host


def _desc(xg, affine, packed, bias, res, out):
    from ctmr_b200 import _lib, ops

    d = _lib.Conv3dDesc()
    d.batch, d.depth, d.height, d.width = (int(n) for n in (xg.shape[0], *xg.shape[2:]))
    d.x = ops.view(xg)
    d.x2 = ops.view(None)
    d.out_channels, d.kernel_size, d.stride = packed.out_channels, 3, 1
    d.precision = _lib.PRECISION_FP32
    d.weight, d.weight_lo = packed.hi.data_ptr(), packed.lo.data_ptr()
    d.affine, d.silu = affine.data_ptr(), 1
    d.bias, d.bias_per_batch = bias.data_ptr(), 1
    d.residual = ops.view(res)
    d.y, d.y_dtype, d.y_cstride, d.y_coffset = out.data_ptr(), _lib.DTYPE_F32, int(out.shape[1]), 0
    return d


def _with_workspace(desc, dev) -> None:
    from ctmr_b200 import _lib

    nbytes = int(_lib.LIB.ctmr_conv3d_workspace_size(ctypes.byref(desc)))
    assert nbytes > 0, "the case must use scratch memory"
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    _lib.check(_lib.LIB.ctmr_conv3d(ctypes.byref(desc), ws.data_ptr(), nbytes,
                                    torch.cuda.current_stream().cuda_stream), "ctmr_conv3d")
    torch.cuda.synchronize()


def _float64(host) -> torch.Tensor:
    prepared = ops_ref.group_norm_silu_ref(host["x"].double(), host["norm_w"].double(), host["norm_b"].double(),
                                           host["groups"])
    return (ops_ref.conv3d_ref(prepared, host["w"].double()) + host["bias"].double()[:, :, None, None, None]
            + host["res"].double())


def test_noalloc_matches_workspace_entry_point_on_two_calls(cuda):
    from ctmr_b200 import _lib, ops

    stream = torch.cuda.current_stream().cuda_stream
    for seed in (11, 12):  # two calls in a row; the second reuses the scratch the first left behind
        xg, affine, packed, bias, res, host = _case(seed, cuda)
        b, o = int(xg.shape[0]), packed.out_channels
        expected = ops.empty_ndhwc(b, o, *xg.shape[2:], torch.float32, cuda)
        _with_workspace(_desc(xg, affine, packed, bias, res, expected), cuda)
        got = ops.empty_ndhwc(b, o, *xg.shape[2:], torch.float32, cuda)
        got.fill_(float("nan"))
        _lib.check(_lib.LIB.ctmr_conv3d_noalloc(ctypes.byref(_desc(xg, affine, packed, bias, res, got)), stream),
                   "ctmr_conv3d_noalloc")
        torch.cuda.synchronize()
        assert torch.equal(got, expected), f"call with seed {seed} differs from ctmr_conv3d"
        ref = _float64(host)
        err = (got.double().cpu() - ref).abs().max().item()
        assert err <= RELATIVE * ref.abs().max().item(), f"max abs err {err:.3e}"
    assert _lib.device_error(clear=True) == 0


def test_noalloc_refuses_oversized_convolution(cuda):
    from ctmr_b200 import _lib, ops

    limit = 32 << 20
    # fp32 split mode prepares 2 fp16 planes: 2 * 4 bytes per (voxel, channel) -> 2 * 64^3 * 64 * 4 B > 32 MiB.
    x = ops.empty_ndhwc(2, 64, 64, 64, 64, torch.float32, cuda)
    packed = ops.pack_weight(torch.zeros((64, 64, 3, 3, 3), device=cuda), "fp32")
    out = ops.empty_ndhwc(2, 64, 64, 64, 64, torch.float32, cuda)
    d = _lib.Conv3dDesc()
    d.batch, d.depth, d.height, d.width = 2, 64, 64, 64
    d.x, d.x2, d.residual = ops.view(x), ops.view(None), ops.view(None)
    d.out_channels, d.kernel_size, d.stride, d.precision = 64, 3, 1, _lib.PRECISION_FP32
    d.weight, d.weight_lo = packed.hi.data_ptr(), packed.lo.data_ptr()
    d.y, d.y_dtype, d.y_cstride = out.data_ptr(), _lib.DTYPE_F32, 64
    assert int(_lib.LIB.ctmr_conv3d_workspace_size(ctypes.byref(d))) > limit
    status = _lib.LIB.ctmr_conv3d_noalloc(ctypes.byref(d), torch.cuda.current_stream().cuda_stream)
    assert status == _lib.CTMR_ERR_WORKSPACE
    assert b"32 MiB" in _lib.LIB.ctmr_last_error()
    assert _lib.device_error(clear=True) == 0
