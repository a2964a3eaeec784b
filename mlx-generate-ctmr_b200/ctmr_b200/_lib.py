"""ctypes binding of ``libctmr_b200.so`` (the C ABI declared in ``include/ctmr_b200.h``).

The library is loaded from the package's ``lib/`` directory. There is no
fallback: if the shared object is missing or fails to load, importing the ops
raises ``ImportError``, so no caller can silently run on another backend.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libctmr_b200.so"

CTMR_OK = 0
CTMR_ERR_INVALID = 1
CTMR_ERR_UNSUPPORTED = 2
CTMR_ERR_WORKSPACE = 3
CTMR_ERR_CUDA = 4

DTYPE_F32 = 0
DTYPE_BF16 = 1
DTYPE_F16 = 2  # ctmr_transform outputs only
DTYPE_LABEL8 = 3  # conv input only: int16 label ids read as 8 bit-plane channels
PRECISION_FP32 = 0
PRECISION_BF16 = 1
PRECISION_FP16 = 2
PRECISION_TF32 = 3
TRANSFORM_COPY = 0
TRANSFORM_TRILINEAR = 1
TRANSFORM_AVGPOOL = 2
CONV_PREPARE = 1
CONV_GEMM = 2

# Every symbol the header declares; tests check the library exports all of them.
EXPORTED_SYMBOLS = (
    "ctmr_packed_weight_elems",
    "ctmr_packed_weight_bytes",
    "ctmr_pack_weight",
    "ctmr_pack_weight_channels_last",
    "ctmr_attention_d32",
    "ctmr_conv3d_workspace_size",
    "ctmr_conv3d",
    "ctmr_conv3d_stages",
    "ctmr_conv3d_noalloc",
    "ctmr_group_norm_workspace_size",
    "ctmr_group_norm_affine",
    "ctmr_conv3d_stats_slots",
    "ctmr_conv3d_launch_count",
    "ctmr_group_norm_launch_count",
    "ctmr_group_norm_affine_from_stats",
    "ctmr_group_norm_moments",
    "ctmr_group_norm_affine_from_moments",
    "ctmr_transform",
    "ctmr_ncdhw_to_ndhwc",
    "ctmr_ndhwc_to_ncdhw",
    "ctmr_window_accumulate",
    "ctmr_window_finalize",
    "ctmr_rflow_step",
    "ctmr_get_device_error",
    "ctmr_status_string",
    "ctmr_last_error",
)


class Tensor(ctypes.Structure):
    """``ctmr_tensor``: an NDHWC activation view."""

    _fields_ = [
        ("data", ctypes.c_void_p),
        ("dtype", ctypes.c_int),
        ("channels", ctypes.c_int),
        ("cstride", ctypes.c_longlong),
    ]


class Conv3dDesc(ctypes.Structure):
    """``ctmr_conv3d_desc``."""

    _fields_ = [
        ("batch", ctypes.c_int),
        ("depth", ctypes.c_int),
        ("height", ctypes.c_int),
        ("width", ctypes.c_int),
        ("x", Tensor),
        ("x2", Tensor),
        ("out_channels", ctypes.c_int),
        ("kernel_size", ctypes.c_int),
        ("stride", ctypes.c_int),
        ("upsample", ctypes.c_int),
        ("trilinear", ctypes.c_int),
        ("avgpool", ctypes.c_int),
        ("precision", ctypes.c_int),
        ("weight", ctypes.c_void_p),
        ("weight_lo", ctypes.c_void_p),
        ("affine", ctypes.c_void_p),
        ("silu", ctypes.c_int),
        ("bias", ctypes.c_void_p),
        ("bias_per_batch", ctypes.c_int),
        ("residual", Tensor),
        ("residual_upsampled", ctypes.c_int),
        ("y", ctypes.c_void_p),
        ("y_dtype", ctypes.c_int),
        ("y_cstride", ctypes.c_longlong),
        ("y_coffset", ctypes.c_int),
        ("stats", ctypes.c_void_p),
        ("stats_slots", ctypes.c_int),
        ("gn_gamma", ctypes.c_void_p),
        ("gn_beta", ctypes.c_void_p),
        ("gn_groups", ctypes.c_int),
        ("gn_eps", ctypes.c_float),
        ("bias_row_stride", ctypes.c_longlong),
    ]


class TransformDesc(ctypes.Structure):
    """``ctmr_transform_desc``."""

    _fields_ = [
        ("batch", ctypes.c_int),
        ("depth", ctypes.c_int),
        ("height", ctypes.c_int),
        ("width", ctypes.c_int),
        ("x", Tensor),
        ("x2", Tensor),
        ("mode", ctypes.c_int),
        ("affine", ctypes.c_void_p),
        ("silu", ctypes.c_int),
        ("y", ctypes.c_void_p),
        ("y_dtype", ctypes.c_int),
        ("y_channels", ctypes.c_int),
        ("y_cstride", ctypes.c_longlong),
    ]


def _load() -> ctypes.CDLL:
    if not LIB_PATH.exists():
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python mlx-generate-ctmr_b200/build_ext.py` "
            "(ctmr_b200 has no CPU fallback)"
        )
    lib = ctypes.CDLL(str(LIB_PATH))
    vp, i, ll, sz, f = ctypes.c_void_p, ctypes.c_int, ctypes.c_longlong, ctypes.c_size_t, ctypes.c_float
    protos = {
        "ctmr_packed_weight_elems": (sz, [i, i, i, i]),
        "ctmr_packed_weight_bytes": (sz, [i, i, i, i, i]),
        "ctmr_pack_weight": (i, [vp, i, i, i, i, i, vp, vp, vp]),
        "ctmr_pack_weight_channels_last": (i, [vp, i, i, i, i, i, vp, vp, vp]),
        "ctmr_attention_d32": (i, [vp, i, i, i, i, ctypes.c_float, vp, vp]),
        "ctmr_conv3d_workspace_size": (sz, [ctypes.POINTER(Conv3dDesc)]),
        "ctmr_conv3d": (i, [ctypes.POINTER(Conv3dDesc), vp, sz, vp]),
        "ctmr_conv3d_stages": (i, [ctypes.POINTER(Conv3dDesc), vp, sz, i, vp]),
        "ctmr_conv3d_noalloc": (i, [ctypes.POINTER(Conv3dDesc), vp]),
        "ctmr_group_norm_workspace_size": (sz, [i, ll, i]),
        "ctmr_group_norm_affine": (i, [Tensor, Tensor, i, ll, vp, vp, i, f, vp, vp, sz, vp]),
        "ctmr_conv3d_stats_slots": (i, [ctypes.POINTER(Conv3dDesc)]),
        "ctmr_conv3d_launch_count": (i, [ctypes.POINTER(Conv3dDesc)]),
        "ctmr_group_norm_launch_count": (i, [ll, i, i]),
        "ctmr_group_norm_affine_from_stats": (i, [vp, i, vp, i, i, i, vp, vp, i, f, vp, vp]),
        "ctmr_group_norm_moments": (i, [Tensor, Tensor, i, ll, i, vp, vp, sz, vp]),
        "ctmr_group_norm_affine_from_moments": (i, [vp, i, i, i, vp, vp, i, f, vp, vp]),
        "ctmr_transform": (i, [ctypes.POINTER(TransformDesc), vp]),
        "ctmr_ncdhw_to_ndhwc": (i, [vp, i, vp, i, i, i, ll, vp]),
        "ctmr_ndhwc_to_ncdhw": (i, [vp, i, vp, i, i, i, ll, vp]),
        "ctmr_window_accumulate": (i, [Tensor, i, i, i, i, i, i, i, i, i, i, vp, vp, vp, i, f, vp, vp, vp]),
        "ctmr_window_finalize": (i, [vp, vp, vp, i, i, i, i, i, i, i, i, i, i, i, vp]),
        "ctmr_rflow_step": (i, [vp, vp, ll, f, i, f, vp, vp, vp]),
        "ctmr_get_device_error": (i, [ctypes.POINTER(ctypes.c_uint), i]),
        "ctmr_status_string": (ctypes.c_char_p, [i]),
        "ctmr_last_error": (ctypes.c_char_p, []),
    }
    for name, (restype, argtypes) in protos.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    return lib


LIB = _load()


class CtmrError(RuntimeError):
    """A CUDA-side failure reported by the library (status CTMR_ERR_CUDA or a device wait timeout)."""


def check(status: int, what: str) -> None:
    """Map a status code to the reference's exception types (ValueError for bad arguments)."""
    if status == CTMR_OK:
        return
    detail = (LIB.ctmr_last_error() or b"").decode(errors="replace")
    message = f"{what}: {LIB.ctmr_status_string(status).decode()}: {detail}"
    if status in (CTMR_ERR_INVALID, CTMR_ERR_UNSUPPORTED):
        raise ValueError(message)
    if status == CTMR_ERR_WORKSPACE:
        raise ValueError(message)
    raise CtmrError(message)


def device_error(clear: bool = False) -> int:
    """Device error word: non-zero when a bounded device wait gave up. Synchronises."""
    bits = ctypes.c_uint(0)
    check(LIB.ctmr_get_device_error(ctypes.byref(bits), int(clear)), "ctmr_get_device_error")
    return int(bits.value)
