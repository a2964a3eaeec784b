"""NIfTI-1 output of generated volumes, without nibabel.

The reference saves its int16 image as ``synthetic_<configuration>.nii.gz`` through nibabel
(``image_runner.py:332-336``: ``Nifti1Image(image[0, 0], affine)``, units mm, ``nib.save``;
the typed wrapper is ``_nifti.py:80-87``). nibabel is not a dependency here, so this module
writes the single-file NIfTI-1 format directly from its public specification: a 348-byte
little-endian header, a 4-byte extension flag (no extensions), then the voxels with the first
array axis fastest, gzip-compressed when the name ends in ``.gz``. The orientation is stored
twice, as the reference's nibabel header carries it: the affine's rows as the sform (code 2,
"aligned"), and its rotation as the qform quaternion (code 2), computed with Shepperd's
method for a rotation matrix's quaternion (after moving a reflection into ``qfac``).
"""

from __future__ import annotations

import gzip
import struct
from pathlib import Path

import numpy as np

HEADER_BYTES = 348
DATA_OFFSET = 352
_DTYPES = {np.dtype(np.uint8): (2, 8), np.dtype(np.int16): (4, 16), np.dtype(np.int32): (8, 32),
           np.dtype(np.float32): (16, 32), np.dtype(np.float64): (64, 64)}
_UNITS = {"unknown": 0, "meter": 1, "mm": 2, "micron": 3}


def _quaternion(affine: np.ndarray) -> tuple[float, float, float, float, tuple[float, float, float]]:
    """(b, c, d, qfac, zooms) of the qform for a 4x4 affine: the rotation part normalised by its
    column norms, a reflection folded into qfac = -1, and the quaternion (a >= 0) of the rest by
    Shepperd's method (largest of the four squared components first, for stability)."""
    m = np.asarray(affine, dtype=np.float64)[:3, :3]
    zooms = np.sqrt((m * m).sum(axis=0))
    if np.any(zooms == 0):
        raise ValueError("affine has a zero-length axis")
    r = m / zooms
    qfac = 1.0
    if np.linalg.det(r) < 0:
        r[:, 2] = -r[:, 2]
        qfac = -1.0
    t = np.trace(r)
    cand = np.array([1.0 + t, 1.0 + 2 * r[0, 0] - t, 1.0 + 2 * r[1, 1] - t, 1.0 + 2 * r[2, 2] - t])
    k = int(np.argmax(cand))
    s = 0.5 * np.sqrt(max(cand[k], 0.0))
    if k == 0:
        a, b, c, d = s, (r[2, 1] - r[1, 2]) / (4 * s), (r[0, 2] - r[2, 0]) / (4 * s), (r[1, 0] - r[0, 1]) / (4 * s)
    elif k == 1:
        b = s
        a, c, d = (r[2, 1] - r[1, 2]) / (4 * s), (r[0, 1] + r[1, 0]) / (4 * s), (r[0, 2] + r[2, 0]) / (4 * s)
    elif k == 2:
        c = s
        a, b, d = (r[0, 2] - r[2, 0]) / (4 * s), (r[0, 1] + r[1, 0]) / (4 * s), (r[1, 2] + r[2, 1]) / (4 * s)
    else:
        d = s
        a, b, c = (r[1, 0] - r[0, 1]) / (4 * s), (r[0, 2] + r[2, 0]) / (4 * s), (r[1, 2] + r[2, 1]) / (4 * s)
    if a < 0:  # the format stores b, c, d with a = sqrt(1 - b^2 - c^2 - d^2) >= 0
        b, c, d = -b, -c, -d
    return float(b), float(c), float(d), qfac, (float(zooms[0]), float(zooms[1]), float(zooms[2]))


def header_bytes(shape: tuple[int, ...], dtype: np.dtype, affine: np.ndarray, *, xyz_units: str = "mm") -> bytes:
    """The 348-byte NIfTI-1 header of a 3-D volume of ``shape`` and ``dtype`` at ``affine``."""
    if len(shape) != 3:
        raise ValueError(f"a 3-D volume is expected, got shape {tuple(shape)}")
    dtype = np.dtype(dtype)
    if dtype not in _DTYPES:
        raise ValueError(f"unsupported NIfTI data type {dtype}")
    code, bitpix = _DTYPES[dtype]
    aff = np.asarray(affine, dtype=np.float64)
    if aff.shape != (4, 4):
        raise ValueError("affine must be 4x4")
    b, c, d, qfac, zooms = _quaternion(aff)
    h = bytearray(HEADER_BYTES)
    struct.pack_into("<i", h, 0, HEADER_BYTES)
    h[38] = ord("r")  # regular
    struct.pack_into("<8h", h, 40, 3, *(int(n) for n in shape), 1, 1, 1, 1)
    struct.pack_into("<hh", h, 70, code, bitpix)
    struct.pack_into("<8f", h, 76, qfac, *zooms, 1.0, 1.0, 1.0, 1.0)
    struct.pack_into("<f", h, 108, float(DATA_OFFSET))
    struct.pack_into("<ff", h, 112, 1.0, 0.0)  # scl_slope, scl_inter: stored values as is
    h[123] = _UNITS[xyz_units]  # xyzt_units: spatial unit, time unknown
    struct.pack_into("<hh", h, 252, 2, 2)  # qform_code, sform_code: aligned
    struct.pack_into("<6f", h, 256, b, c, d, *(float(v) for v in aff[:3, 3]))
    for row in range(3):
        struct.pack_into("<4f", h, 280 + 16 * row, *(float(v) for v in aff[row]))
    h[344:348] = b"n+1\0"
    return bytes(h)


def write_nifti(path, data: np.ndarray, affine: np.ndarray, *, xyz_units: str = "mm") -> Path:
    """Write ``data`` (first axis = x) with ``affine`` as a single-file NIfTI-1 (``.nii`` or ``.nii.gz``)."""
    path = Path(path)
    data = np.asarray(data)
    payload = header_bytes(data.shape, data.dtype, affine, xyz_units=xyz_units) + b"\0\0\0\0"
    payload += data.astype(data.dtype.newbyteorder("<"), copy=False).tobytes(order="F")
    path.parent.mkdir(parents=True, exist_ok=True)
    if path.name.endswith(".gz"):
        with gzip.open(path, "wb", compresslevel=1) as f:
            f.write(payload)
    else:
        path.write_bytes(payload)
    return path


def read_nifti(path) -> tuple[dict, np.ndarray]:
    """Header fields and voxels of a file ``write_nifti`` wrote (a reader for checks, not a general one)."""
    path = Path(path)
    raw = gzip.decompress(path.read_bytes()) if path.name.endswith(".gz") else path.read_bytes()
    if struct.unpack_from("<i", raw, 0)[0] != HEADER_BYTES or raw[344:348] != b"n+1\0":
        raise ValueError("not a single-file NIfTI-1")
    dim = struct.unpack_from("<8h", raw, 40)
    code, bitpix = struct.unpack_from("<hh", raw, 70)
    pixdim = struct.unpack_from("<8f", raw, 76)
    offset = int(struct.unpack_from("<f", raw, 108)[0])
    qform_code, sform_code = struct.unpack_from("<hh", raw, 252)
    quat = struct.unpack_from("<6f", raw, 256)
    srow = [struct.unpack_from("<4f", raw, 280 + 16 * r) for r in range(3)]
    dtype = next(dt for dt, (c, _) in _DTYPES.items() if c == code).newbyteorder("<")
    shape = tuple(int(n) for n in dim[1:1 + dim[0]])
    data = np.frombuffer(raw, dtype=dtype, count=int(np.prod(shape)), offset=offset).reshape(shape, order="F")
    affine = np.eye(4)
    affine[:3] = np.asarray(srow)
    fields = {"dim": dim, "datatype": code, "bitpix": bitpix, "pixdim": pixdim, "vox_offset": offset,
              "qform_code": qform_code, "sform_code": sform_code, "quatern": quat[:3], "qoffset": quat[3:],
              "xyzt_units": raw[123], "affine": affine}
    return fields, data
