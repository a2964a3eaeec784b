"""NIfTI-1 writer (``ctmr_b200.nifti``) against the format's specification: header fields,
voxel order (first axis fastest), gzip, and the qform quaternion of rotated affines."""

from __future__ import annotations

import math

import numpy as np
import pytest

from ctmr_b200 import nifti


def _rotation(axis, angle):
    axis = np.asarray(axis, dtype=np.float64) / np.linalg.norm(axis)
    k = np.array([[0, -axis[2], axis[1]], [axis[2], 0, -axis[0]], [-axis[1], axis[0], 0]])
    return np.eye(3) + math.sin(angle) * k + (1 - math.cos(angle)) * (k @ k)


def _quat_matrix(b, c, d):
    a = math.sqrt(max(0.0, 1.0 - b * b - c * c - d * d))
    return np.array([[a * a + b * b - c * c - d * d, 2 * (b * c - a * d), 2 * (b * d + a * c)],
                     [2 * (b * c + a * d), a * a + c * c - b * b - d * d, 2 * (c * d - a * b)],
                     [2 * (b * d - a * c), 2 * (c * d + a * b), a * a + d * d - c * c - b * b]])


@pytest.mark.parametrize("name", ["synthetic_mr_brain.nii.gz", "volume.nii"])
def test_round_trip_of_an_int16_volume(tmp_path, name):
    rng = np.random.default_rng(0)
    image = rng.integers(-1000, 3000, size=(7, 5, 3), dtype=np.int16)
    affine = np.diag([0.94, 0.94, 1.36, 1.0])
    path = nifti.write_nifti(tmp_path / name, image, affine)
    fields, data = nifti.read_nifti(path)
    assert data.dtype == np.int16 and data.shape == image.shape and np.array_equal(data, image)
    assert fields["dim"][:4] == (3, 7, 5, 3) and fields["datatype"] == 4 and fields["bitpix"] == 16
    assert fields["vox_offset"] == 352 and fields["xyzt_units"] == 2  # mm
    assert fields["sform_code"] == 2 and fields["qform_code"] == 2
    np.testing.assert_allclose(fields["pixdim"][1:4], [0.94, 0.94, 1.36], rtol=1e-6)
    assert fields["pixdim"][0] == 1.0 and fields["quatern"] == (0.0, 0.0, 0.0)
    np.testing.assert_allclose(fields["affine"], affine, rtol=1e-6)
    raw = path.read_bytes()
    if name.endswith(".gz"):
        import gzip
        raw = gzip.decompress(raw)
    assert len(raw) == 352 + image.size * 2
    # First axis fastest: voxel (1, 0, 0) directly follows voxel (0, 0, 0).
    assert np.frombuffer(raw, "<i2", count=2, offset=352).tolist() == [image[0, 0, 0], image[1, 0, 0]]


@pytest.mark.parametrize(("axis", "angle", "flip"), [((0, 0, 1), 0.3, False), ((1, 2, 3), 2.9, False),
                                                     ((1, 0, 0), math.pi, False), ((0, 1, 1), 1.1, True)])
def test_qform_quaternion_reproduces_the_rotation(axis, angle, flip):
    r = _rotation(axis, angle)
    zooms = np.array([1.5, 0.7, 2.0])
    m = r * zooms
    if flip:
        m[:, 2] = -m[:, 2]
    affine = np.eye(4)
    affine[:3, :3] = m
    affine[:3, 3] = [10.0, -4.0, 3.5]
    b, c, d, qfac, got_zooms = nifti._quaternion(affine)
    rebuilt = _quat_matrix(b, c, d)
    rebuilt[:, 2] *= qfac
    np.testing.assert_allclose(rebuilt * np.array(got_zooms), m, atol=1e-12)
    assert qfac == (-1.0 if flip else 1.0)


def test_rejects_what_the_format_cannot_hold(tmp_path):
    with pytest.raises(ValueError):
        nifti.write_nifti(tmp_path / "x.nii", np.zeros((2, 2), np.int16), np.eye(4))
    with pytest.raises(ValueError):
        nifti.write_nifti(tmp_path / "x.nii", np.zeros((2, 2, 2), np.complex64), np.eye(4))
    with pytest.raises(ValueError):
        nifti.write_nifti(tmp_path / "x.nii", np.zeros((2, 2, 2), np.int16), np.diag([1.0, 0.0, 1.0, 1.0]))
