"""CT-from-mask host logic on the CPU: label validation, bit-plane condition, spacing, HU mapping.

Mirrors the reference's checks in ``from_mask._require_label`` (``from_mask.py:356-376``),
``condition.binarize_labels_ncdhw`` / ``spacing_tensor_ncdhw`` (``condition.py:20-64``) and
``decode.to_hu_ncdhw`` (``decode.py:248-259``) against the oracle.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import networks_ref as N


def _label(shape=(1, 1, 8, 8, 8)) -> np.ndarray:
    rng = np.random.default_rng(0)
    lab = rng.choice(np.array([0, 1, 5, 62, 132, 200], dtype=np.int32), size=shape)
    lab.flat[0] = 200
    return lab


def test_require_label_accepts_valid_mask():
    from ctmr_b200 import pipeline as P

    host = P.require_label(_label())
    assert host.shape == (1, 1, 8, 8, 8)


@pytest.mark.parametrize(("mutate", "message"), [
    (lambda a: a.astype(np.float32), "integer"),
    (lambda a: a[:, :, :6], "multiples of 4"),
    (lambda a: np.where(a == 200, 1, a), "body-envelope label 200"),
    (lambda a: np.where(a == 62, 150, a), "outside 0..132"),
    (lambda a: a[:, 0], "NCDHW"),
    (lambda a: np.concatenate([a, a], axis=1), "1 channel"),
])
def test_require_label_rejects(mutate, message):
    from ctmr_b200 import pipeline as P

    with pytest.raises(ValueError, match=message):
        P.require_label(mutate(_label()))


def test_binarize_matches_oracle():
    from ctmr_b200 import pipeline as P

    lab = torch.from_numpy(_label())
    ours = P.binarize_labels_ncdhw(lab)
    assert ours.shape == (1, 8, 8, 8, 8) and ours.is_contiguous(memory_format=torch.channels_last_3d)
    assert torch.equal(ours, N.binarize_labels(lab))


def test_spacing_and_hu_match_oracle():
    from ctmr_b200 import pipeline as P

    sp = P.spacing_tensor_ncdhw((1.5, 1.5, 2.0), "cpu")
    assert torch.equal(sp, N.spacing_tensor((1.5, 1.5, 2.0)))
    assert sp[0, 0].item() == pytest.approx(150.0)  # no FP16 rounding on the CT path
    with pytest.raises(ValueError):
        P.spacing_tensor_ncdhw((1.0, -1.0, 1.0), "cpu")
    lab = torch.from_numpy(_label())
    dec = torch.randn(lab.shape, generator=torch.Generator().manual_seed(1))
    assert torch.equal(P.to_hu_ncdhw(dec, lab), N.to_hu(dec, lab))


def test_sampler_rejects_guidance_and_bad_scale():
    from ctmr_b200 import pipeline as P

    with pytest.raises(ValueError, match="guidance"):
        P.sample_ct_from_mask_ncdhw(_label(), (1, 1, 1), unet_weights={}, controlnet_weights={}, vae_weights={},
                                    guidance_scale=1.0, seed=0, device="cpu")
    with pytest.raises(ValueError, match="scale_factor"):
        P.sample_ct_from_mask_ncdhw(_label(), (1, 1, 1), unet_weights={}, controlnet_weights={}, vae_weights={},
                                    scale_factor=0.0, seed=0, device="cpu")
