"""ControlNet residuals and the CT-from-mask sampler on the B200 against the CPU oracle.

Production ControlNet/UNet/VAE constructors with random weights (the zero
convolutions initialised non-zero so the residuals carry signal) at reduced
latent sizes; fp32 held to the reference's 1e-5 network budget, the 16-bit
operand modes to 1e-2 relative L2.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import networks_ref as N
from oracle import ops_ref

pytestmark = pytest.mark.gpu


def _on(d, dev):
    return {k: v.to(dev) for k, v in d.items()}


def _label(spatial, seed=0) -> np.ndarray:
    """Blocky label map: body 200 inside a margin, organ ids in 4^3 blocks, background outside."""
    rng = np.random.default_rng(seed)
    d, h, w = spatial
    lab = np.zeros((1, 1, d, h, w), dtype=np.int32)
    lab[..., 2:d - 2, 2:h - 2, 2:w - 2] = 200
    blocks = rng.choice(np.array([1, 3, 14, 62, 132], dtype=np.int32), size=(d // 4, h // 4, w // 4))
    organs = np.kron(blocks, np.ones((4, 4, 4), dtype=np.int32))
    inner = np.zeros_like(lab[0, 0], dtype=bool)
    inner[4:d - 4, 4:h - 4, 4:w - 4] = True
    lab[0, 0][inner] = organs[inner]
    return lab


@pytest.mark.parametrize(("precision", "budget"), [("fp32", 1e-5), ("fp16", 1e-2), ("bf16", 1e-2)])
def test_production_controlnet_residuals(cuda, precision, budget):
    """Production ControlNet on a 16^3 latent with the label embedding from a 64^3 mask."""
    from ctmr_b200 import fast_b200, networks
    from ctmr_b200 import pipeline as P
    from ctmr_b200 import weights as W

    ctor = P.PRODUCTION_CONTROLNET
    w = W.random_weights(W.controlnet_shapes(ctor), seed=4, device="cpu")
    lab = torch.from_numpy(_label((64, 64, 64)))
    z = torch.randn((1, 4, 16, 16, 16), generator=torch.Generator().manual_seed(6))
    tt, cls = torch.tensor([700.0]), torch.tensor([1])
    with torch.inference_mode():
        cond = N.binarize_labels(lab)
        ref_down, ref_mid = N.controlnet_residuals(z, tt, cls, cond, w, ctor)
    wd = _on(w, cuda)
    with fast_b200.arithmetic_precision(precision):
        emb = networks.encode_controlnet_condition_ncdhw(P.binarize_labels_ncdhw(lab.to(cuda)), wd, constructor=ctor)
        down, mid = networks.controlnet_residuals_ncdhw(z.to(cuda), tt.to(cuda), cls.to(cuda), None, wd,
                                                        constructor=ctor, conditioning_embedding=emb)
    assert len(down) == len(ref_down)
    for i, (a, b) in enumerate(zip(down, ref_down, strict=True)):
        err = ops_ref.rel_l2(a.float().cpu(), b)
        assert err <= budget, f"{precision} down residual {i} rel-L2 {err:.3e}"
    err = ops_ref.rel_l2(mid.float().cpu(), ref_mid)
    assert err <= budget, f"{precision} mid residual rel-L2 {err:.3e}"


@pytest.mark.parametrize(("precision", "budget"), [("fp32", 1e-5), ("fp16", 1e-2)])
def test_ct_from_mask_sampler(cuda, precision, budget):
    """Two ControlNet-conditioned rflow steps on a 32^3 mask (8^3 latent), default ROI decode, HU mapping."""
    from ctmr_b200 import fast_b200
    from ctmr_b200 import pipeline as P
    from ctmr_b200 import weights as W

    unet = W.random_weights(W.unet_shapes(P.PRODUCTION_UNET), seed=0, device="cpu")
    cn = W.random_weights(W.controlnet_shapes(P.PRODUCTION_CONTROLNET), seed=4, device="cpu")
    vae = W.random_weights(W.vae_decoder_shapes(P.PRODUCTION_VAE), seed=1, device="cpu")
    lab = _label((32, 32, 32), seed=3)
    z0 = torch.randn((1, 4, 8, 8, 8), generator=torch.Generator().manual_seed(9))
    spacing, steps, scale = (1.5, 1.5, 2.0), 2, 1.25
    with torch.inference_mode():
        ref_z, ref_dec, ref_hu = N.sample_ct_from_mask(torch.from_numpy(lab), spacing, unet, P.PRODUCTION_UNET, cn,
                                                       P.PRODUCTION_CONTROLNET, vae, P.PRODUCTION_VAE, z0, steps,
                                                       scale, P.CT_ROI, P.CT_OVERLAP)
    with fast_b200.arithmetic_precision(precision):
        res = P.sample_ct_from_mask_ncdhw(lab, spacing, unet_weights=_on(unet, cuda), controlnet_weights=_on(cn, cuda),
                                          vae_weights=_on(vae, cuda), scale_factor=scale, latent=z0.to(cuda),
                                          num_inference_steps=steps)
    assert ops_ref.rel_l2(res.latent.float().cpu(), ref_z) <= budget
    assert ops_ref.rel_l2(res.decoded.float().cpu(), ref_dec) <= budget
    hu, lab_t = res.hu.float().cpu(), torch.from_numpy(lab)
    assert torch.all(hu[lab_t == 0] == -1000.0)
    assert torch.equal(hu, N.to_hu(res.decoded.float().cpu(), lab_t))
    if precision == "fp32":
        assert float((hu - ref_hu).abs().max()) <= 2000.0 * 1e-4 * max(1.0, float(ref_dec.abs().max()))


@pytest.mark.parametrize("precision", ["fp32", "fp16", "bf16"])
def test_condition_bit_planes_formed_in_the_conv(cuda, precision):
    """The ControlNet condition embedding read straight from the int16 labels (the 8 bit planes
    formed in conv_in's operand pass, ``ops.LabelBits``) equals, bitwise, the embedding of the
    materialised fp32 bit-plane condition; a label input refuses resampling and a second source."""
    from ctmr_b200 import fast_b200, networks, ops
    from ctmr_b200 import pipeline as P
    from ctmr_b200 import weights as W

    ctor = P.PRODUCTION_CONTROLNET
    wd = _on(W.random_weights(W.controlnet_shapes(ctor), seed=5, device="cpu"), cuda)
    lab = torch.from_numpy(_label((64, 64, 32), seed=3)).to(cuda)
    with fast_b200.arithmetic_precision(precision):
        fused = networks.encode_controlnet_condition_ncdhw(ops.LabelBits(lab), wd, constructor=ctor)
        plain = networks.encode_controlnet_condition_ncdhw(P.binarize_labels_ncdhw(lab), wd, constructor=ctor)
        torch.cuda.synchronize()
        assert torch.equal(fused, plain)
        packed = fast_b200._pack(wd["controlnet_cond_embedding.conv_in.conv.weight"])
        with pytest.raises(ValueError):
            ops.conv3d(ops.LabelBits(lab), packed, None, stride=2)
        with pytest.raises(ValueError):
            ops.conv3d(ops.LabelBits(lab), packed, None, trilinear=True)
