"""The benchmark's reference arm times the reference's arithmetic (the CPU oracle) and nothing of the
product: building its sample must import no ``ctmr_b200`` module (so no library is loaded), and the
oracle's production parameters have exactly the product's parameter inventory."""

from __future__ import annotations

import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def test_reference_sample_imports_no_product_code():
    code = (
        "import sys; sys.path[:0] = [%r]\n"
        "import bench\n"
        "s = bench.CpuSample()\n"
        "assert s.windows == 4 and s.slabs_per_volume == 12, (s.windows, s.slabs_per_volume)\n"
        "bad = sorted(m for m in sys.modules if m.startswith('ctmr_b200'))\n"
        "assert not bad, bad\n"
        "print('ok')\n" % str(ROOT))
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, cwd=ROOT, timeout=300)
    assert out.returncode == 0 and out.stdout.strip().endswith("ok"), out.stderr[-2000:]


def test_oracle_production_parameters_match_the_product_inventory():
    from ctmr_b200 import pipeline as P
    from ctmr_b200 import weights as W
    from oracle import production as OP

    for net, shapes in (("unet", W.unet_shapes(P.PRODUCTION_UNET)),
                        ("controlnet", W.controlnet_shapes(P.PRODUCTION_CONTROLNET)),
                        ("vae", W.vae_decoder_shapes(P.PRODUCTION_VAE))):
        params = OP.parameters(net, seed=0)
        assert {k: tuple(v.shape) for k, v in params.items()} == shapes, net
    p = OP.parameters("vae", seed=1)
    assert (p["decoder.blocks.1.norm1.weight"] == 1).all() and (p["decoder.blocks.1.norm1.bias"] == 0).all()
    w = p["decoder.blocks.1.conv1.conv.conv.weight"]
    assert w.abs().max().item() <= (1 + 1e-6) / (256 * 27) ** 0.5
