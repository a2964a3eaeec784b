"""Extract the reference's recorded golden vectors into small fixtures under tests/golden/.

Run in a checkout that has the reference project (read-only) at REFERENCE_ROOT:
    python tests/golden/make_goldens.py REFERENCE_ROOT
It copies, without modification, the recorded inputs/outputs of the reference's
own test fixtures (``tests/fixtures/darwin-arm64``) that pin this build's hot
path, plus each fixture's weight recipe (seed, skip, shapes), from which the
parameters are regenerated at test time (``oracle.networks_ref.seeded_parameters``,
the algorithm of the reference's ``tests/fixture_parameters.py:15-25``). No
model tensors are stored. The GPU box never needs the reference: the tests read
only these files.
"""

from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np

OUT = Path(__file__).resolve().parent


def _load(path: Path) -> dict[str, np.ndarray]:
    with np.load(path, allow_pickle=False) as z:
        return {k: np.array(z[k]) for k in z.files}


def _write(name: str, arrays: dict[str, np.ndarray], meta: dict) -> None:
    payload = {k: v for k, v in arrays.items()}
    payload["meta"] = np.array(json.dumps(meta, sort_keys=True))
    np.savez_compressed(OUT / f"{name}.npz", **payload)
    print(f"wrote {name}.npz ({sum(v.nbytes for v in arrays.values())} bytes of arrays)")


def main(ref_root: Path) -> None:
    fx = ref_root / "tests" / "fixtures" / "darwin-arm64"
    maisi = fx / "maisi"
    # Block boundaries recorded from MONAI (tests/test_maisi_mlx_residual_attention.py:26-55).
    for name in ("residual", "attention"):
        manifest = json.loads((maisi / f"{name}.json").read_text())
        arrays = _load(maisi / f"{name}.npz")
        _write(f"maisi_{name}", arrays, {"constructor": manifest["constructor"], "recipe": manifest["weight_recipe"],
                                        "source": f"tests/fixtures/darwin-arm64/maisi/{name}.npz"})
    # Networks whose parameters come from the parent fixture's recipe (tests/fixture_parameters.py:62-79).
    for boundary, parent in (("vae", "vae"), ("diffusion", "unet")):
        manifest = json.loads((maisi / f"{boundary}.json").read_text())
        parent_meta = json.loads(str(_load(fx / f"{parent}.npz")["metadata"]))
        _write(f"maisi_{boundary}", _load(maisi / f"{boundary}.npz"),
               {"constructor": manifest["constructor"], "recipe": parent_meta["weight_recipe"],
                "extra": {k: manifest[k] for k in ("spacing_mm", "spacing_scale", "class_index") if k in manifest},
                "source": f"tests/fixtures/darwin-arm64/maisi/{boundary}.npz"})
    manifest = json.loads((maisi / "scheduler.json").read_text())
    _write("maisi_scheduler", _load(maisi / "scheduler.npz"),
           {"constructor": manifest["constructor"], "input_img_size_numel": manifest["input_img_size_numel"],
            "source": "tests/fixtures/darwin-arm64/maisi/scheduler.npz"})
    # Native-case fixtures (tests/fixture_cases.py): vae decode + tiled decode, unet velocity, rflow schedule.
    for name in ("vae", "unet", "rflow"):
        arrays = _load(fx / f"{name}.npz")
        meta = json.loads(str(arrays.pop("metadata")))
        keep = {k: v for k, v in arrays.items()
                if not k.startswith("output.") or k in ("output.decoded", "output.tiled", "output.velocity",
                                                          "output.timesteps", "output.next_timesteps",
                                                          "output.step", "output.origin", "output.sample")}
        _write(name, keep, {"constructor": meta.get("constructor"), "recipe": meta.get("weight_recipe"),
                            "source": f"tests/fixtures/darwin-arm64/{name}.npz"})
    # MR / MR-Brain pipelines (tests/test_mr.py:183-247): CFG velocity batch, 30-step latent, decode, int16 image.
    for name in ("mr-brain", "mr"):
        arrays = _load(fx / f"{name}.npz")
        meta = json.loads(str(arrays.pop("metadata")))
        _write(name.replace("-", "_"), arrays,
               {"constructor": meta["constructor"], "recipe": meta["weight_recipe"], "modality": meta["modality"],
                "guidance_scale": meta["guidance_scale"], "configuration": meta["configuration"],
                "seed": meta["seed"], "source": f"tests/fixtures/darwin-arm64/{name}.npz"})


def catalog(ref_root: Path) -> None:
    """Names and Torch shapes of the production networks' parameters (inventory only, no values)."""
    src = ref_root / "src" / "mlx_generate_ctmr" / "data" / "maisi_mlx_from_mask_weight_catalog.json"
    data = json.loads(src.read_text())
    out = {net: [[t["name"], t["torch_shape"]] for t in spec["tensors"] if t.get("used_at_from_mask_infer", True)]
           for net, spec in data["networks"].items()}
    (OUT / "production_catalog.json").write_text(json.dumps(out, indent=0, sort_keys=True))
    print("wrote production_catalog.json")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: python tests/golden/make_goldens.py <reference project root>")
    root = Path(sys.argv[1])
    main(root)
    catalog(root)
