"""Loading of the committed golden fixtures (tests/golden/*.npz) and their regenerated weights."""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import torch

from oracle.networks_ref import seeded_parameters

GOLDEN = Path(__file__).resolve().parent / "golden"


def load(name: str) -> tuple[dict[str, np.ndarray], dict]:
    with np.load(GOLDEN / f"{name}.npz", allow_pickle=False) as z:
        arrays = {k: np.array(z[k]) for k in z.files}
    meta = json.loads(str(arrays.pop("meta")))
    return arrays, meta


def weights(meta: dict, prefix: str = "weight.", dtype=torch.float32) -> dict[str, torch.Tensor]:
    """Regenerate a fixture's parameters and strip ``prefix`` from their names."""
    params = seeded_parameters(meta["recipe"])
    return {k[len(prefix):]: torch.from_numpy(v).to(dtype) for k, v in params.items() if k.startswith(prefix)}


def t(a: np.ndarray, dtype=torch.float32) -> torch.Tensor:
    return torch.from_numpy(np.asarray(a)).to(dtype)
