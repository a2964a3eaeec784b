"""The attention kernel's FMA-pipe 2^x (``poly_exp2`` in ``csrc/attention.cu``), restated on the host
in float32 with the kernel's own constants read from the source: Cody-Waite reduction x = n + f with
the 1.5 * 2^23 rounding constant, the degree-3 polynomial for 2^f, n added to the exponent field.
Its relative error must stay well inside the fp16 P operand's half-ulp (4.9e-4) over the whole
range the softmax feeds it (x <= 0), and 2^-125 and below must come out as (near) zero."""

from __future__ import annotations

import re
from pathlib import Path

import numpy as np

SRC = Path(__file__).resolve().parents[1] / "mlx-generate-ctmr_b200" / "csrc" / "attention.cu"


def _constants() -> list[np.float32]:
    text = SRC.read_text()
    return [np.float32(float(re.search(rf"kExp2C{k} = ([0-9.e+-]+)f;", text).group(1))) for k in range(4)]


def _poly_exp2(x: np.ndarray) -> np.ndarray:
    c0, c1, c2, c3 = _constants()
    x = np.maximum(x.astype(np.float32), np.float32(-125.0))
    magic = np.float32(12582912.0)
    j = (x + magic).astype(np.float32)
    f = (x - (j - magic)).astype(np.float32)
    p = np.float32(c3) * f + c2
    p = (p * f + c1).astype(np.float32)
    p = (p * f + c0).astype(np.float32)
    bits = p.view(np.int32) + (j.view(np.int32) << 23)
    return bits.astype(np.int32).view(np.float32)


def test_relative_error_over_the_softmax_range():
    x = np.concatenate([np.linspace(-124.0, 0.0, 2_000_001, dtype=np.float32),
                        -np.random.default_rng(0).exponential(3.0, 200_000).astype(np.float32)])
    x = x[x >= -124.0]
    got = _poly_exp2(x).astype(np.float64)
    want = np.exp2(x.astype(np.float64))
    rel = np.abs(got / want - 1.0)
    assert rel.max() < 1e-4, rel.max()


def test_underflow_and_the_row_maximum():
    assert np.all(_poly_exp2(np.array([-125.0, -200.0, -1e30], dtype=np.float32)) < 1e-37)
    assert abs(float(_poly_exp2(np.array([0.0], dtype=np.float32))[0]) - 1.0) < 1e-4
