"""Test configuration: import paths, the ``gpu`` marker and shared fixtures.

``-m gpu`` tests need a CUDA device (a B200) and call the CUDA library through
its C ABI; everything else runs on the CPU. The product package lives in
``mlx-generate-ctmr_b200/``; the oracle in ``oracle/`` is imported only here,
as the checker.
"""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
for path in (ROOT, ROOT / "mlx-generate-ctmr_b200"):
    if str(path) not in sys.path:
        sys.path.insert(0, str(path))


def pytest_configure(config: pytest.Config) -> None:
    config.addinivalue_line("markers", "gpu: needs a CUDA (sm_100a) device; runs the CUDA library")


@pytest.fixture(scope="session")
def cuda():
    """The CUDA device; GPU tests fail (not skip) without one."""
    import torch

    if not torch.cuda.is_available():
        pytest.fail("this test needs a CUDA device (run with -m 'not gpu' on a CPU host)")
    return torch.device("cuda:0")
