"""CPU oracle for the mlx-generate-ctmr conv3d hot path — TEST INFRASTRUCTURE ONLY.

This package restates the reference's arithmetic in plain torch on the CPU
(float32 and float64) so the CUDA path can be checked against it. Only
``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline /
``--impl reference`` legs may import it; the product (``ctmr_b200``) never
does and has no CPU fallback.

Parity pinning: the restatement reproduces the reference's own recorded golden
vectors (``tests/golden/*.npz``, extracted from the reference's
``tests/fixtures/darwin-arm64``) — see ``tests/test_oracle_goldens.py``.
The reference itself (MLX + Metal) cannot run in this environment, so bitwise
reduction order is not pinned; parity is pinned at the reference's own
tolerances (``maisi_mlx_feasibility.py:10-29``).
"""
