"""Host-side logic of the multi-GPU split on two gloo ranks (CPU): pair groups, the
[cond, uncond] velocity gather the guided Euler update depends on, and the
window split whose all-reduced partial blends must equal the single-process blend."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, results) -> None:
    import sys
    from pathlib import Path

    root = Path(__file__).resolve().parents[1]
    sys.path[:0] = [str(root), str(root / "mlx-generate-ctmr_b200")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from ctmr_b200 import distributed as D
        from ctmr_b200 import pipeline as P
        from oracle import networks_ref as N

        pairs = D.Pairs(rank, world)
        # CFG: member 0 holds the conditional velocity, member 1 the unconditional one.
        n = 4 * 3 * 2 * 2
        local = torch.full((n,), float(rank + 1))
        buf = torch.empty(2 * n)
        D.gather_pair(local, buf, pairs.group)
        cond, uncond = buf[:n], buf[n:]
        z = torch.zeros(n)
        guided = z + (uncond + 2.0 * (cond - uncond)) * 0.5
        # Windows: each member blends its share; the all-reduced blend equals the full blend.
        latent = torch.randn((1, 1, 6, 4, 4), generator=torch.Generator().manual_seed(0))
        roi = (2, 4, 4)
        plan = P.plan_windows(latent.shape[2:], roi, 0.5)
        mine = set(D.window_partition(len(plan.starts), pairs.member))
        predict = lambda w: w.repeat_interleave(4, 2).repeat_interleave(4, 3).repeat_interleave(4, 4) * 2  # noqa: E731
        imp = torch.from_numpy(P.gaussian_1d(roi[0]))[:, None, None] * torch.from_numpy(P.gaussian_1d(roi[1]))[
            None, :, None] * torch.from_numpy(P.gaussian_1d(roi[2]))[None, None, :]
        imp = torch.maximum(imp, torch.tensor(1e-3)).repeat_interleave(4, 0).repeat_interleave(4, 1).repeat_interleave(
            4, 2)
        acc = torch.zeros((1, 1, 24, 16, 16))
        wsum = torch.zeros((24, 16, 16))
        for i, (a, b, c) in enumerate(plan.starts):
            if i not in mine:
                continue
            pred = predict(latent[:, :, a:a + roi[0], b:b + roi[1], c:c + roi[2]])
            sl = (slice(4 * a, 4 * (a + roi[0])), slice(4 * b, 4 * (b + roi[1])), slice(4 * c, 4 * (c + roi[2])))
            acc[(0, 0, *sl)] += pred[0, 0] * imp
            wsum[sl] += imp
        dist.all_reduce(acc, group=pairs.group)
        dist.all_reduce(wsum, group=pairs.group)
        blended = acc / wsum
        full = N.sliding_window(latent, predict, roi, 0.5)
        results[rank] = (pairs.member, pairs.leader, cond[0].item(), uncond[0].item(), guided[0].item(),
                         float((blended - full).abs().max()), sorted(mine), len(plan.starts))
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(120)
def test_pair_split_on_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, results)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(100)
        assert p.exitcode == 0, f"rank exited with {p.exitcode}"
    r0, r1 = results[0], results[1]
    assert (r0[0], r1[0]) == (0, 1) and r0[1] == r1[1] == 0
    for r in (r0, r1):
        assert (r[2], r[3]) == (1.0, 2.0)          # [cond from member 0, uncond from member 1]
        assert r[4] == pytest.approx(0.5 * (2.0 + 2.0 * (1.0 - 2.0)))
        assert r[5] < 1e-5                          # all-reduced partial blends == full blend
    assert sorted(r0[6] + r1[6]) == list(range(r0[7])) and not set(r0[6]) & set(r1[6])


def test_window_partition_covers_every_window_once():
    from ctmr_b200 import distributed as D

    for n in (1, 3, 4, 9):
        parts = [D.window_partition(n, m) for m in range(2)]
        assert sorted(parts[0] + parts[1]) == list(range(n))
