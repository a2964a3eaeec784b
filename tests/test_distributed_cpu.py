"""Host-side logic of the multi-GPU partition on gloo ranks (CPU): volume groups and their
process groups, the [cond, uncond] velocity gather the guided Euler update depends on, the
window split whose reduced partial blends must equal the single-process blend, and the depth
split's halo planes, whole-tensor gather and shard take."""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _blend_check(group, D, P, N) -> float:
    """Each member blends its windows; the reduced blend on the leader equals the full blend."""
    latent = torch.randn((1, 1, 6, 4, 4), generator=torch.Generator().manual_seed(0))
    roi = (2, 4, 4)
    plan = P.plan_windows(latent.shape[2:], roi, 0.5)
    mine = set(group.windows(len(plan.starts)))
    predict = lambda w: w.repeat_interleave(4, 2).repeat_interleave(4, 3).repeat_interleave(4, 4) * 2  # noqa: E731
    imp = torch.from_numpy(P.gaussian_1d(roi[0]))[:, None, None] * torch.from_numpy(P.gaussian_1d(roi[1]))[
        None, :, None] * torch.from_numpy(P.gaussian_1d(roi[2]))[None, None, :]
    imp = torch.maximum(imp, torch.tensor(1e-3)).repeat_interleave(4, 0).repeat_interleave(4, 1).repeat_interleave(4, 2)
    acc = torch.zeros((1, 1, 24, 16, 16))
    wsum = torch.zeros((24, 16, 16))
    for i, (a, b, c) in enumerate(plan.starts):
        if i not in mine:
            continue
        pred = predict(latent[:, :, a:a + roi[0], b:b + roi[1], c:c + roi[2]])
        sl = (slice(4 * a, 4 * (a + roi[0])), slice(4 * b, 4 * (b + roi[1])), slice(4 * c, 4 * (c + roi[2])))
        acc[(0, 0, *sl)] += pred[0, 0] * imp
        wsum[sl] += imp
    dist.reduce(acc, dst=group.leader, group=group.group)
    dist.reduce(wsum, dst=group.leader, group=group.group)
    if group.member != 0:
        return 0.0
    full = N.sliding_window(latent, predict, roi, 0.5)
    return float((acc / wsum - full).abs().max())


def _depth_split_check(group, DS) -> dict:
    """Halo planes after take / exchange, and the whole-tensor gather, on the branch's ranks."""
    if group.shards == 1:
        return {}
    split = DS.DepthShard(16, group.shards, group.shard, DS.ProcessGroupComm(group.branch_group))
    full = torch.randn((1, 3, 16, 4, 5), generator=torch.Generator().manual_seed(7)).contiguous(
        memory_format=torch.channels_last_3d)
    t = split.take(full)
    p, s0 = split.local, group.shard * split.local
    ok_take = torch.equal(split.inner(t), full[:, :, s0:s0 + p])
    # Spoil the halos, then refresh them from the neighbours' inner planes.
    t[:, :, 0].fill_(float("nan"))
    t[:, :, -1].fill_(float("nan"))
    split.exchange([t])
    ok_lo = split.first or torch.equal(t[:, :, 0], full[:, :, s0 - 1])
    ok_hi = split.last or torch.equal(t[:, :, -1], full[:, :, s0 + p])
    lo, hi = split.bounds(p)
    span_ok = (lo, hi) == ((1 if split.first else 0), (p + 1 if split.last else p + 2))
    gathered = split.gather_inner(t)
    return {"take": ok_take, "lo": ok_lo, "hi": ok_hi, "span": span_ok, "gather": torch.equal(gathered, full)}


def _worker(rank: int, world: int, size: int, port: int, results) -> None:
    import sys
    from pathlib import Path

    root = Path(__file__).resolve().parents[1]
    sys.path[:0] = [str(root), str(root / "mlx-generate-ctmr_b200")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from ctmr_b200 import depth_shard as DS
        from ctmr_b200 import distributed as D
        from ctmr_b200 import pipeline as P
        from oracle import networks_ref as N

        group = D.VolumeGroup(rank, world, size)
        # CFG: the two ranks holding one depth shard exchange [cond from branch 0, uncond from branch 1].
        n = 4 * 3 * 2 * 2
        local = torch.full((n,), float(group.branch + 1) + 10.0 * group.shard)
        buf = torch.empty(2 * n)
        D.gather_pair(local, buf, group.peers)
        cond, uncond = buf[:n], buf[n:]
        guided = (uncond + 2.0 * (cond - uncond)) * 0.5
        results[rank] = dict(member=group.member, branch=group.branch, shard=group.shard, leader=group.leader,
                             index=group.index, cond=cond[0].item(), uncond=uncond[0].item(),
                             guided=guided[0].item(), blend=_blend_check(group, D, P, N),
                             windows=group.windows(4), split=_depth_split_check(group, DS))
    finally:
        dist.destroy_process_group()


def _run(world: int, size: int) -> dict:
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, size, port, results)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(280)
        assert p.exitcode == 0, f"rank exited with {p.exitcode}"
    return dict(results)


@pytest.mark.timeout(300)
@pytest.mark.parametrize(("world", "size"), [(2, 2), (4, 4), (4, 2), (8, 8)])
def test_volume_groups_on_gloo_ranks(world, size):
    res = _run(world, size)
    shards = size // 2
    for rank, r in res.items():
        assert r["index"] == rank // size and r["member"] == rank % size and r["leader"] == rank - rank % size
        assert (r["branch"], r["shard"]) == divmod(r["member"], shards)
        # [cond, uncond] of the same depth shard: branch 0 wrote 1 + 10 s, branch 1 wrote 2 + 10 s.
        assert (r["cond"], r["uncond"]) == (1.0 + 10 * r["shard"], 2.0 + 10 * r["shard"])
        assert r["guided"] == pytest.approx(0.5 * (r["uncond"] + 2.0 * (r["cond"] - r["uncond"])))
        if r["member"] == 0:
            assert r["blend"] < 1e-5  # reduced partial blends == the full blend
        if shards > 1:
            assert all(r["split"].values()), r["split"]
    for g in range(world // size):
        members = [r for r in res.values() if r["index"] == g]
        covered = sorted(w for r in members for w in r["windows"])
        assert covered == [0, 1, 2, 3]  # every window decoded exactly once per volume


def test_window_partition_covers_every_window_once():
    from ctmr_b200 import distributed as D

    for members in (2, 4, 8):
        for n in (1, 3, 4, 9):
            parts = [D.window_partition(n, m, members) for m in range(members)]
            assert sorted(sum(parts, [])) == list(range(n))


def test_depth_split_bounds_without_collectives():
    from ctmr_b200 import depth_shard as DS

    for shards in (2, 4):
        for shard in range(shards):
            s = DS.DepthShard(32, shards, shard, comm=None)
            lo, hi = s.bounds(s.local)
            assert lo == (1 if shard == 0 else 0) and hi == (s.local + 1 if shard == shards - 1 else s.local + 2)
    with pytest.raises(ValueError):
        DS.DepthShard(30, 4, 0, comm=None)
    with pytest.raises(ValueError):
        DS.DepthShard(32, 2, 2, comm=None)
