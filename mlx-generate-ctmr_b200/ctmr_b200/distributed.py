"""Multi-GPU partitioning of one MR/MR-Brain volume where the work shards naturally.

One process per GPU (``torchrun``), NCCL over NVLink through ``torch.distributed``.
Ranks form volume groups of G = 2, 4 or 8 consecutive ranks; each group generates
one volume:
  * classifier-free guidance: the group's first half evaluates the conditional
    branch and the second half the unconditional one (the two halves of the
    reference's batch-2 UNet pass, ``image.py:163-175``, are independent within a
    step). The ranks of a branch split the latent's depth between them
    (``ctmr_b200.depth_shard``; G = 2 leaves one rank per branch, unsplit). After each
    UNet pass the two ranks holding the same depth shard of the two branches
    exchange their velocity shards (one ``all_gather`` of two ranks), and both apply
    ``u + s (c - u)`` and the Euler update to that shard identically;
  * sliding-window VAE decode: the G members decode windows round-robin
    (``decode.py:154-178``; each window has its own group-norm statistics) and one
    ``reduce`` of the blend accumulators to the group's first rank joins them.
No TMA multicast and no peer-memory operand is used anywhere: every collective
is a library (NCCL) call on local buffers.
"""

from __future__ import annotations

import datetime
import os

import numpy as np
import torch
import torch.distributed as dist

from . import networks, ops
from .pipeline import euler_dt, sliding_window_decode_ncdhw

GROUP_SIZES = (2, 4, 8)


def init_from_env(timeout_s: int = 120) -> tuple[int, int, int]:
    """Initialise NCCL from torchrun's environment; returns (rank, world, local_rank)."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and not dist.is_initialized():
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=timeout_s),
                                device_id=torch.device("cuda", local))
    return rank, world, local


class VolumeGroup:
    """This rank's place in a partition of ``world`` ranks into volume groups of ``size``.

    ``member`` = position in the group; ``branch`` = 0 (conditional) for the first half,
    1 (unconditional) for the second; ``shard`` = depth shard within the branch
    (``shards`` = size / 2 of them). Process groups (every rank creates every one, in
    the same order): ``group`` (the whole volume group), ``peers`` (the two ranks that
    hold the same shard of the two branches) and ``branch_group`` (the ranks of one
    branch, when it has more than one).
    """

    def __init__(self, rank: int, world: int, size: int) -> None:
        if size not in GROUP_SIZES or world % size:
            raise ValueError(f"volume groups of {size} ranks do not partition {world} ranks")
        self.rank, self.world, self.size = rank, world, size
        self.count = world // size
        self.index, self.member = divmod(rank, size)
        self.shards = size // 2
        self.branch, self.shard = divmod(self.member, self.shards)
        self.leader = rank - self.member
        self.group = self.peers = self.branch_group = None
        self.branch_ranks: list[int] = []
        for g in range(self.count):
            base = g * size
            grp = dist.new_group(list(range(base, base + size)))
            if g == self.index:
                self.group = grp
            for s in range(self.shards):
                pg = dist.new_group([base + s, base + self.shards + s])
                if g == self.index and s == self.shard:
                    self.peers = pg
            if self.shards > 1:
                for b in range(2):
                    ranks = [base + b * self.shards + s for s in range(self.shards)]
                    bg = dist.new_group(ranks)
                    if g == self.index and b == self.branch:
                        self.branch_group, self.branch_ranks = bg, ranks

    def windows(self, n_windows: int) -> list[int]:
        return window_partition(n_windows, self.member, self.size)


def describe_partition(size: int) -> str:
    shards = size // 2
    unet = ("CFG branches on the 2 ranks" if shards == 1 else
            f"CFG branches on 2 x {shards} ranks, each branch's UNet depth-split {shards} ways (halo planes and "
            "GroupNorm moments exchanged by NCCL all_gather)")
    return (f"{size} ranks per volume: {unet}, one velocity all_gather per rflow step between the ranks holding the "
            f"same depth shard; VAE decode windows round-robin over the {size} ranks, one reduce of the blend")


def gather_pair(local: torch.Tensor, out: torch.Tensor, group) -> torch.Tensor:
    """``out = [branch 0's local, branch 1's local]`` (flat): the [cond, uncond] velocity."""
    n = local.numel()
    dist.all_gather([out[:n], out[n:]], local.reshape(-1), group=group)
    return out


def window_partition(n_windows: int, member: int, members: int = 2) -> list[int]:
    """Windows a group member decodes: round-robin, so every window is decoded exactly once."""
    return [i for i in range(n_windows) if i % members == member]


class GroupGuidedStep:
    """One guided step with the two CFG branches on the two halves of a volume group.

    Each rank runs its branch's UNet pass (on its depth shard when the branch has
    several ranks) as a captured CUDA graph; the velocity all_gather with the other
    branch's rank and the fused CFG + Euler update of the shard follow each replay.
    """

    def __init__(self, weights, constructor, latent_shape, *, class_label: int, spacing: torch.Tensor,
                 guidance_scale: float, device, group: VolumeGroup, use_cuda_graph: bool = True) -> None:
        self.weights, self.constructor, self.vg = weights, constructor, group
        self.guidance = float(guidance_scale)
        self.latent_shape = tuple(int(n) for n in latent_shape)
        b, c, d, h, w = self.latent_shape
        if b != 1:
            raise ValueError("the CFG split takes one latent (batch 1)")
        self.t = torch.zeros((1,), dtype=torch.float32, device=device)
        self.dt = torch.zeros((), dtype=torch.float32, device=device)
        label = int(class_label) if group.branch == 0 else 0
        self.classes = torch.tensor([label], dtype=torch.int64, device=device)
        self.spacing = spacing.to(device=device, dtype=torch.float32).reshape(1, 3)
        self.sharded = None
        if group.shards > 1:
            from .depth_shard import DepthShard, ProcessGroupComm, ShardedUNet

            self.split = DepthShard(d, group.shards, group.shard, ProcessGroupComm(group.branch_group))
            self.sharded = ShardedUNet(weights, constructor, self.split, device=device)
            local_d = self.split.local
        else:
            self.split = None
            local_d = d
        # The latent this rank integrates: the whole latent, or its depth shard with halo planes.
        self.z = (self.split.empty(c, h, w, device) if self.split is not None else
                  torch.zeros(self.latent_shape, dtype=torch.float32, device=device).contiguous(
                      memory_format=torch.channels_last_3d))
        self.v_pair = torch.empty((2 * c * local_d * h * w,), dtype=torch.float32, device=device)
        self.v_pair_view = self.v_pair.view(2, local_d, h, w, c).permute(0, 4, 1, 2, 3)
        self.v_local: torch.Tensor | None = None
        self.use_cuda_graph = use_cuda_graph
        self.graph: torch.cuda.CUDAGraph | None = None
        self.launches_per_step = 0

    def _inner(self, t: torch.Tensor) -> torch.Tensor:
        return t if self.split is None else self.split.inner(t)

    def _unet(self) -> None:
        if self.sharded is None:
            _, v = networks.denoise_unet_ncdhw(self.z, self.t, self.classes, self.spacing, self.weights,
                                               constructor=self.constructor)
        else:
            v = self.sharded(self.z, self.t, self.classes, self.spacing)
        self.v_local = self._inner(v).to(torch.float32).contiguous(memory_format=torch.channels_last_3d)

    def prepare(self) -> None:
        saved = self.z.clone()
        self._unet()
        torch.cuda.synchronize()
        if self.use_cuda_graph:
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):
                self._unet()
            torch.cuda.current_stream().wait_stream(side)
            self.graph = torch.cuda.CUDAGraph()
            before = ops.LAUNCHES[0]
            with torch.cuda.graph(self.graph):
                self._unet()
            self.launches_per_step = ops.LAUNCHES[0] - before
        self.z.copy_(saved)

    def _load(self, z0: torch.Tensor) -> None:
        if self.split is None:
            self.z.copy_(z0)
        else:
            self.split.scatter_from_full(z0, self.z)

    def sample(self, z0: torch.Tensor, timesteps: np.ndarray) -> torch.Tensor:
        """Integrate ``z0`` over the schedule; every rank returns the whole final latent."""
        if self.graph is None and self.use_cuda_graph:
            self.prepare()
        self._load(z0)
        nxt = np.concatenate([timesteps[1:], np.zeros((1,), dtype=np.float32)])
        for t, n in zip(timesteps.tolist(), nxt.tolist(), strict=True):
            self.t.fill_(float(t))
            self.dt.fill_(euler_dt(t, n))
            if self.split is not None:
                self.split.exchange([self.z])  # the latent's halo planes for conv_in
            if self.graph is not None:
                self.graph.replay()
                ops.LAUNCHES[0] += self.launches_per_step
            else:
                self._unet()
            gather_pair(self.v_local.permute(0, 2, 3, 4, 1), self.v_pair, self.vg.peers)
            zi = self._inner(self.z)
            ops.rflow_step(zi, self.v_pair_view, guidance=self.guidance, dt=self.dt, out=zi)
        if self.split is None:
            return self.z.clone()
        return self.split.gather_full(self.z)

    def release(self) -> None:
        self.graph = None


def group_window_decode(latent, weights, *, constructor, roi, overlap, scale_factor,
                        group: VolumeGroup) -> torch.Tensor | None:
    """Sliding-window decode with the windows spread over the group; the blends are reduced to
    the group's first rank, which returns the decoded volume (the others return None)."""

    def reduce_fn(acc: torch.Tensor, wsum: torch.Tensor) -> bool:
        dist.reduce(acc, dst=group.leader, group=group.group)
        dist.reduce(wsum, dst=group.leader, group=group.group)
        return group.member == 0

    return sliding_window_decode_ncdhw(latent, weights, constructor=constructor, roi=roi, overlap=overlap,
                                       scale_factor=scale_factor,
                                       window_filter=lambda i: i % group.size == group.member,
                                       reduce_fn=reduce_fn)
