"""Multi-GPU partitioning of one MR/MR-Brain volume where the work shards naturally.

One process per GPU (``torchrun``), NCCL over NVLink through ``torch.distributed``.
Ranks form pairs; each pair generates one volume:
  * classifier-free guidance: pair member 0 evaluates the conditional branch
    and member 1 the unconditional one (the two halves of the reference's
    batch-2 UNet pass, ``image.py:163-175``, are independent within a step);
    one ``all_gather`` of the (1, 4, D, H, W) fp32 velocity per step lets both
    members apply ``u + s (c - u)`` and the Euler update identically;
  * sliding-window VAE decode: the members decode alternate windows
    (``decode.py:154-178``; each window has its own group-norm statistics) and
    one ``all_reduce`` of the blend accumulators joins them.
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


class Pairs:
    """Rank pairs (0,1), (2,3), ...; every rank creates every pair group in the same order."""

    def __init__(self, rank: int, world: int) -> None:
        if world % 2:
            raise ValueError("pair partitioning needs an even world size")
        self.rank, self.world = rank, world
        self.member = rank % 2
        groups = [dist.new_group([2 * i, 2 * i + 1]) for i in range(world // 2)]
        self.group = groups[rank // 2]
        self.leader = rank - self.member


def gather_pair(local: torch.Tensor, out: torch.Tensor, group) -> torch.Tensor:
    """``out = [member 0's local, member 1's local]`` (flat), the pair's [cond, uncond] velocity."""
    n = local.numel()
    dist.all_gather([out[:n], out[n:]], local.reshape(-1), group=group)
    return out


def window_partition(n_windows: int, member: int, members: int = 2) -> list[int]:
    """Windows a pair member decodes: round-robin, so every window is decoded exactly once."""
    return [i for i in range(n_windows) if i % members == member]


class CfgSplitStep:
    """One guided step with the two CFG branches on the two members of a pair.

    The branch's UNet pass is captured as a CUDA graph; the all_gather and the
    fused CFG + Euler update run after each replay.
    """

    def __init__(self, weights, constructor, latent_shape, *, class_label: int, spacing: torch.Tensor,
                 guidance_scale: float, device, pairs: Pairs, use_cuda_graph: bool = True) -> None:
        self.weights, self.constructor, self.pairs = weights, constructor, pairs
        self.guidance = float(guidance_scale)
        self.z = torch.zeros(tuple(latent_shape), dtype=torch.float32, device=device).contiguous(
            memory_format=torch.channels_last_3d)
        self.t = torch.zeros((1,), dtype=torch.float32, device=device)
        self.dt = torch.zeros((), dtype=torch.float32, device=device)
        label = int(class_label) if pairs.member == 0 else 0
        self.classes = torch.tensor([label], dtype=torch.int64, device=device)
        self.spacing = spacing.to(device=device, dtype=torch.float32).reshape(1, 3)
        b, c, d, h, w = (int(n) for n in latent_shape)
        self.v_pair = torch.empty((2 * b * c * d * h * w,), dtype=torch.float32, device=device)
        self.v_pair_view = self.v_pair.view(2, d, h, w, c).permute(0, 4, 1, 2, 3)
        self.v_local: torch.Tensor | None = None
        self.use_cuda_graph = use_cuda_graph
        self.graph: torch.cuda.CUDAGraph | None = None
        self.launches_per_step = 0

    def _unet(self) -> None:
        _, v = networks.denoise_unet_ncdhw(self.z, self.t, self.classes, self.spacing, self.weights,
                                           constructor=self.constructor)
        self.v_local = v.to(torch.float32).contiguous(memory_format=torch.channels_last_3d)

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

    def sample(self, z0: torch.Tensor, timesteps: np.ndarray) -> torch.Tensor:
        if self.graph is None and self.use_cuda_graph:
            self.prepare()
        self.z.copy_(z0)
        nxt = np.concatenate([timesteps[1:], np.zeros((1,), dtype=np.float32)])
        for t, n in zip(timesteps.tolist(), nxt.tolist(), strict=True):
            self.t.fill_(float(t))
            self.dt.fill_(euler_dt(t, n))
            if self.graph is not None:
                self.graph.replay()
                ops.LAUNCHES[0] += self.launches_per_step
            else:
                self._unet()
            gather_pair(self.v_local.permute(0, 2, 3, 4, 1), self.v_pair, self.pairs.group)
            ops.rflow_step(self.z, self.v_pair_view, guidance=self.guidance, dt=self.dt, out=self.z)
        return self.z.clone()

    def release(self) -> None:
        self.graph = None


def pair_window_decode(latent, weights, *, constructor, roi, overlap, scale_factor, pairs: Pairs) -> torch.Tensor:
    """Sliding-window decode with the windows split across the pair and the blends all-reduced."""

    def reduce_fn(acc: torch.Tensor, wsum: torch.Tensor) -> None:
        dist.all_reduce(acc, group=pairs.group)
        dist.all_reduce(wsum, group=pairs.group)

    return sliding_window_decode_ncdhw(latent, weights, constructor=constructor, roi=roi, overlap=overlap,
                                       scale_factor=scale_factor, window_filter=lambda i: i % 2 == pairs.member,
                                       reduce_fn=reduce_fn)
