"""Depth-sharded rflow UNet: one branch's UNet pass split along the latent's depth over S GPUs.

The reference runs the whole UNet on one device (``unet.py:42-187``); a 3x3x3 convolution
and a GroupNorm both reach across a depth cut, so splitting one pass needs two exchanges,
which this module makes with one NCCL ``all_gather`` over the branch's ranks per exchange:

* **halo planes**: every activation of a split level is held as ``(1, C, P + 2, H, W)``
  (channels-last), ``P`` = this shard's depth planes plus one halo plane below and one above
  holding the neighbouring shards' boundary planes. A convolution runs over the planes it can
  use (``span``): the halos towards neighbouring shards, never one at the volume's face, where
  the kernel's zero padding is the right boundary (it pads the normalised, SiLU'd operand). Its
  output is exact on the inner planes; its halo planes are refreshed before the next use;
* **GroupNorm statistics**: each shard reduces its inner planes to per-(group) moments
  (``ctmr_group_norm_moments``), the moments travel with the halo planes, and every shard
  forms the same affine from all shards' moments in shard order
  (``ctmr_group_norm_affine_from_moments``).

Which levels split: the leading levels without attention (at MAISI's production size, levels
0 and 1 hold ~70 % of a pass's convolution work). The last split level's downsampler and
everything deeper (the attention levels, the middle block) run replicated on every rank of
the branch, on the whole tensor all-gathered at the cut; the up path returns to split levels
by each shard taking its planes (and halos) of the replicated upsampler's output.

Nearest-2x up blocks keep their output on a grid of 2 (P + 2) planes: the folded-weight
conv1 then yields the output's halo planes exactly (they derive from the input's halos), and
conv2 sees the skip on the half grid plane for plane, as the unsplit block does.

Batch 1 only: each rank of a CFG-split volume holds one branch.
"""

from __future__ import annotations

from collections.abc import Mapping

import torch
import torch.distributed as dist

from . import _lib, networks, ops
from . import fast_b200 as A

F32 = torch.float32


class ProcessGroupComm:
    """The shards' one collective, ``all_gather_into_tensor`` in shard order, over a torch.distributed
    process group whose ranks are the shards in order (NCCL on the GPUs, gloo in CPU tests)."""

    def __init__(self, group) -> None:
        self.group = group

    def all_gather_into_tensor(self, out: torch.Tensor, inp: torch.Tensor) -> None:
        dist.all_gather_into_tensor(out, inp, group=self.group)


class DepthShard:
    """Depth split of one tensor level by level: ``shards`` shards exchanging through ``comm`` (a
    ``ProcessGroupComm`` over the shards' ranks in order, or any object with the same
    ``all_gather_into_tensor``), this one holding shard ``shard`` of ``depth`` planes at level 0."""

    def __init__(self, depth: int, shards: int, shard: int, comm) -> None:
        if shards < 2 or depth % shards:
            raise ValueError(f"cannot split {depth} planes into {shards} shards")
        if not 0 <= shard < shards:
            raise ValueError(f"shard {shard} out of range for {shards} shards")
        self.depth, self.shards, self.shard = int(depth), int(shards), int(shard)
        self.local = self.depth // self.shards
        self.comm = comm
        self.first, self.last = self.shard == 0, self.shard == self.shards - 1

    # -- buffers and views
    def buffer(self, c: int, planes: int, h: int, w: int, device) -> torch.Tensor:
        """An uninitialised halo'd activation ``(1, c, planes + 2, h, w)`` stored channels-last."""
        return torch.empty((1, c, planes + 2, h, w), dtype=F32, device=device, memory_format=torch.channels_last_3d)

    def empty(self, c: int, h: int, w: int, device, planes: int | None = None) -> torch.Tensor:
        """A zeroed halo'd activation of ``planes`` (default: this shard's level-0 planes)."""
        t = self.buffer(c, self.local if planes is None else planes, h, w, device)
        return t.zero_()

    @staticmethod
    def inner(t: torch.Tensor) -> torch.Tensor:
        return t[:, :, 1:-1]

    def bounds(self, planes: int) -> tuple[int, int]:
        """Planes ``[lo, hi)`` of a halo'd tensor a same-grid convolution reads: the halos towards
        other shards, not the one at a face of the volume (where zero padding applies)."""
        return (1 if self.first else 0), (planes + 1 if self.last else planes + 2)

    def span(self, t: torch.Tensor | None) -> torch.Tensor | None:
        if t is None:
            return None
        lo, hi = self.bounds(int(t.shape[2]) - 2)
        return t[:, :, lo:hi]

    @staticmethod
    def _plane(t: torch.Tensor, p: int) -> torch.Tensor:
        """Plane ``p`` of a channels-last batch-1 tensor as a flat contiguous (H * W * C) view."""
        return t[0, :, p].permute(1, 2, 0).reshape(-1)

    # -- exchanges
    def exchange(self, tensors: list[torch.Tensor], norm: tuple | None = None) -> torch.Tensor | None:
        """Refresh the halo planes of every halo'd tensor in ``tensors`` from the neighbouring
        shards and, with ``norm = (gamma, beta, groups, eps, sources)``, return the GroupNorm
        affine ``(1, C, 2)`` of the channel concat of ``sources`` (halo'd tensors) over the whole
        depth. One all_gather over the branch's ranks carries both."""
        sizes = [self._plane(t, 1).numel() for t in tensors]
        n_planes = 2 * sum(sizes)
        groups = int(norm[2]) if norm is not None else 0
        width = n_planes + 3 * groups
        device = (tensors[0] if tensors else norm[4][0]).device
        send = torch.empty((width,), dtype=F32, device=device)
        off = 0
        for t, n in zip(tensors, sizes, strict=True):
            planes = int(t.shape[2]) - 2
            send[off:off + n].copy_(self._plane(t, 1))
            send[off + n:off + 2 * n].copy_(self._plane(t, planes))
            off += 2 * n
        if norm is not None:
            srcs = norm[4]
            ops.group_norm_moments(self.inner(srcs[0]), groups=groups,
                                   x2=self.inner(srcs[1]) if len(srcs) > 1 else None,
                                   out=send[n_planes:].view(1, groups, 3))
        flat = torch.empty((self.shards * width,), dtype=F32, device=device)
        self.comm.all_gather_into_tensor(flat, send)
        recv = flat.view(self.shards, width)
        off = 0
        for t, n in zip(tensors, sizes, strict=True):
            planes = int(t.shape[2]) - 2
            if not self.first:  # the lower neighbour's last inner plane
                self._plane(t, 0).copy_(recv[self.shard - 1, off + n:off + 2 * n])
            if not self.last:   # the upper neighbour's first inner plane
                self._plane(t, planes + 1).copy_(recv[self.shard + 1, off:off + n])
            off += 2 * n
        if norm is None:
            return None
        gamma, beta, _, eps, srcs = norm
        channels = sum(int(s.shape[1]) for s in srcs)
        return ops.group_norm_affine_from_moments(recv[:, n_planes:].reshape(self.shards, 1, groups, 3), gamma, beta,
                                                  channels=channels, groups=groups, eps=eps)

    def gather_inner(self, t: torch.Tensor) -> torch.Tensor:
        """The whole tensor (all shards' inner planes in depth order) on every rank of the branch."""
        inner = self.inner(t)
        _, c, p, h, w = (int(n) for n in inner.shape)
        full = torch.empty((1, c, p * self.shards, h, w), dtype=inner.dtype, device=inner.device,
                           memory_format=torch.channels_last_3d)
        self.comm.all_gather_into_tensor(full.permute(0, 2, 3, 4, 1).reshape(-1),
                                         inner.permute(0, 2, 3, 4, 1).reshape(-1))
        return full

    def take(self, full: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """This shard's planes of a whole tensor, with its halo planes (those inside the volume)."""
        _, c, d, h, w = (int(n) for n in full.shape)
        planes = d // self.shards
        if out is None:
            out = self.buffer(c, planes, h, w, full.device)
        s0 = self.shard * planes
        lo, hi = max(s0 - 1, 0), min(s0 + planes + 1, d)
        out[:, :, lo - (s0 - 1):hi - (s0 - 1)].copy_(full[:, :, lo:hi])
        return out

    def scatter_from_full(self, full: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        return self.take(full, out)

    def gather_full(self, t: torch.Tensor) -> torch.Tensor:
        return self.gather_inner(t)


class ShardedUNet:
    """The rflow UNet pass (``unet.py:42-187``, the fused blocks of ``fast_fp32.py:214-291``) on
    one depth shard of a batch-1 latent; ``__call__`` takes the halo'd latent (halos current)
    and returns the halo'd velocity (inner planes exact)."""

    def __init__(self, weights: Mapping[str, torch.Tensor], constructor: Mapping, split: DepthShard, *,
                 device) -> None:
        networks._refuse_unsupported(constructor)
        self.w, self.ctor, self.s = weights, constructor, split
        ch, res, attn, heads, g, eps, fc = networks._levels(constructor)
        self.ch, self.res, self.attn, self.heads, self.g, self.eps, self.fc = ch, res, attn, heads, g, eps, fc
        if not bool(constructor.get("resblock_updown", True)):
            raise ValueError("the B200 path implements the resblock_updown=True MAISI networks")
        # Split levels: the leading attention-free levels whose shard keeps >= 2 planes.
        n = 0
        while n < len(ch) - 1 and not attn[n] and (split.local >> n) >= 2:
            n += 1
        if n == 0:
            raise ValueError("no UNet level can be depth-split at this size")
        self.split_levels = n
        self.device = device

    # -- primitives on halo'd tensors
    def _conv(self, x, weight, bias, *, x2=None, affine=None, silu=False, residual=None, residual_upsampled=False):
        """Same-grid (3x3x3 or 1x1x1) convolution of halo'd ``x`` (++ ``x2``) into a new halo'd tensor."""
        s = self.s
        _, _, pp, h, w = (int(n) for n in x.shape)
        o = int(weight.shape[0])
        out = s.buffer(o, pp - 2, h, w, x.device)
        ops.conv3d(s.span(x), A._pack(weight), bias, x2=s.span(x2), affine=affine, silu=silu,
                   residual=s.span(residual), residual_upsampled=residual_upsampled, out=s.span(out))
        return out

    def _norm(self, tensors, sources, prefix_w: Mapping, name: str):
        return self.s.exchange(tensors, (prefix_w[f"{name}.weight"], prefix_w[f"{name}.bias"], self.g, self.eps,
                                         sources))

    def _resblock(self, x, skip_in, bias1, w: Mapping):
        """ResBlock on a split level; ``x`` (++ ``skip_in``, the up path's virtual concat) halo'd."""
        s = self.s
        srcs = [x] if skip_in is None else [x, skip_in]
        aff1 = self._norm(srcs, srcs, w, "norm1")
        cin = sum(int(t.shape[1]) for t in srcs)
        cout = int(w["conv1.conv.weight"].shape[0])
        hidden = self._conv(x, w["conv1.conv.weight"], bias1, x2=skip_in, affine=aff1, silu=True)
        if cin != cout:
            skip = self._conv(x, w["skip_connection.conv.weight"], w["skip_connection.conv.bias"], x2=skip_in)
        else:
            skip = x
        aff2 = self._norm([hidden], [hidden], w, "norm2")
        return self._conv(hidden, w["conv2.conv.weight"], w["conv2.conv.bias"], affine=aff2, silu=True,
                          residual=skip)

    def _down(self, x, bias1, w: Mapping):
        """Downsampler ResBlock from a split level to the next split level: the 2x2x2 means of the inner
        planes (pooled after GroupNorm + SiLU for conv1, plain for the skip), then convs on the pooled shard.
        The pooling reads no halo, so only the moments travel in the first exchange."""
        s = self.s
        aff1 = self._norm([], [x], w, "norm1")
        xi = s.inner(x)
        _, c, p, h, wd = (int(n) for n in xi.shape)
        pooled = s.buffer(c, p // 2, h // 2, wd // 2, x.device)
        ops.transform(xi, mode=_lib.TRANSFORM_AVGPOOL, affine=aff1, silu=True, out=s.inner(pooled))
        cout = int(w["conv1.conv.weight"].shape[0])
        skip = s.buffer(cout, p // 2, h // 2, wd // 2, x.device)
        if c != cout:
            ops.conv3d(xi, A._pack(w["skip_connection.conv.weight"]), w["skip_connection.conv.bias"], avgpool=True,
                       out=s.inner(skip))
        else:
            ops.transform(xi, mode=_lib.TRANSFORM_AVGPOOL, out=s.inner(skip))
        s.exchange([pooled])
        hidden = self._conv(pooled, w["conv1.conv.weight"], bias1)
        aff2 = self._norm([hidden], [hidden], w, "norm2")
        return self._conv(hidden, w["conv2.conv.weight"], w["conv2.conv.bias"], affine=aff2, silu=True,
                          residual=skip)

    def _up(self, x, bias1, w: Mapping):
        """Nearest-2x upsampler ResBlock between split levels (x halo'd, halos current). Works on a
        grid of 2 (P + 2) planes (input plane i -> output planes 2i, 2i + 1); returns the halo'd view
        of its inner 2P planes plus one halo each side."""
        s = self.s
        aff1 = self._norm([x], [x], w, "norm1")
        _, c, pp, h, wd = (int(n) for n in x.shape)
        lo, hi = s.bounds(pp - 2)
        cout = int(w["conv1.conv.weight"].shape[0])
        hidden = torch.empty((1, cout, 2 * pp, 2 * h, 2 * wd), dtype=F32, device=x.device,
                             memory_format=torch.channels_last_3d)
        ops.conv3d(x[:, :, lo:hi], A._pack(w["conv1.conv.weight"], upsample=True), bias1, affine=aff1, silu=True,
                   out=hidden[:, :, 2 * lo:2 * hi])
        skip = x if c == cout else self._conv(x, w["skip_connection.conv.weight"], w["skip_connection.conv.bias"])
        # The hidden tensor's inner planes are [2, 2P + 2); its halos (planes 1 and 2P + 2) came out exact.
        aff2 = self._norm([], [hidden[:, :, 1:-1]], w, "norm2")
        out = torch.empty_like(hidden, memory_format=torch.channels_last_3d)
        ops.conv3d(hidden[:, :, 2 * lo:2 * hi], A._pack(w["conv2.conv.weight"]), w["conv2.conv.bias"], affine=aff2,
                   silu=True, residual=skip[:, :, lo:hi], residual_upsampled=True, out=out[:, :, 2 * lo:2 * hi])
        return out[:, :, 1:-1]

    # -- the pass
    def __call__(self, z: torch.Tensor, timesteps, class_labels, spacing) -> torch.Tensor:
        s, w, ctor = self.s, self.w, self.ctor
        ch, res, attn, heads, g, eps, fc = self.ch, self.res, self.attn, self.heads, self.g, self.eps, self.fc
        nl, ns = len(ch), self.split_levels
        pw = networks.prefixed_weights
        _, emb = networks.condition_embedding(timesteps, class_labels, spacing, w, ctor)
        table = A.TimeBiasTable(emb, w)

        def bias1(bw):
            return table.bias_for(bw)

        hidden = self._conv(z, networks.required_weight(w, "conv_in.conv.weight"),
                            networks.required_weight(w, "conv_in.conv.bias"))
        skips = [hidden]
        for i in range(nl):
            for r in range(res[i]):
                bw = pw(w, f"down_blocks.{i}.resnets.{r}")
                if i < ns:
                    hidden = self._resblock(hidden, None, bias1(bw), bw)
                else:
                    hidden = networks.residual_block_ncdhw(hidden, table, bw, num_groups=g, eps=eps)
                    if attn[i]:
                        hidden = A.spatial_attention_ncdhw(hidden, pw(w, f"down_blocks.{i}.attentions.{r}"),
                                                           num_groups=g, eps=eps, num_head_channels=heads[i],
                                                           include_fc=fc)
                skips.append(hidden)
            if i != nl - 1:
                bw = pw(w, f"down_blocks.{i}.downsampler")
                if i < ns - 1:
                    hidden = self._down(hidden, bias1(bw), bw)
                else:
                    if i == ns - 1:  # leave the split levels: the whole tensor on every rank
                        hidden = s.gather_inner(hidden)
                    hidden = networks.residual_block_ncdhw(hidden, table, bw, num_groups=g, eps=eps, down=True)
                skips.append(hidden)
        hidden = networks.apply_mid_block(hidden, table, w, ctor)
        res_r, attn_r, heads_r = list(reversed(res)), list(reversed(attn)), list(reversed(heads))
        for i in range(nl):
            level = nl - 1 - i
            k = res_r[i] + 1
            samples, skips = skips[-k:], skips[:-k]
            for r in range(k):
                skip = samples.pop()
                bw = pw(w, f"up_blocks.{i}.resnets.{r}")
                if level < ns:
                    hidden = self._resblock(hidden, skip, bias1(bw), bw)
                else:
                    hidden = networks.residual_block_ncdhw(A.concat_channels_ncdhw(hidden, skip), table, bw,
                                                           num_groups=g, eps=eps)
                    if attn_r[i]:
                        hidden = A.spatial_attention_ncdhw(hidden, pw(w, f"up_blocks.{i}.attentions.{r}"),
                                                           num_groups=g, eps=eps, num_head_channels=heads_r[i],
                                                           include_fc=fc)
            if i != nl - 1:
                bw = pw(w, f"up_blocks.{i}.upsampler")
                if level <= ns - 1:
                    hidden = self._up(hidden, bias1(bw), bw)
                else:
                    hidden = networks.residual_block_ncdhw(hidden, table, bw, num_groups=g, eps=eps, up=True)
                    if level == ns:  # back onto the split levels: this shard's planes
                        hidden = s.take(hidden)
        out_w = (networks.required_weight(w, "out.0.weight"), networks.required_weight(w, "out.0.bias"))
        aff = s.exchange([hidden], (out_w[0], out_w[1], g, eps, [hidden]))
        return self._conv(hidden, networks.required_weight(w, "out.2.conv.weight"),
                          networks.required_weight(w, "out.2.conv.bias"), affine=aff, silu=True)
