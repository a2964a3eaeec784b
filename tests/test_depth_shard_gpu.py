"""The depth-split UNet pass on one GPU, its shards emulated by threads, against the unsplit pass.

``ctmr_b200.depth_shard`` splits one branch's UNet along the latent's depth over S ranks,
exchanging halo planes and GroupNorm moments with one all_gather per exchange. Here the S
shards run as S host threads on one device, exchanging through an in-process all_gather (each
shard waits for its own work, deposits its buffer, and copies every shard's buffer after a
barrier): the same code path as on S GPUs, without a second GPU. The result must equal the
unsplit UNet's velocity within fp32 rounding (the group statistics merge per shard, and the
convolutions see different tile counts). Also: GroupNorm moments of the parts of a tensor merge
to the whole tensor's affine.
"""

from __future__ import annotations

import threading

import pytest
import torch

from oracle import ops_ref

pytestmark = pytest.mark.gpu


class ThreadHub:
    """In-process all_gather for shards running as threads on one device."""

    def __init__(self, n: int) -> None:
        self.n = n
        self.barrier = threading.Barrier(n, timeout=120)
        self.slots: list[torch.Tensor | None] = [None] * n

    def member(self, k: int) -> "ThreadMember":
        return ThreadMember(self, k)


class ThreadMember:
    def __init__(self, hub: ThreadHub, k: int) -> None:
        self.hub, self.k = hub, k

    def all_gather_into_tensor(self, out: torch.Tensor, inp: torch.Tensor) -> None:
        hub = self.hub
        torch.cuda.current_stream().synchronize()
        hub.slots[self.k] = inp.reshape(-1)
        hub.barrier.wait()
        rows = out.view(hub.n, -1)
        for j in range(hub.n):
            rows[j].copy_(hub.slots[j])
        torch.cuda.current_stream().synchronize()
        hub.barrier.wait()


def _sharded_velocity(cuda, weights, ctor, z, t, cls, spacing, shards: int, precision: str) -> torch.Tensor:
    from ctmr_b200 import depth_shard as DS
    from ctmr_b200 import fast_b200

    hub = ThreadHub(shards)
    outs: list[torch.Tensor | None] = [None] * shards
    errors: list[BaseException] = []
    depth = int(z.shape[2])

    def run(k: int) -> None:
        try:
            torch.cuda.set_device(cuda)
            with fast_b200.arithmetic_precision(precision):
                split = DS.DepthShard(depth, shards, k, hub.member(k))
                unet = DS.ShardedUNet(weights, ctor, split, device=cuda)
                zk = split.take(z)
                v = unet(zk, t, cls, spacing)
                outs[k] = split.inner(v).clone()
                torch.cuda.current_stream().synchronize()
        except BaseException as e:  # noqa: BLE001 - re-raised in the test thread
            errors.append(e)
            hub.barrier.abort()

    threads = [threading.Thread(target=run, args=(k,)) for k in range(shards)]
    for th in threads:
        th.start()
    for th in threads:
        th.join(300)
    if errors:
        raise errors[0]
    return torch.cat(outs, dim=2)


@pytest.mark.parametrize(("latent", "shards", "precision", "budget"), [
    ((1, 4, 32, 32, 16), 2, "fp32", 1e-5),
    ((1, 4, 32, 32, 16), 4, "fp32", 1e-5),
    ((1, 4, 32, 32, 16), 2, "fp16", 1e-3),
    ((1, 4, 64, 64, 32), 2, "fp16", 1e-3),
    ((1, 4, 64, 64, 32), 4, "fp16", 1e-3),
])
def test_depth_split_unet_matches_unsplit(cuda, latent, shards, precision, budget):
    """Production rflow UNet (random init), conditional branch: S depth shards vs one pass."""
    from ctmr_b200 import fast_b200, networks
    from ctmr_b200 import pipeline as P
    from ctmr_b200 import weights as W

    w = W.random_weights(W.unet_shapes(P.PRODUCTION_UNET), seed=0, device=cuda)
    z = torch.randn(latent, generator=torch.Generator().manual_seed(8)).to(cuda).contiguous(
        memory_format=torch.channels_last_3d)
    t, cls = torch.tensor([640.0], device=cuda), torch.tensor([9], device=cuda)
    spacing = P.image_spacing_tensor((0.94, 0.94, 1.36), cuda)
    with fast_b200.arithmetic_precision(precision):
        _, ref = networks.denoise_unet_ncdhw(z, t, cls, spacing, w, constructor=P.PRODUCTION_UNET)
    got = _sharded_velocity(cuda, w, P.PRODUCTION_UNET, z, t, cls, spacing, shards, precision)
    err = ops_ref.rel_l2(got.float().cpu(), ref.double().cpu())
    print(f"[depth split] {latent} S={shards} {precision}: rel-L2 vs unsplit {err:.3e}")
    assert err <= budget, f"depth-split velocity rel-L2 {err:.3e}"


@pytest.mark.parametrize("parts", [2, 4])
def test_group_norm_moments_merge_to_the_whole_tensor(cuda, parts):
    """Moments of depth parts (ctmr_group_norm_moments) merged by ctmr_group_norm_affine_from_moments
    equal the whole tensor's GroupNorm affine, incl. a virtual channel concat."""
    from ctmr_b200 import ops

    gen = torch.Generator().manual_seed(4)
    x = ops.to_ndhwc((torch.randn((1, 64, 16, 12, 10), generator=gen) * 3 + 1).to(cuda))
    x2 = ops.to_ndhwc(torch.randn((1, 32, 16, 12, 10), generator=gen).to(cuda))
    gamma = torch.rand(96, generator=gen).to(cuda) + 0.5
    beta = torch.randn(96, generator=gen).to(cuda)
    whole = ops.group_norm_affine(x, gamma, beta, groups=32, eps=1e-6, x2=x2)
    step = 16 // parts
    moments = torch.stack([ops.group_norm_moments(x[:, :, k * step:(k + 1) * step], groups=32,
                                                  x2=x2[:, :, k * step:(k + 1) * step]) for k in range(parts)])
    merged = ops.group_norm_affine_from_moments(moments, gamma, beta, channels=96, groups=32, eps=1e-6)
    torch.testing.assert_close(merged, whole, rtol=2e-6, atol=2e-6)
    # Every holder of the same moments forms the same affine, bit for bit.
    again = ops.group_norm_affine_from_moments(moments.clone(), gamma, beta, channels=96, groups=32, eps=1e-6)
    assert torch.equal(merged, again)
