"""The multi-GPU volume partition against one GPU: a volume group of 2 ranks (CFG branches
split, decode windows split) and, where 4 GPUs are visible, of 4 ranks (each branch's UNet
depth-split over 2 ranks as well, windows over 4).

Runs only where enough CUDA devices are visible; the ranks are child processes
(torchrun-style, NCCL, NVLS off). The group leader's volume and every rank's final latent
must match the single-GPU result within fp32 budgets: the paths differ in how the deep
convolutions split K, in the GroupNorm moments' merge order across shards and in the order
the window blends are summed.
"""

from __future__ import annotations

import os
import socket
import subprocess
import sys
import textwrap
from pathlib import Path

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]

SCRIPT = textwrap.dedent("""
    import os, sys, numpy as np, torch
    sys.path[:0] = [{root!r}, {pkg!r}]
    from ctmr_b200 import distributed as D, pipeline as P, weights as W, fast_b200 as A
    rank, world, local = D.init_from_env()
    dev = torch.device("cuda", local)
    shape = (1, 4, 16, 16, 8)
    ctor = dict(P.PRODUCTION_UNET)
    unet = W.random_weights(W.unet_shapes(ctor), seed=0, device=dev)
    vae = W.random_weights(W.vae_decoder_shapes(P.PRODUCTION_VAE), seed=1, device=dev)
    z0 = torch.randn(shape, generator=torch.Generator().manual_seed(5)).to(dev).contiguous(
        memory_format=torch.channels_last_3d)
    spacing = P.image_spacing_tensor((0.94, 0.94, 1.36), dev)
    ts, _ = P.set_timesteps_rflow(num_inference_steps=3, input_img_size_numel=16 * 16 * 8)
    group = D.VolumeGroup(rank, world, world)
    step = D.GroupGuidedStep(unet, ctor, shape, class_label=9, spacing=spacing, guidance_scale=2.0, device=dev,
                             group=group)
    latent = step.sample(z0, ts)
    dec = D.group_window_decode(latent, vae, constructor=P.PRODUCTION_VAE, roi=(8, 16, 8), overlap=0.25,
                                scale_factor=1.0, group=group)
    step.release()
    if dec is not None:
        np.save(os.path.join({out!r}, f"rank{{rank}}.npy"), dec.cpu().numpy())
    np.save(os.path.join({out!r}, f"latent{{rank}}.npy"), latent.float().cpu().numpy())
    torch.distributed.barrier(device_ids=[local])
    torch.distributed.destroy_process_group()
""")


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("ranks", [2, 4])
def test_volume_group_matches_single_gpu(cuda, tmp_path, ranks):
    if torch.cuda.device_count() < ranks:
        pytest.skip(f"needs {ranks} GPUs")
    from ctmr_b200 import pipeline as P
    from ctmr_b200 import weights as W
    from oracle import ops_ref

    script = tmp_path / "pair.py"
    script.write_text(SCRIPT.format(root=str(ROOT), pkg=str(ROOT / "mlx-generate-ctmr_b200"), out=str(tmp_path)))
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", str(ranks), "--master-addr",
           "127.0.0.1", "--master-port", str(_port()), str(script)]
    subprocess.run(["timeout", "-k", "30", "400", *cmd], check=True, env=env, timeout=460)
    # the same volume on one GPU
    shape = (1, 4, 16, 16, 8)
    unet = W.random_weights(W.unet_shapes(P.PRODUCTION_UNET), seed=0, device=cuda)
    vae = W.random_weights(W.vae_decoder_shapes(P.PRODUCTION_VAE), seed=1, device=cuda)
    z0 = torch.randn(shape, generator=torch.Generator().manual_seed(5)).to(cuda).contiguous(
        memory_format=torch.channels_last_3d)
    ts, _ = P.set_timesteps_rflow(num_inference_steps=3, input_img_size_numel=16 * 16 * 8)
    step = P.GuidedUNetStep(unet, P.PRODUCTION_UNET, shape, class_label=9,
                            spacing=P.image_spacing_tensor((0.94, 0.94, 1.36), cuda), guidance_scale=2.0,
                            device=cuda)
    latent = step.sample(z0, ts)
    dec = P.sliding_window_decode_ncdhw(latent, vae, constructor=P.PRODUCTION_VAE, roi=(8, 16, 8), overlap=0.25,
                                        scale_factor=1.0)
    ref_dec, ref_lat = dec.cpu(), latent.float().cpu()
    for r in range(ranks):
        got_lat = torch.from_numpy(np.load(tmp_path / f"latent{r}.npy"))
        assert ops_ref.rel_l2(got_lat, ref_lat) <= 1e-5
    got_dec = torch.from_numpy(np.load(tmp_path / "rank0.npy"))  # the group leader holds the volume
    assert ops_ref.rel_l2(got_dec, ref_dec) <= 1e-5
    assert not any((tmp_path / f"rank{r}.npy").exists() for r in range(1, ranks))
