"""Samplers and the ``run()`` entry point on the B200 path.

Mirrors the reference's rectified-flow sampler (``rflow.py``), modality
classifier-free guidance (``image.py:118-175``), sliding-window VAE decode
(``decode.py``) and the image-only ``run(model=..., modality=..., seed=...)``
(``medmlx.py:240-597`` -> ``image_runner.py``), with the guided UNet step
captured once as a CUDA graph and replayed for every timestep.
"""

from __future__ import annotations

import math
import time
from collections.abc import Callable, Sequence
from dataclasses import dataclass, field
from typing import Any

import numpy as np
import torch
import torch.nn.functional as F

from . import fast_b200 as A
from . import networks, ops
from . import weights as W

Z_SCALE = 4
IMAGE_ROI = (80, 80, 80)
IMAGE_OVERLAP = 0.4
CT_ROI = (48, 48, 64)
CT_OVERLAP = 0.6666
SIGMA_SCALE = 0.125
GAUSSIAN_FLOOR = 1e-3

PRODUCTION_UNET = {
    "spatial_dims": 3, "in_channels": 4, "out_channels": 4, "num_channels": [64, 128, 256, 512],
    "attention_levels": [False, False, True, True], "num_head_channels": [0, 0, 32, 32], "num_res_blocks": 2,
    "norm_num_groups": 32, "norm_eps": 1e-6, "use_flash_attention": False, "include_top_region_index_input": False,
    "include_bottom_region_index_input": False, "include_spacing_input": True, "num_class_embeds": 128,
    "resblock_updown": True, "include_fc": True, "with_conditioning": False, "use_combined_linear": False,
}
PRODUCTION_CONTROLNET = {
    "spatial_dims": 3, "in_channels": 4, "num_channels": [64, 128, 256, 512],
    "attention_levels": [False, False, True, True], "num_head_channels": [0, 0, 32, 32], "num_res_blocks": 2,
    "norm_num_groups": 32, "norm_eps": 1e-6, "use_flash_attention": False, "conditioning_embedding_in_channels": 8,
    "conditioning_embedding_num_channels": [8, 32, 64], "num_class_embeds": 128, "resblock_updown": True,
    "include_fc": True, "with_conditioning": False, "use_combined_linear": False,
}
PRODUCTION_VAE = {
    "spatial_dims": 3, "in_channels": 1, "out_channels": 1, "latent_channels": 4, "num_channels": [64, 128, 256],
    "num_res_blocks": [2, 2, 2], "norm_num_groups": 32, "norm_eps": 1e-6, "attention_levels": [False, False, False],
    "with_encoder_nonlocal_attn": False, "with_decoder_nonlocal_attn": False, "include_fc": False,
    "use_combined_linear": False, "use_flash_attention": False, "use_convtranspose": False, "num_splits": 4,
    "dim_split": 1,
}

# Configuration defaults (the reference's ``data/configurations.json``).
CONFIGURATIONS: dict[str, dict[str, Any]] = {
    "ct": {"output_size": (256, 256, 128), "spacing_mm": (1.7, 1.7, 2.0), "modality": 1, "guidance_scale": 0.0,
           "modalities": (1,)},
    "mr": {"output_size": (128, 256, 256), "spacing_mm": (1.25, 1.0, 1.0), "modality": 9, "guidance_scale": 15.0,
           "modalities": (8, 9)},
    "mr-brain": {"output_size": (256, 256, 128), "spacing_mm": (0.94, 0.94, 1.36), "modality": 9,
                 "guidance_scale": 2.0, "modalities": (9, 10, 11, 16, 20, 29, 30, 31, 32, 33)},
}
MODELS = {"mlx-generate-ctmr-mr-brain": "mr-brain", "mlx-generate-ctmr-mr": "mr", "mlx-generate-ctmr-ct": "ct"}


# ---------------------------------------------------------------- rflow schedule (rflow.py)
def timestep_transform_rflow(t: float, input_img_size_numel: int, *, base_img_size_numel: int = 32 ** 3,
                             num_train_timesteps: int = 1000) -> float:
    """``rflow.timestep_transform_rflow`` (``rflow.py:19-45``)."""
    unit = float(t) / float(num_train_timesteps)
    ratio = (float(input_img_size_numel) / float(base_img_size_numel)) ** (1.0 / 3.0)
    return float(num_train_timesteps) * ratio * unit / (1.0 + (ratio - 1.0) * unit)


def set_timesteps_rflow(*, num_inference_steps: int = 30, input_img_size_numel: int,
                        num_train_timesteps: int = 1000) -> tuple[np.ndarray, np.ndarray]:
    """``rflow.set_timesteps_rflow`` (``rflow.py:48-98``): FP16-rounded shifted schedule."""
    if num_inference_steps < 1 or num_inference_steps > num_train_timesteps:
        raise ValueError(f"num_inference_steps {num_inference_steps} must be in 1..{num_train_timesteps}")
    steps = [timestep_transform_rflow((1.0 - i / num_inference_steps) * num_train_timesteps, input_img_size_numel)
             for i in range(num_inference_steps)]
    ts = np.asarray(steps, dtype=np.float16).astype(np.float32)
    return ts, np.concatenate([ts[1:], np.zeros((1,), dtype=np.float32)])


def euler_dt(timestep: float, next_timestep: float, num_train_timesteps: int = 1000) -> float:
    """``rflow.step_rflow``'s ``dt = (t - int(next_t)) / T`` (``rflow.py:101-121``)."""
    return (float(timestep) - int(float(next_timestep))) / float(num_train_timesteps)


def image_spacing_tensor(spacing_mm: Sequence[float], device) -> torch.Tensor:
    """``spacing_mm * 100`` rounded through FP16, ``(1, 3)`` fp32 (``image.py:90-115``)."""
    if len(spacing_mm) != 3:
        raise ValueError("spacing_mm must have three values")
    scaled = np.asarray([spacing_mm], dtype=np.float64) * 100.0
    if not np.isfinite(scaled).all() or np.any(scaled <= 0) or np.any(scaled > np.finfo(np.float16).max):
        raise ValueError("scaled spacing must be positive, finite and representable in FP16")
    return torch.from_numpy(scaled.astype(np.float16).astype(np.float32)).to(device)


def output_intensities(decoded: np.ndarray, *, configuration: str = "ct") -> np.ndarray:
    """int16 image (``image.py:68-87``): CT clip(x*2000-1000, +-1000); MR max(x*1000, 0)."""
    data = np.asarray(decoded, dtype=np.float32)
    if not np.isfinite(data).all():
        raise ValueError("decoded image must be finite")
    if configuration == "ct":
        scaled = np.clip(data * 2000.0 - 1000.0, -1000.0, 1000.0)
    else:
        scaled = np.clip(data * 1000.0, 0.0, None)
    return scaled.astype(np.int16)


def output_intensities_device(decoded: torch.Tensor, *, configuration: str = "ct") -> torch.Tensor:
    """``output_intensities`` on the device, returning int16 on the same device.

    The same float32 operations in the same order (a multiply, then the offset for
    CT, then the clip; no fused multiply-add) and the same float -> int16 cast
    (toward zero through int32, wrapping out-of-range values as numpy's astype
    does), so the result is bitwise the host function's; only the int16 volume
    crosses to the host.
    """
    if not bool(torch.isfinite(decoded).all()):
        raise ValueError("decoded image must be finite")
    data = decoded.to(torch.float32)
    if configuration == "ct":
        scaled = torch.clamp(torch.sub(torch.mul(data, 2000.0), 1000.0), -1000.0, 1000.0)
    else:
        scaled = torch.clamp(torch.mul(data, 1000.0), min=0.0)
    return scaled.to(torch.int32).to(torch.int16)


def init_latent_ncdhw(shape: Sequence[int], *, seed: int, device) -> torch.Tensor:
    """Seeded N(0, 1) fp32 latent. (The reference seeds MLX's generator, whose stream cannot be reproduced here.)"""
    gen = torch.Generator(device=device).manual_seed(int(seed))
    return torch.randn(tuple(int(s) for s in shape), generator=gen, device=device, dtype=torch.float32)


# ---------------------------------------------------------------- guided UNet step (captured)
class GuidedUNetStep:
    """One guided velocity evaluation + Euler update on static buffers, optionally a CUDA graph.

    ``z <- z + dt * (u + s (c - u))`` with ``[c, u] = UNet([z, z], t, [class, 0], spacing)``
    (``image.py:163-175``); without guidance a single conditional pass.
    """

    def __init__(self, weights, constructor, latent_shape, *, class_label: int, spacing: torch.Tensor,
                 guidance_scale: float, device, use_cuda_graph: bool = True, velocity_hook=None) -> None:
        self.weights, self.constructor = weights, constructor
        self.guided = float(guidance_scale) != 0.0
        self.guidance = float(guidance_scale)
        batch = 2 if self.guided else 1
        self.z = torch.zeros(tuple(latent_shape), dtype=torch.float32, device=device).contiguous(
            memory_format=torch.channels_last_3d)
        self.t = torch.zeros((batch,), dtype=torch.float32, device=device)
        self.dt = torch.zeros((), dtype=torch.float32, device=device)
        labels = [int(class_label), 0] if self.guided else [int(class_label)]
        self.classes = torch.tensor(labels, dtype=torch.int64, device=device)
        self.spacing = spacing.to(device=device, dtype=torch.float32).repeat(batch, 1)
        self.velocity_hook = velocity_hook
        self.use_cuda_graph = use_cuda_graph
        self.graph: torch.cuda.CUDAGraph | None = None
        self.launches_per_step = 0

    def _step(self) -> None:
        x = torch.cat([self.z, self.z]) if self.guided else self.z
        _, v = networks.denoise_unet_ncdhw(x, self.t, self.classes, self.spacing, self.weights,
                                           constructor=self.constructor)
        v = v.to(torch.float32).contiguous(memory_format=torch.channels_last_3d)
        if self.velocity_hook is not None:
            v = self.velocity_hook(v)
        ops.rflow_step(self.z, v, guidance=self.guidance if self.guided else None, dt=self.dt, out=self.z)

    def prepare(self) -> None:
        """Pack weights eagerly (one un-timed pass), then capture the step graph."""
        saved = self.z.clone()
        self._step()
        torch.cuda.synchronize()
        if self.use_cuda_graph:
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):
                self._step()
            torch.cuda.current_stream().wait_stream(side)
            self.graph = torch.cuda.CUDAGraph()
            before = ops.LAUNCHES[0]
            with torch.cuda.graph(self.graph):
                self._step()
            self.launches_per_step = ops.LAUNCHES[0] - before
        self.z.copy_(saved)

    def sample(self, z0: torch.Tensor, timesteps: np.ndarray) -> torch.Tensor:
        """Integrate ``z0`` over the schedule (``rflow.sample_rflow``, ``rflow.py:144-177``)."""
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
                self._step()
        return self.z.clone()

    def release(self) -> None:
        self.graph = None


# ---------------------------------------------------------------- sliding-window decode (decode.py)
def scan_interval(size, roi, overlap):
    """``decode.scan_interval`` (``decode.py:30-47``)."""
    out = []
    for s, r in zip(size, roi, strict=True):
        if r == s:
            out.append(r)
            continue
        step = int(r * (1.0 - float(overlap)))
        out.append(step if step > 0 else 1)
    return tuple(out)


def window_starts(size, roi, interval) -> list[list[int]]:
    """Per-axis window starts of ``decode.dense_patch_slices`` (``decode.py:50-85``)."""
    starts = []
    for s, r, step in zip(size, roi, interval, strict=True):
        count = int(math.ceil(float(s) / float(step)))
        last = next((i for i in range(count) if i * step + r >= s), None)
        n = 1 if last is None else last + 1
        starts.append([i * step - max(i * step + r - s, 0) for i in range(n)])
    return starts


def gaussian_1d(length: int, sigma_scale: float = SIGMA_SCALE) -> np.ndarray:
    """One axis of the Gaussian importance map (``decode.py:88-112``), fp32."""
    half = (length - 1) / 2.0
    x = np.arange(-half, half + 1.0, dtype=np.float32)
    sigma = float(sigma_scale) * float(length)
    return np.exp((x * x) / np.float32(-2.0 * sigma * sigma)).astype(np.float32)


@dataclass
class WindowPlan:
    roi: tuple[int, int, int]
    pads: list[tuple[int, int]]
    starts: list[tuple[int, int, int]]
    spatial: tuple[int, int, int]


def plan_windows(latent_spatial, roi, overlap) -> WindowPlan:
    pads = []
    for s, r in zip(latent_spatial, roi, strict=True):
        extra = max(r - int(s), 0)
        pads.append((extra // 2, extra - extra // 2))
    spatial = tuple(int(s) + a + b for s, (a, b) in zip(latent_spatial, pads, strict=True))
    per_axis = window_starts(spatial, roi, scan_interval(spatial, roi, overlap))
    starts = [(a, b, c) for a in per_axis[0] for b in per_axis[1] for c in per_axis[2]]
    return WindowPlan(tuple(roi), pads, starts, spatial)


def sliding_window_decode_ncdhw(latent: torch.Tensor, weights, *, constructor, roi=CT_ROI, overlap=CT_OVERLAP,
                                sigma_scale: float = SIGMA_SCALE, scale_factor: float | None = None,
                                window_filter: Callable[[int], bool] | None = None,
                                reduce_fn: Callable[[torch.Tensor, torch.Tensor], bool | None] | None = None
                                ) -> torch.Tensor | None:
    """``decode.sliding_window_decode_ncdhw`` (``decode.py:187-245``); returns NCDHW fp32 (contiguous).

    ``window_filter(i)`` selects the windows this caller decodes and
    ``reduce_fn(acc, wsum)`` combines the partial blends (the multi-GPU split); when it
    returns False this caller holds no combined blend and gets None. By default every
    window is decoded here.
    """
    if len(roi) != 3 or any(int(r) < 1 for r in roi):
        raise ValueError(f"roi must be three positive ints; got {tuple(roi)}")
    if not 0.0 <= float(overlap) < 1.0:
        raise ValueError(f"overlap must be >= 0 and < 1; got {overlap}")
    x = latent.to(torch.float32)
    if scale_factor is not None:
        value = float(scale_factor)
        if not math.isfinite(value) or value == 0.0:
            raise ValueError("scale_factor must be a finite non-zero caller value")
        x = x / torch.tensor(value, dtype=torch.float32, device=x.device)
    spatial = tuple(int(n) for n in x.shape[2:])

    def decode(win):
        return networks.decode_vae_ncdhw(win, weights, constructor=constructor)[1]

    if math.prod(spatial) <= math.prod(tuple(int(r) for r in roi)):
        return ops.to_ncdhw(decode(x))
    adjusted = tuple(min(int(r), s) for r, s in zip(roi, spatial, strict=True))
    plan = plan_windows(spatial, adjusted, overlap)
    if any(a or b for a, b in plan.pads):
        p = plan.pads
        x = F.pad(x, (p[2][0], p[2][1], p[1][0], p[1][1], p[0][0], p[0][1]))
    dev = x.device
    tables = [torch.from_numpy(gaussian_1d(r, sigma_scale)).to(dev) for r in adjusted]
    out_sp = tuple(n * Z_SCALE for n in plan.spatial)
    acc = wsum = None
    for index, (zd, zh, zw) in enumerate(plan.starts):
        if window_filter is not None and not window_filter(index):
            continue
        win = x[:, :, zd:zd + adjusted[0], zh:zh + adjusted[1], zw:zw + adjusted[2]]
        pred = decode(win)
        if acc is None:
            acc = torch.zeros((int(pred.shape[0]), *out_sp, int(pred.shape[1])), dtype=torch.float32, device=dev)
            wsum = torch.zeros(out_sp, dtype=torch.float32, device=dev)
        ops.window_accumulate(pred, acc, wsum, origin=(zd * Z_SCALE, zh * Z_SCALE, zw * Z_SCALE), tables=tables,
                              scale=Z_SCALE, floor=GAUSSIAN_FLOOR)
    if acc is None:  # this caller decoded no window; contribute zeros to the reduction
        acc = torch.zeros((int(x.shape[0]), *out_sp, int(constructor["out_channels"])), dtype=torch.float32, device=dev)
        wsum = torch.zeros(out_sp, dtype=torch.float32, device=dev)
    if reduce_fn is not None and reduce_fn(acc, wsum) is False:
        return None
    crop = [(a * Z_SCALE, n * Z_SCALE - (a + b) * Z_SCALE) for (a, b), n in zip(plan.pads, plan.spatial, strict=True)]
    return ops.window_finalize(acc, wsum, origin=tuple(c[0] for c in crop), extent=tuple(c[1] for c in crop))


def to_host_array(t: torch.Tensor) -> np.ndarray:
    """Copy a device tensor to a host numpy array through pinned memory.

    The block comes from torch's caching host allocator and the returned array keeps
    it alive, so repeated calls reuse already-mapped pinned pages (no first-touch
    faults on a fresh pageable array, full-speed DMA); the block returns to the cache
    when the array is dropped.
    """
    host = torch.empty(tuple(t.shape), dtype=t.dtype, pin_memory=True)
    host.copy_(t.contiguous(), non_blocking=True)
    torch.cuda.current_stream(t.device).synchronize()
    return host.numpy()


# ---------------------------------------------------------------- image-only sampling (image.py)
@dataclass
class ImageResult:
    latent: torch.Tensor
    decoded: torch.Tensor
    image: np.ndarray | None
    affine: np.ndarray
    stage_timings_s: dict[str, float] = field(default_factory=dict)


def sample_image_ncdhw(output_size: Sequence[int], spacing_mm: Sequence[float], *, unet_weights, vae_weights,
                       unet_constructor=PRODUCTION_UNET, vae_constructor=PRODUCTION_VAE, scale_factor: float = 1.0,
                       configuration: str = "mr-brain", modality: int | None = None,
                       guidance_scale: float | None = None, seed: int | None = 0, latent: torch.Tensor | None = None,
                       num_inference_steps: int = 30, roi=IMAGE_ROI, overlap=IMAGE_OVERLAP, device=None,
                       use_cuda_graph: bool = True, to_host: bool = True, sampler: GuidedUNetStep | None = None
                       ) -> ImageResult:
    """``image.sample_image_ncdhw`` (``image.py:204-346``) on the B200 path.

    ``stage_timings_s`` holds device times (CUDA events, seconds) of the rflow loop and of the
    decode plus intensity readback; the host waits for the device only once, at the end.
    """
    config = CONFIGURATIONS[configuration]
    device = torch.device(device or "cuda")
    divisor = Z_SCALE * 2 ** (len(unet_constructor["num_channels"]) - 1)
    if len(output_size) != 3 or any(int(v) <= 0 or int(v) % divisor for v in output_size):
        raise ValueError(f"output_size must be three positive multiples of {divisor}")
    shape = (1, int(unet_constructor["in_channels"]), *(int(v) // Z_SCALE for v in output_size))
    if latent is None:
        if seed is None or int(seed) < 0:
            raise ValueError("seed must be a non-negative integer when latent is omitted")
        latent = init_latent_ncdhw(shape, seed=int(seed), device=device)
    elif tuple(latent.shape) != shape:
        raise ValueError(f"image-only latent shape {tuple(latent.shape)} != {shape}")
    mod = config["modality"] if modality is None else int(modality)
    guidance = config["guidance_scale"] if guidance_scale is None else float(guidance_scale)
    if not math.isfinite(guidance) or guidance < 0:
        raise ValueError("guidance_scale must be finite and non-negative")
    spacing = image_spacing_tensor(spacing_mm, device)
    timesteps, _ = set_timesteps_rflow(num_inference_steps=num_inference_steps,
                                       input_img_size_numel=math.prod(shape[2:]))
    if sampler is None:
        sampler = GuidedUNetStep(unet_weights, unet_constructor, shape, class_label=mod, spacing=spacing,
                                 guidance_scale=guidance, device=device, use_cuda_graph=use_cuda_graph)
    # Stage times come from CUDA events: no host wait between the stages, so the decode's launches
    # are queued while the rflow steps still run on the device.
    marks = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    marks[0].record()
    final = sampler.sample(latent.to(device=device, dtype=torch.float32).contiguous(
        memory_format=torch.channels_last_3d), timesteps)
    marks[1].record()
    decoded = sliding_window_decode_ncdhw(final, vae_weights, constructor=vae_constructor, roi=roi, overlap=overlap,
                                          scale_factor=scale_factor)
    image = None
    if to_host:
        image = to_host_array(output_intensities_device(decoded, configuration=configuration))
    marks[2].record()
    torch.cuda.synchronize(device)
    return ImageResult(final, decoded, image, np.diag((*map(float, spacing_mm), 1.0)),
                       {"rflow_unet": marks[0].elapsed_time(marks[1]) * 1e-3,
                        "vae_decode": marks[1].elapsed_time(marks[2]) * 1e-3})


def run(*, model: str = "mlx-generate-ctmr-mr-brain", output_dir=None, modality: int | None = None, seed: int = 0,
        output_size: Sequence[int] | None = None, spacing_mm: Sequence[float] | None = None,
        guidance_scale: float | None = None, num_inference_steps: int = 30, precision: str = "fp32",
        unet_weights=None, vae_weights=None, weights_seed: int = 0, scale_factor: float = 1.0,
        roi: Sequence[int] | None = None, overlap: float | None = None, device=None,
        use_cuda_graph: bool = True) -> dict[str, Any]:
    """Image-only generation entry point (``medmlx.run``, ``medmlx.py:240-597``), returning
    ``{"outputs", "artifacts", "details"}``.

    Without ``unet_weights``/``vae_weights`` the production architectures are
    random-initialised from ``weights_seed`` (no checkpoint download exists
    here). ``output_dir``, when given, receives the int16 image as
    ``synthetic_<configuration>.nii.gz`` with its affine and mm units, the
    reference's file (``image_runner.py:218, 332-336``), and ``outputs["image"]``
    is that path.
    """
    if model not in MODELS:
        raise ValueError(f"unknown model {model!r}; supported: {sorted(MODELS)}")
    configuration = MODELS[model]
    if configuration == "ct":
        raise ValueError("mlx-generate-ctmr-ct generates from a label mask: use sample_ct_from_mask_ncdhw")  # noqa
    config = CONFIGURATIONS[configuration]
    mod = config["modality"] if modality is None else int(modality)
    if mod not in config["modalities"]:
        raise ValueError(f"modality {mod!r} is unsupported for {configuration}; supported: {config['modalities']}")
    device = torch.device(device or "cuda")
    out_size = tuple(output_size or config["output_size"])
    spacing = tuple(spacing_mm or config["spacing_mm"])
    if unet_weights is None:
        unet_weights = W.random_weights(W.unet_shapes(PRODUCTION_UNET), seed=weights_seed, device=device)
    if vae_weights is None:
        vae_weights = W.random_weights(W.vae_decoder_shapes(PRODUCTION_VAE), seed=weights_seed + 1, device=device)
    started = time.perf_counter()
    with A.arithmetic_precision(precision):
        result = sample_image_ncdhw(out_size, spacing, unet_weights=unet_weights, vae_weights=vae_weights,
                                    scale_factor=scale_factor, configuration=configuration, modality=mod,
                                    guidance_scale=guidance_scale, seed=seed, num_inference_steps=num_inference_steps,
                                    roi=tuple(roi or IMAGE_ROI), overlap=IMAGE_OVERLAP if overlap is None else overlap,
                                    device=device, use_cuda_graph=use_cuda_graph)
    outputs: dict[str, Any] = {"image": result.image}
    if output_dir is not None:
        from pathlib import Path

        from .nifti import write_nifti

        destination = Path(output_dir) / f"synthetic_{configuration.replace('-', '_')}.nii.gz"
        write_nifti(destination, result.image[0, 0], result.affine, xyz_units="mm")
        outputs = {"image": destination.as_posix()}
    details = {
        "model": model, "configuration": configuration, "modality": mod, "seed": seed, "precision": precision,
        "output_size": list(out_size), "spacing_mm": list(spacing), "num_inference_steps": num_inference_steps,
        "stage_timings_s": dict(result.stage_timings_s, total=time.perf_counter() - started),
        "peak_memory_bytes": int(torch.cuda.max_memory_allocated(device)),
    }
    return {"outputs": outputs, "artifacts": {}, "details": details}


# ---------------------------------------------------------------- CT from a label mask (from_mask.py)
VALID_LABELS = frozenset(range(133)) | {200}


def require_label(label) -> np.ndarray:
    """``from_mask._require_label`` (``from_mask.py:356-376``): integer NCDHW, ids 0..132 + body 200."""
    host = np.asarray(label.cpu() if isinstance(label, torch.Tensor) else label)
    if host.ndim != 5 or int(host.shape[1]) != 1:
        raise ValueError(f"label must be NCDHW with 1 channel; got {host.shape}")
    if not np.issubdtype(host.dtype, np.integer):
        raise ValueError(f"label must be integer; got {host.dtype}")
    unique = {int(v) for v in np.unique(host)}
    unknown = sorted(v for v in unique if v not in VALID_LABELS)
    if unknown:
        raise ValueError("MAISI mask contains labels outside 0..132 plus body label 200: "
                         + ", ".join(str(v) for v in unknown[:10]))
    if 200 not in unique:
        raise ValueError("MAISI mask is missing body-envelope label 200; add it before generation")
    if any(int(s) % Z_SCALE for s in host.shape[2:]):
        raise ValueError(f"label spatial {tuple(host.shape[2:])} must be multiples of {Z_SCALE}")
    return host


def binarize_labels_ncdhw(label: torch.Tensor, bits: int = 8) -> torch.Tensor:
    """Bit k of each label id as channel k, fp32, channels-last (``condition.py:20-43``)."""
    if bits != 8:
        raise ValueError("from-mask dest packs 8 bits")
    ids = label.to(torch.int32)
    planes = ((ids >> torch.arange(bits, device=ids.device, dtype=torch.int32).reshape(1, bits, 1, 1, 1)) & 1)
    return planes.to(torch.float32).contiguous(memory_format=torch.channels_last_3d)


def spacing_tensor_ncdhw(spacing_mm: Sequence[float], device) -> torch.Tensor:
    """``spacing_mm * 100`` as ``(1, 3)`` fp32, no FP16 rounding (``condition.py:46-64``)."""
    values = [float(a) * 100.0 for a in spacing_mm]
    if len(values) != 3 or any(not math.isfinite(v) or v <= 0 for v in values):
        raise ValueError(f"spacing_mm * 100 must be three finite values > 0; got {values}")
    return torch.tensor([values], dtype=torch.float32, device=device)


def synthetic_ct_mask(size: int = 256, seed: int = 0, boxes: int = 48) -> np.ndarray:
    """A synthetic CT label mask in the shape of the CT-from-mask configuration: a body (label 200)
    ellipsoid holding ``boxes`` random axis-aligned boxes whose labels are drawn uniformly from
    0..132; int16 ``(1, 1, size, size, size)``. (The reference's real masks are not available here.)"""
    rng = np.random.default_rng(seed)
    ax = (np.arange(size, dtype=np.float32) + 0.5) / size - 0.5
    d, h, w = np.meshgrid(ax, ax, ax, indexing="ij")
    body = (d / 0.46) ** 2 + (h / 0.40) ** 2 + (w / 0.44) ** 2 <= 1.0
    lab = np.where(body, 200, 0).astype(np.int16)
    for _ in range(boxes):
        lo = rng.integers(0, size - 8, size=3)
        ext = rng.integers(8, max(size // 5, 9), size=3)
        hi = np.minimum(lo + ext, size)
        box = (slice(lo[0], hi[0]), slice(lo[1], hi[1]), slice(lo[2], hi[2]))
        inside = lab[box]
        inside[body[box]] = int(rng.integers(0, 133))
    return lab[None, None]


def to_hu_ncdhw(image: torch.Tensor, label: torch.Tensor) -> torch.Tensor:
    """``clip(x, 0, 1) * 2000 - 1000`` HU with background (label 0) at -1000 (``decode.py:248-259``)."""
    hu = image.clamp(0.0, 1.0) * 2000.0 - 1000.0
    return torch.where(label.to(hu.device) == 0, torch.full_like(hu, -1000.0), hu)


class ControlNetUNetStep:
    """One ControlNet-conditioned UNet velocity + Euler update (``from_mask.py:298-338``), graph-captured.

    The label's conditioning embedding is computed once (``controlnet.py:167-194``)
    and reused by every step, as the reference does.
    """

    def __init__(self, unet_weights, controlnet_weights, unet_constructor, controlnet_constructor, latent_shape, *,
                 conditioning_embedding: torch.Tensor, class_label: int, spacing: torch.Tensor, device,
                 use_cuda_graph: bool = True) -> None:
        self.uw, self.cw = unet_weights, controlnet_weights
        self.uc, self.cc = unet_constructor, controlnet_constructor
        batch = int(latent_shape[0])
        self.z = torch.zeros(tuple(latent_shape), dtype=torch.float32, device=device).contiguous(
            memory_format=torch.channels_last_3d)
        self.t = torch.zeros((batch,), dtype=torch.float32, device=device)
        self.dt = torch.zeros((), dtype=torch.float32, device=device)
        self.classes = torch.full((batch,), int(class_label), dtype=torch.int64, device=device)
        self.spacing = spacing.to(device=device, dtype=torch.float32).expand(batch, 3).contiguous()
        self.embedding = conditioning_embedding
        self.use_cuda_graph = use_cuda_graph
        self.graph: torch.cuda.CUDAGraph | None = None
        self.launches_per_step = 0

    def velocity(self) -> torch.Tensor:
        # The ControlNet pass runs on a side stream beside the UNet's embedding, conv_in and down
        # path, which need its residuals only where the skips collect them (``unet.py:274-356``);
        # the join sits there. CTMR_SKIP_SIDE_STREAM=0 runs it first on the caller's stream.
        if not A.SKIP_SIDE_STREAM:
            down, mid = networks.controlnet_residuals_ncdhw(self.z, self.t, self.classes, None, self.cw,
                                                            constructor=self.cc,
                                                            conditioning_embedding=self.embedding)
            _, v = networks.denoise_unet_ncdhw(self.z, self.t, self.classes, self.spacing, self.uw,
                                               constructor=self.uc, down_block_additional_residuals=down,
                                               mid_block_additional_residual=mid)
            return v
        with A.beside(self.z.device) as side:
            down, mid = networks.controlnet_residuals_ncdhw(self.z, self.t, self.classes, None, self.cw,
                                                            constructor=self.cc,
                                                            conditioning_embedding=self.embedding)
        _, v = networks.denoise_unet_ncdhw(self.z, self.t, self.classes, self.spacing, self.uw, constructor=self.uc,
                                           down_block_additional_residuals=networks.Joined(down, side),
                                           mid_block_additional_residual=mid)
        return v

    def _step(self) -> None:
        v = self.velocity().to(torch.float32).contiguous(memory_format=torch.channels_last_3d)
        ops.rflow_step(self.z, v, guidance=None, dt=self.dt, out=self.z)

    prepare = GuidedUNetStep.prepare
    sample = GuidedUNetStep.sample
    release = GuidedUNetStep.release


@dataclass
class FromMaskResult:
    latent: torch.Tensor
    decoded: torch.Tensor
    hu: torch.Tensor
    stage_timings_s: dict[str, float] = field(default_factory=dict)


def sample_ct_from_mask_ncdhw(label, spacing_mm: Sequence[float], *, unet_weights, controlnet_weights, vae_weights,
                              unet_constructor=PRODUCTION_UNET, controlnet_constructor=PRODUCTION_CONTROLNET,
                              vae_constructor=PRODUCTION_VAE, scale_factor: float = 1.0, seed: int | None = None,
                              latent: torch.Tensor | None = None, num_inference_steps: int = 30,
                              guidance_scale: float = 0.0, roi=CT_ROI, overlap=CT_OVERLAP, device=None,
                              use_cuda_graph: bool = True) -> FromMaskResult:
    """CT volume from a MAISI label map (``from_mask.sample_ct_from_mask_ncdhw``, ``from_mask.py:121-295``)."""
    if float(guidance_scale) != 0.0:
        raise ValueError("the CT path uses ControlNet conditioning, not guidance")
    if not math.isfinite(float(scale_factor)) or float(scale_factor) == 0.0:
        raise ValueError("scale_factor must be a finite non-zero caller value")
    device = torch.device(device or "cuda")
    host = require_label(label)
    label_dev = torch.from_numpy(host).to(device)
    shape = (int(host.shape[0]), 4, *(int(s) // Z_SCALE for s in host.shape[2:]))
    if latent is None:
        if seed is None:
            raise ValueError("seed is required when latent is omitted")
        latent = init_latent_ncdhw(shape, seed=int(seed), device=device)
    elif tuple(latent.shape) != shape:
        raise ValueError(f"latent shape {tuple(latent.shape)} != {shape}")
    started = time.perf_counter()
    # The 8 bit planes of the labels are formed inside the first embedding conv's operand pass.
    embedding = networks.encode_controlnet_condition_ncdhw(ops.LabelBits(label_dev), controlnet_weights,
                                                            constructor=controlnet_constructor)
    timesteps, _ = set_timesteps_rflow(num_inference_steps=num_inference_steps,
                                       input_img_size_numel=math.prod(shape[2:]))
    step = ControlNetUNetStep(unet_weights, controlnet_weights, unet_constructor, controlnet_constructor, shape,
                              conditioning_embedding=embedding, class_label=CONFIGURATIONS["ct"]["modality"],
                              spacing=spacing_tensor_ncdhw(spacing_mm, device), device=device,
                              use_cuda_graph=use_cuda_graph)
    final = step.sample(latent.to(device=device, dtype=torch.float32).contiguous(
        memory_format=torch.channels_last_3d), timesteps)
    step.release()
    torch.cuda.synchronize(device)
    rflow_s = time.perf_counter() - started
    started = time.perf_counter()
    decoded = sliding_window_decode_ncdhw(final, vae_weights, constructor=vae_constructor, roi=roi, overlap=overlap,
                                          scale_factor=scale_factor)
    hu = to_hu_ncdhw(decoded, label_dev)
    torch.cuda.synchronize(device)
    return FromMaskResult(final, decoded, hu, {"rflow_controlnet_unet": rflow_s,
                                               "vae_decode": time.perf_counter() - started})
