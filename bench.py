"""Benchmark: 256x256x128 MR-Brain volumes/min on B200 (the headline metric).

One step = one MR-Brain volume: 30 guided rectified-flow steps of the production
UNet (CFG batch 2, latent 1x4x64x64x32) and the production VAE decode to
256x256x128 as four overlapping depth windows (ROI (24,64,32), overlap 0.25,
Gaussian blend): the MR-Brain generation and the VAE decode stages together. Weights are random-init of
the named architectures (no checkpoints exist offline), inputs synthetic.

  python bench.py [--gpus N --steps K --warmup W] [--precision bf16|fp32] [--impl reference]

N = 1: one GPU per volume. N >= 2 (torchrun, one process per GPU), `--mode
replicas` (default): every rank makes its own volumes (seed = rank), no
collective on the data path; `--mode split`: ranks pair up and each pair makes
one volume per step with the CFG branches split across the pair (one velocity
all_gather per step) and the decode windows split (one all_reduce of the blend).
Per-GPU work is fixed either way, so scaling is "weak". In replicas mode with an
even N the split mode is timed too and reported beside the headline ("split").
``--impl reference`` times the reference's arithmetic on the host CPU (the
torch-CPU restatement in ``oracle/``; the reference itself needs MLX/Metal).
"""

from __future__ import annotations

import argparse
import contextlib
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for _p in (ROOT, ROOT / "mlx-generate-ctmr_b200"):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = "256x256x128 MR-Brain volumes/min (30 rflow steps CFG batch 2 + VAE decode)"
UNIT = "volumes/min"
LATENT = (1, 4, 64, 64, 32)
OUTPUT = (256, 256, 128)
SPACING = (0.94, 0.94, 1.36)
MODALITY = 9
GUIDANCE = 2.0
STEPS_RFLOW = 30
DECODE_ROI = (24, 64, 32)
DECODE_OVERLAP = 0.25
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def _args():
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=2)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=("ours", "reference"), default="ours")
    p.add_argument("--precision", choices=("fp16", "bf16", "tf32", "fp32"), default="fp16")
    p.add_argument("--mode", choices=("replicas", "partition"), default="replicas",
                   help="N > 1: independent volumes per GPU (the partition is timed beside them), or all N GPUs "
                        "on one volume as the headline")
    p.add_argument("--no-fp32-line", action="store_true",
                   help="N = 1: skip the fp32- and tf32-mode volume rates printed beside the headline")
    p.add_argument("--no-graph", action="store_true")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--case", choices=("volume", "sweep", "conv", "gn", "unet-step", "vae-window", "breakdown",
                                      "attention", "ct"),
                   default="volume",
                   help="volume: the benchmark; sweep: the reference's conv-kernel sweep (TFLOP/s per shape); "
                        "conv / unet-step / vae-window: one kernel shape, one UNet step or one decode window "
                        "(bounded workloads for profiler captures); breakdown: per-stage device times of one "
                        "UNet step and one decode window")
    p.add_argument("--shape", default="2,64,64,64,32,64", help="conv case: B,C,D,H,W,O")
    p.add_argument("--iters", type=int, default=3)
    p.add_argument("--input", choices=("plain", "norm", "tri"), default="plain",
                   help="conv case: input as is, group-norm affine + SiLU, or trilinear 2x of a half grid")
    return p.parse_args()


def _peaks() -> tuple[dict, str]:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        return json.loads(path.read_text()), "measured"
    return FALLBACK_PEAKS, "fallback"


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int) -> None:
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(gpu_index)], stdout=self.file, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.file.flush()
        rows = [r.split(",") for r in Path(self.file.name).read_text().strip().splitlines() if r.strip()]
        os.unlink(self.file.name)
        sm = [float(r[1]) for r in rows if len(r) >= 9 and r[1].strip().replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if len(r) >= 9 and r[2].strip().replace(".", "").isdigit()]
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        reasons = sorted({n for r in rows if len(r) >= 9 for n, v in zip(names, r[5:9]) if v.strip() == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


# ---------------------------------------------------------------- CPU baseline (oracle)
WORKLOAD = ("MR-Brain 256x256x128: 30 rflow steps (CFG batch 2, latent 1x4x64x64x32) + VAE decode as 4 depth "
            "windows ROI (24,64,32) overlap 0.25")


def workload_config() -> dict:
    """The ``config`` object of every volume line, identical in both arms."""
    return {"workload": WORKLOAD,
            "networks": "MAISI rflow UNet [64,128,256,512] + VAE decoder [64,128,256], random init",
            "inputs": "synthetic N(0,1) latent; MR-Brain spacing (0.94,0.94,1.36), modality 9, guidance 2",
            "l2": "working set far above L2 (VAE activations 2.1 GB per tensor): no flush needed"}


def _cpu_model() -> str:
    try:
        return next(line.split(":", 1)[1].strip() for line in Path("/proc/cpuinfo").read_text().splitlines()
                    if line.startswith("model name"))
    except (OSError, StopIteration):
        return "unknown"


class CpuSample:
    """The reference's arithmetic restated in torch on the host CPU (``oracle/``), one bounded sample
    of the volume workload: one guided UNet step (CFG batch 2, 64x64x32) and the VAE decoder on one
    (8, 64, 32) latent slab. A volume is 30 UNet steps plus the 4 decode windows, whose work is 12
    such slabs (4 x 24 / 8 depth planes), so the volume time is ``30 x unet_s + 12 x slab_s``.
    Imports only the oracle: no product code is loaded on this path."""

    def __init__(self) -> None:
        from oracle import networks_ref as N
        from oracle import production as OP

        self.N = N
        self.threads = len(os.sched_getaffinity(0))
        torch.set_num_threads(self.threads)
        self.unet_w = OP.parameters("unet", seed=0)
        self.vae_w = OP.parameters("vae", seed=1)
        self.unet_ctor, self.vae_ctor = OP.UNET, OP.VAE
        gen = torch.Generator().manual_seed(0)
        self.z = torch.randn(LATENT, generator=gen)
        self.slab = torch.randn((1, 4, 8, 64, 32), generator=gen)
        self.spacing = N.image_spacing_tensor(SPACING)
        starts = N.window_starts(LATENT[2:], DECODE_ROI, N.scan_interval(LATENT[2:], DECODE_ROI, DECODE_OVERLAP))
        self.windows = math.prod(len(s) for s in starts)
        self.slabs_per_volume = self.windows * math.prod(DECODE_ROI) / (8 * 64 * 32)

    def run(self) -> dict:
        N = self.N
        with torch.inference_mode():
            t0 = time.perf_counter()
            N.guided_velocity(self.z, 1000.0, torch.tensor([MODALITY]), self.spacing, self.unet_w, self.unet_ctor,
                              GUIDANCE)
            t1 = time.perf_counter()
            N.decode_vae(self.slab, self.vae_w, self.vae_ctor)
            t2 = time.perf_counter()
        unet_s, slab_s = t1 - t0, t2 - t1
        per_volume = STEPS_RFLOW * unet_s + self.slabs_per_volume * slab_s
        return {"value": 60.0 / per_volume, "unit": UNIT, "cores": self.threads, "kind": "port",
                "sample_s": t2 - t0, "per_volume_s": per_volume,
                "sample": (f"torch-CPU fp32 oracle on {self.threads} threads ({_cpu_model()}): one guided UNet step "
                           f"(CFG batch 2, 64x64x32) {unet_s:.2f} s x {STEPS_RFLOW} + the VAE decoder on one "
                           f"(8,64,32) latent slab {slab_s:.2f} s x {self.slabs_per_volume:g} (the {self.windows} "
                           f"windows of {DECODE_ROI}) = {per_volume:.1f} s per volume")}


def cpu_baseline() -> dict:
    sample = CpuSample()
    sample.run()  # warm-up (first-touch of the weights, oneDNN primitive creation)
    return sample.run()


def run_reference(args, rank: int) -> None:
    """``--impl reference``: the oracle port on all host cores. Each step is one bounded sample
    (``CpuSample``) timed on the host; ``ms_per_step`` is that sample's wall time, ``value`` the
    volumes/min the sample extrapolates to (``extrapolation``)."""
    if rank != 0:
        return
    sample = CpuSample()
    for _ in range(args.warmup):
        sample.run()
    samples = [sample.run() for _ in range(args.steps)]
    value = statistics.median(s["value"] for s in samples)
    sample_ms = statistics.median(s["sample_s"] for s in samples) * 1e3
    base = {k: v for k, v in samples[-1].items() if k not in ("sample_s", "per_volume_s")}
    base["value"] = value
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(sample_ms, 1),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (random-init weights, N(0,1) latent)", "config": workload_config(),
            "device": "host CPU",
            "extrapolation": {"step": "one sample: 1 guided UNet step + the VAE decoder on one (8,64,32) slab",
                              "ms_per_step": "wall time of one sample (median over the timed steps)",
                              "value": "60 / (30 x UNet-step s + 12 x slab s): volumes/min of whole volumes",
                              "per_volume_s": round(60.0 / value, 2)},
            "cpu_baseline": base,
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- kernel-level cases
# The bench roofline's launch: the VAE decoder's full-resolution 64 -> 64 conv (B, C, D, H, W, O),
# and the DRAM bytes per output voxel ncu measured for that kernel (246.6 MB over 786,432 voxels).
DOMINANT_CONV = (1, 64, 96, 256, 128, 64)
DOMINANT_TRAFFIC_PER_VOXEL = (100.98944e6 + 145.607168e6) / 786432

SWEEP_SHAPES = [(b, c, n, n, n, o) for n in (16, 32, 64) for c, o in ((32, 32), (64, 64), (128, 128), (256, 256))
                for b in (1, 2)] + [(2, 512, 8, 8, 4, 512), (2, 512, 16, 16, 8, 512), (1, 128, 128, 128, 64, 128),
                                    (1, 64, 128, 128, 64, 64)]


def _time_conv(shape, precision: str, iters: int, dev, input_kind: str = "plain") -> tuple[float, float, float]:
    """Device ms of one GEMM launch, its TFLOP/s, and the prepare stage's ms, for one conv3d shape
    (output grid D, H, W): each stage is captured in its own CUDA graph and replayed ``iters`` times
    back to back, so no host gap enters the CUDA-event time (inputs below L2 size stay resident).

    ``input_kind``: plain (the input as is), norm (group-norm affine + SiLU applied
    by the prepare pass) or tri (trilinear 2x upsampling of a half-grid input).
    """
    from ctmr_b200 import ops

    b, c, d, h, w, o = shape
    gen = torch.Generator(device=dev).manual_seed(0)
    sp = (d // 2, h // 2, w // 2) if input_kind == "tri" else (d, h, w)
    x = torch.randn((b, c, *sp), device=dev, generator=gen).contiguous(memory_format=torch.channels_last_3d)
    wt = torch.randn((o, c, 3, 3, 3), device=dev, generator=gen) / (27 * c) ** 0.5
    bias = torch.randn(o, device=dev, generator=gen)
    packed = ops.pack_weight(wt, precision)
    kw = {}
    if input_kind == "norm":
        affine = torch.stack([torch.rand((b, c), device=dev, generator=gen) + 0.5,
                              torch.randn((b, c), device=dev, generator=gen)], dim=-1).contiguous()
        kw = {"affine": affine, "silu": True}
    elif input_kind == "tri":
        kw = {"trilinear": True}
    for _ in range(2):
        ops.conv3d(x, packed, bias, **kw)
    prof: list = []
    ops.PROFILE = prof
    ops.conv3d(x, packed, bias, **kw)
    ops.PROFILE = None
    torch.cuda.synchronize(dev)
    gemm = [r for r in prof if r["kind"] == "gemm"]
    flops = gemm[0]["flops"]
    # Device time of each stage without host gaps: one CUDA graph per stage, replayed back to back.
    from ctmr_b200 import _lib

    need = _conv_workspace_bytes(x, packed, bias, kw)
    ws = torch.empty(max(need, 1), dtype=torch.uint8, device=dev)
    out = ops.conv3d(x, packed, bias, **kw, workspace=ws, stages=_lib.CONV_PREPARE | _lib.CONV_GEMM)
    times = {}
    for name, stage in (("prepare", _lib.CONV_PREPARE), ("gemm", _lib.CONV_GEMM)):
        if stage == _lib.CONV_PREPARE and need == 0:
            times[name] = 0.0
            continue
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            ops.conv3d(x, packed, bias, **kw, out=out, workspace=ws, stages=stage)
        torch.cuda.current_stream(dev).wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            ops.conv3d(x, packed, bias, **kw, out=out, workspace=ws, stages=stage)
        for _ in range(3):
            graph.replay()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(iters):
            graph.replay()
        end.record()
        torch.cuda.synchronize(dev)
        times[name] = start.elapsed_time(end) / iters
    ms = times["gemm"]
    return ms, flops / (ms * 1e-3) / 1e12, times["prepare"]


def _conv_workspace_bytes(x, packed, bias, kw) -> int:
    """Workspace bytes ops.conv3d needs for this call (by asking with an empty workspace)."""
    from ctmr_b200 import ops

    try:
        ops.conv3d(x, packed, bias, **kw, workspace=torch.empty(0, dtype=torch.uint8, device=x.device), stages=2)
    except ops.WorkspaceTooSmall as e:
        return e.needed
    return 0


def _total_ms(records) -> float:
    return sum(r["start"].elapsed_time(r["end"]) for r in records)


def _breakdown(part: str, records, total_ms: float) -> None:
    """Per-stage and per-shape device times of one eager pass (CUDA events around each launch group)."""
    by_kind: dict[str, float] = {}
    rows: dict[tuple[str, str], list[float]] = {}
    for r in records:
        t = r["start"].elapsed_time(r["end"])
        by_kind[r["kind"]] = by_kind.get(r["kind"], 0.0) + t
        acc = rows.setdefault((r["kind"], r["what"]), [0, 0.0, 0.0])
        acc[0] += 1
        acc[1] += t
        acc[2] += r["flops"]
    other = total_ms - sum(by_kind.values())
    print(json.dumps({"part": part, "total_ms": round(total_ms, 3),
                      "by_kind_ms": {k: round(v, 3) for k, v in sorted(by_kind.items())},
                      "other_ms": round(other, 3)}), flush=True)
    for (kind, what), (n, t, fl) in sorted(rows.items(), key=lambda kv: -kv[1][1]):
        line = {"part": part, "kind": kind, "what": what, "n": n, "ms": round(t, 4),
                "share": round(t / total_ms, 4)}
        if fl:
            line["tflops"] = round(fl / (t * 1e-3) / 1e12, 1)
        print(json.dumps(line), flush=True)


@contextlib.contextmanager
def _one_stream():
    """Every launch on the caller's stream (no side-stream branches), so that the CUDA events of
    a profiled pass bracket each launch alone instead of two overlapping chains."""
    from ctmr_b200 import fast_b200 as A

    was = A.SKIP_SIDE_STREAM
    A.SKIP_SIDE_STREAM = False
    try:
        yield
    finally:
        A.SKIP_SIDE_STREAM = was


def _profile_pass(part: str, fn, dev) -> None:
    from ctmr_b200 import ops

    torch.cuda.synchronize(dev)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    plain = []
    for _ in range(3):
        start.record()
        fn()
        end.record()
        torch.cuda.synchronize(dev)
        plain.append(start.elapsed_time(end))
    prof: list = []
    ops.PROFILE = prof
    torch.cuda._sleep(SPIN_CYCLES)  # the host queues the pass while the device waits: no launch gaps inside
    start.record()
    with _one_stream():
        fn()
    end.record()
    ops.PROFILE = None
    torch.cuda.synchronize(dev)
    total = start.elapsed_time(end)
    print(json.dumps({"part": part, "plain_ms": [round(v, 3) for v in plain], "profiled_ms": round(total, 3)}))
    _breakdown(part, prof, total)


def _time_groupnorm(shape: tuple[int, ...], iters: int, dev: torch.device) -> None:
    """The memory-bound passes around each conv on one (B, C, D, H, W) fp32 tensor, each captured
    as a CUDA graph and replayed ``iters`` times between events: the GroupNorm statistics
    (``ctmr_group_norm_affine``: one read) and the normalise + SiLU + fp16 cast the conv's operand
    pass performs (``ctmr_transform``: one read, one half-size write). GB/s of algorithmic bytes
    against the measured HBM copy bandwidth; inputs above L2 (126 MB) come from HBM."""
    from ctmr_b200 import ops

    b, c, d, h, w = shape
    gen = torch.Generator(device=dev).manual_seed(0)
    x = ops.to_ndhwc(torch.randn((b, c, d, h, w), device=dev, generator=gen))
    gamma = torch.rand(c, device=dev, generator=gen) + 0.5
    beta = torch.randn(c, device=dev, generator=gen)
    affine = ops.group_norm_affine(x, gamma, beta, groups=32, eps=1e-6)
    out = ops.empty_ndhwc(b, c, d, h, w, torch.float16, dev)
    elems = b * c * d * h * w
    peaks, kind = _peaks()
    hbm = float(peaks.get("hbm_gbs", FALLBACK_PEAKS.get("hbm_gbs", 6650.0)))
    passes = {"gn_statistics": (lambda: ops.group_norm_affine(x, gamma, beta, groups=32, eps=1e-6),
                                elems * 4),
              "normalise_silu_fp16": (lambda: ops.transform(x, affine=affine, silu=True, out=out), elems * 6)}
    for name, (fn, nbytes) in passes.items():
        for _ in range(3):
            fn()
        torch.cuda.synchronize(dev)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for _ in range(iters):
                fn()
        g.replay()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        g.replay()
        e1.record()
        torch.cuda.synchronize(dev)
        ms = e0.elapsed_time(e1) / iters
        gbs = nbytes / (ms * 1e-3) / 1e9
        print(json.dumps({"case": name, "shape_bcdhw": list(shape), "ms": round(ms, 4),
                          "algorithmic_bytes": nbytes, "gbs": round(gbs, 1), "frac_of_hbm": round(gbs / hbm, 3),
                          "peak": f"{kind} hbm_gbs {hbm}",
                          "l2": "input above L2" if elems * 4 > 126e6 else "input fits L2 (stays resident)"}),
              flush=True)
        del g


def _time_attention(iters: int, dev: torch.device) -> None:
    """Head-size-32 attention of the UNet's attention levels (batch 2: 2048 tokens x 8 heads, 256 x 16)
    on this library's kernel and on torch's SDPA backends, each captured in a CUDA graph and replayed
    ``iters`` times between CUDA events (inputs stay L2-resident: a kernel comparison)."""
    import torch.nn.functional as F
    from torch.nn.attention import SDPBackend, sdpa_kernel

    from ctmr_b200 import ops

    for length, heads in ((2048, 8), (256, 16)):
        gen = torch.Generator(device=dev).manual_seed(0)
        qkv = torch.randn((2, length, 3 * heads * 32), device=dev, generator=gen).to(torch.float16)
        q, k, v = (t.reshape(2, length, heads, 32).transpose(1, 2) for t in qkv.chunk(3, dim=-1))
        scale = 32 ** -0.5
        runs = {"ctmr_attention_d32": lambda: ops.attention_d32(qkv, heads, scale)}
        for name, backend in (("cudnn", SDPBackend.CUDNN_ATTENTION), ("flash", SDPBackend.FLASH_ATTENTION)):
            def call(backend=backend):
                with sdpa_kernel([backend]):
                    return F.scaled_dot_product_attention(q, k, v, scale=scale)
            runs[name] = call
        for name, fn in runs.items():
            try:
                for _ in range(3):
                    fn()
                torch.cuda.synchronize(dev)
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    for _ in range(iters):
                        fn()
                g.replay()
                torch.cuda.synchronize(dev)
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                g.replay()
                e1.record()
                torch.cuda.synchronize(dev)
                us = e0.elapsed_time(e1) * 1e3 / iters
                print(json.dumps({"case": "attention", "impl": name, "batch": 2, "tokens": length, "heads": heads,
                                  "us": round(us, 2),
                                  "exp2_per_s": round(2 * heads * length * length / (us * 1e-6) / 1e12, 3)}),
                      flush=True)
                del g
            except RuntimeError as e:
                print(json.dumps({"case": "attention", "impl": name, "tokens": length, "error": str(e)[:120]}))


def _time_ct_from_mask(iters: int, dev: torch.device, precision: str) -> None:
    """The CT-from-mask configuration (C4): a 256^3 int16 label mask, its ControlNet condition embedding
    (bit planes formed in the first conv), 30 ControlNet-conditioned rflow steps of the production UNet
    on the 1x4x64^3 latent (one captured CUDA graph per step) and the default-ROI (48,48,64)
    sliding-window decode to 256^3 with HU mapping: the stages of ``pipeline.sample_ct_from_mask_ncdhw``
    with the step graph captured once, timed with CUDA events over ``iters`` volumes."""
    from ctmr_b200 import networks, ops
    from ctmr_b200 import pipeline as P
    from ctmr_b200 import weights as W

    unet = W.random_weights(W.unet_shapes(P.PRODUCTION_UNET), seed=0, device=dev)
    cn = W.random_weights(W.controlnet_shapes(P.PRODUCTION_CONTROLNET), seed=4, device=dev)
    vae = W.random_weights(W.vae_decoder_shapes(P.PRODUCTION_VAE), seed=1, device=dev)
    label = torch.from_numpy(P.synthetic_ct_mask(256, 0)).to(dev)
    shape = (1, 4, 64, 64, 64)
    timesteps, _ = P.set_timesteps_rflow(num_inference_steps=30, input_img_size_numel=64 ** 3)
    embedding = networks.encode_controlnet_condition_ncdhw(ops.LabelBits(label), cn,
                                                            constructor=P.PRODUCTION_CONTROLNET)
    step = P.ControlNetUNetStep(unet, cn, P.PRODUCTION_UNET, P.PRODUCTION_CONTROLNET, shape,
                                conditioning_embedding=embedding, class_label=1,
                                spacing=P.spacing_tensor_ncdhw((1.7, 1.7, 2.0), dev), device=dev)
    step.prepare()
    z0 = torch.randn(shape, device=dev).contiguous(memory_format=torch.channels_last_3d)

    def volume():
        emb = networks.encode_controlnet_condition_ncdhw(ops.LabelBits(label), cn, constructor=P.PRODUCTION_CONTROLNET)
        step.embedding.copy_(emb)
        final = step.sample(z0, timesteps)
        mid = torch.cuda.Event(enable_timing=True)
        mid.record()
        dec = P.sliding_window_decode_ncdhw(final, vae, constructor=P.PRODUCTION_VAE, roi=P.CT_ROI,
                                            overlap=P.CT_OVERLAP, scale_factor=1.0)
        return P.to_hu_ncdhw(dec, label), mid

    hu, _ = volume()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    mids = []
    e0.record()
    for _ in range(iters):
        hu, mid = volume()
        mids.append(mid)
    e1.record()
    torch.cuda.synchronize(dev)
    assert torch.isfinite(hu).all()
    ms = e0.elapsed_time(e1) / iters
    print(json.dumps({"case": "ct", "precision": precision, "iters": iters,
                      "workload": "CT from a 256^3 mask: condition embedding + ControlNet + UNet 30 rflow steps on "
                                  "1x4x64^3 + 4-window (48,48,64) decode to 256^3 + HU",
                      "ms_per_volume": round(ms, 2), "volumes_per_min": round(60000.0 / ms, 2),
                      "last_volume_decode_ms": round(mids[-1].elapsed_time(e1), 2),
                      "timing": "CUDA events around iters back-to-back volumes"}), flush=True)
    step.release()


def run_case(args) -> None:
    from ctmr_b200 import fast_b200 as A
    from ctmr_b200 import pipeline as P
    from ctmr_b200 import weights as W

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    with A.arithmetic_precision(args.precision):
        if args.case in ("sweep", "conv"):
            shapes = SWEEP_SHAPES if args.case == "sweep" else [tuple(int(v) for v in args.shape.split(","))]
            peaks, kind = _peaks()
            peak = float(peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
            for shape in shapes:
                ms, tflops, prep_ms = _time_conv(shape, args.precision, args.iters, dev, args.input)
                print(json.dumps({"case": "conv3d 3x3x3", "shape_bcdhwo": shape, "precision": args.precision,
                                  "input": args.input, "prepare_ms": round(prep_ms, 4),
                                  "gemm_ms": round(ms, 4), "tflops": round(tflops, 1),
                                  "frac_of_peak": round(tflops / peak, 3), "peak": f"{kind} bf16_tflops {peak}"}),
                      flush=True)
            return
        if args.case == "attention":
            _time_attention(args.iters, dev)
            return
        if args.case == "ct":
            _time_ct_from_mask(args.iters, dev, args.precision)
            return
        if args.case == "gn":
            _time_groupnorm(tuple(int(v) for v in args.shape.split(","))[:5], args.iters, dev)
            return
        if args.case in ("unet-step", "breakdown"):
            w = W.random_weights(W.unet_shapes(P.PRODUCTION_UNET), seed=0, device=dev)
            step = P.GuidedUNetStep(w, P.PRODUCTION_UNET, LATENT, class_label=MODALITY,
                                    spacing=P.image_spacing_tensor(SPACING, dev), guidance_scale=GUIDANCE,
                                    device=dev, use_cuda_graph=False)
            step.z.copy_(torch.randn(LATENT, device=dev))
            step.t.fill_(900.0)
            step.dt.fill_(0.01)
            for _ in range(args.iters):
                step._step()
            if args.case == "breakdown":
                _profile_pass("unet-step", step._step, dev)
                graphed = P.GuidedUNetStep(w, P.PRODUCTION_UNET, LATENT, class_label=MODALITY,
                                           spacing=P.image_spacing_tensor(SPACING, dev), guidance_scale=GUIDANCE,
                                           device=dev, use_cuda_graph=True)
                graphed.prepare()
                start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                for _ in range(3):
                    graphed.graph.replay()
                start.record()
                for _ in range(10):
                    graphed.graph.replay()
                end.record()
                torch.cuda.synchronize(dev)
                print(json.dumps({"part": "unet-step", "graph_replay_ms": round(start.elapsed_time(end) / 10, 3),
                                  "launches_per_step": graphed.launches_per_step}), flush=True)
                graphed.release()
        if args.case in ("vae-window", "breakdown"):
            w = W.random_weights(W.vae_decoder_shapes(P.PRODUCTION_VAE), seed=1, device=dev)
            from ctmr_b200 import networks

            z = torch.randn((1, 4, *DECODE_ROI), device=dev)
            for _ in range(args.iters):
                networks.decode_vae_ncdhw(z, w, constructor=P.PRODUCTION_VAE)
            if args.case == "breakdown":
                _profile_pass("vae-window", lambda: networks.decode_vae_ncdhw(z, w, constructor=P.PRODUCTION_VAE),
                              dev)
        torch.cuda.synchronize(dev)
        print(json.dumps({"case": args.case, "precision": args.precision, "iters": args.iters, "ok": True}))


# ---------------------------------------------------------------- GPU arm
class VolumeRun:
    """One precision's volume workload on this rank: the sampler (CUDA-graph UNet step) and the decode,
    with the device-resident timing (``value``) and the end-to-end timing through the public API
    (``e2e``: the latent copied in from pinned host memory, the int16 image read back, every step)."""

    def __init__(self, precision: str, *, unet_w, vae_w, dev, world: int, rank: int, local: int, group,
                 no_graph: bool) -> None:
        from ctmr_b200 import distributed as D
        from ctmr_b200 import fast_b200 as A
        from ctmr_b200 import pipeline as P

        self.D, self.A, self.P = D, A, P
        self.precision, self.dev, self.world, self.local, self.group = precision, dev, world, local, group
        self.unet_w, self.vae_w = unet_w, vae_w
        self.spacing = P.image_spacing_tensor(SPACING, dev)
        self.timesteps, _ = P.set_timesteps_rflow(num_inference_steps=STEPS_RFLOW,
                                                  input_img_size_numel=math.prod(LATENT[2:]))
        seed = rank if group is None else group.index
        self.latent_host = torch.randn(LATENT, generator=torch.Generator().manual_seed(seed)).pin_memory()
        self.latent_dev = self.latent_host.to(dev).contiguous(memory_format=torch.channels_last_3d)
        with A.arithmetic_precision(precision):
            if group is None:
                self.sampler = P.GuidedUNetStep(unet_w, P.PRODUCTION_UNET, LATENT, class_label=MODALITY,
                                                spacing=self.spacing, guidance_scale=GUIDANCE, device=dev,
                                                use_cuda_graph=not no_graph)
            else:
                self.sampler = D.GroupGuidedStep(unet_w, P.PRODUCTION_UNET, LATENT, class_label=MODALITY,
                                                 spacing=self.spacing, guidance_scale=GUIDANCE, device=dev,
                                                 group=group, use_cuda_graph=not no_graph)
            self.sampler.prepare()
        self.volumes_per_step = world if group is None else group.count

    def decode(self, latent: torch.Tensor) -> torch.Tensor | None:
        if self.group is None:
            return self.P.sliding_window_decode_ncdhw(latent, self.vae_w, constructor=self.P.PRODUCTION_VAE,
                                                      roi=DECODE_ROI, overlap=DECODE_OVERLAP, scale_factor=1.0)
        return self.D.group_window_decode(latent, self.vae_w, constructor=self.P.PRODUCTION_VAE, roi=DECODE_ROI,
                                          overlap=DECODE_OVERLAP, scale_factor=1.0, group=self.group)

    def volume(self) -> torch.Tensor | None:
        with self.A.arithmetic_precision(self.precision):
            return self.decode(self.sampler.sample(self.latent_dev, self.timesteps))

    def e2e_step(self):
        P = self.P
        with self.A.arithmetic_precision(self.precision):
            latent = self.latent_host.to(self.dev, non_blocking=True)
            if self.group is None:
                res = P.sample_image_ncdhw(OUTPUT, SPACING, unet_weights=self.unet_w, vae_weights=self.vae_w,
                                           configuration="mr-brain", modality=MODALITY, guidance_scale=GUIDANCE,
                                           latent=latent, roi=DECODE_ROI, overlap=DECODE_OVERLAP, device=self.dev,
                                           sampler=self.sampler)
                return res.image
            final = self.sampler.sample(latent.contiguous(memory_format=torch.channels_last_3d), self.timesteps)
            dec = self.decode(final)
            return None if dec is None else P.to_host_array(P.output_intensities_device(dec, configuration="mr-brain"))

    def barrier(self) -> None:
        if self.world > 1:
            torch.distributed.barrier(device_ids=[self.local])
        torch.cuda.synchronize(self.dev)

    def max_over_ranks(self, value: float) -> float:
        if self.world == 1:
            return value
        t = torch.tensor([value], device=self.dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        return float(t.item())

    def measure(self, steps: int, warmup: int, *, clocks: bool = False) -> dict:
        from ctmr_b200 import ops

        out = None
        for _ in range(warmup):
            out = self.volume()
        self.barrier()
        sampler_clocks = ClockSampler(self.local) if clocks and self.local == 0 else None
        launches0 = ops.LAUNCHES[0]
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        self.barrier()
        start.record()
        for _ in range(steps):
            out = self.volume()
        end.record()
        self.barrier()
        clock_info = sampler_clocks.stop() if sampler_clocks is not None else None
        ms = self.max_over_ranks(start.elapsed_time(end) / steps)
        launches = (ops.LAUNCHES[0] - launches0) / steps
        if out is not None:
            assert torch.isfinite(out).all(), f"non-finite decoded volume ({self.precision})"
        # End to end through the public API with host buffers. The same W untimed warm-up calls: a
        # repeated caller holds the previous image while the next call reads its result back, so the
        # first two calls fill the pinned host cache that every later call reuses.
        image = None
        for _ in range(warmup):
            image = self.e2e_step()
        self.barrier()
        t0 = time.perf_counter()
        for _ in range(steps):
            image = self.e2e_step()
        self.barrier()
        e2e_s = self.max_over_ranks((time.perf_counter() - t0) / steps)
        if image is not None:
            assert image.dtype == np.int16 and image.shape == (1, 1, *OUTPUT)
        return {"ms": ms, "value": self.volumes_per_step * 60000.0 / ms, "launches": launches, "clocks": clock_info,
                "e2e": {"value": round(self.volumes_per_step * 60.0 / e2e_s, 3), "unit": UNIT,
                        "h2d_bytes_per_step": self.latent_host.numel() * self.latent_host.element_size(),
                        "d2h_bytes_per_step": math.prod(OUTPUT) * 2}}

    def release(self) -> None:
        self.sampler.release()


# Cycles of the device spin that holds the stream while the host queues one eager pass (~0.1 s).
SPIN_CYCLES = 200_000_000


def conv_roofline(precision: str, unet_w, vae_w, dev, ms_per_volume: float) -> dict:
    """The dominant launch against the burst peak, and every conv GEMM of one volume against the
    sustained peak (CUDA events around each GEMM stage of one eager pass, queued behind a device
    spin so the host runs ahead of the device and no launch gap lands between a pair of events)."""
    from ctmr_b200 import fast_b200 as A
    from ctmr_b200 import ops
    from ctmr_b200 import pipeline as P

    peaks, peak_kind = _peaks()
    prof: list = []
    with A.arithmetic_precision(precision), _one_stream():
        timesteps, _ = P.set_timesteps_rflow(num_inference_steps=STEPS_RFLOW,
                                             input_img_size_numel=math.prod(LATENT[2:]))
        eager = P.GuidedUNetStep(unet_w, P.PRODUCTION_UNET, LATENT, class_label=MODALITY,
                                 spacing=P.image_spacing_tensor(SPACING, dev), guidance_scale=GUIDANCE, device=dev,
                                 use_cuda_graph=False)
        eager.z.copy_(torch.randn(LATENT, generator=torch.Generator().manual_seed(0)).to(dev))
        eager.t.fill_(float(timesteps[0]))
        eager.dt.fill_(P.euler_dt(timesteps[0], timesteps[1]))
        ops.PROFILE = prof
        torch.cuda.synchronize(dev)
        torch.cuda._sleep(SPIN_CYCLES)  # the device waits while the host queues the whole pass
        eager._step()
        unet_part = list(prof)
        del prof[:]
        torch.cuda.synchronize(dev)
        torch.cuda._sleep(SPIN_CYCLES)
        P.sliding_window_decode_ncdhw(eager.z, vae_w, constructor=P.PRODUCTION_VAE, roi=DECODE_ROI,
                                      overlap=DECODE_OVERLAP, scale_factor=1.0)
        vae_part = list(prof)
        ops.PROFILE = None
        torch.cuda.synchronize(dev)
        unet_gemm = [r for r in unet_part if r["kind"] == "gemm"]
        vae_gemm = [r for r in vae_part if r["kind"] == "gemm"]
        conv_ms = STEPS_RFLOW * _total_ms(unet_gemm) + _total_ms(vae_gemm)
        conv_flop = STEPS_RFLOW * sum(r["flops"] for r in unet_gemm) + sum(r["flops"] for r in vae_gemm)
        agg = conv_flop / (conv_ms * 1e-3) / 1e12
        sustained = float(peaks.get("bf16_tflops_sustained", FALLBACK_PEAKS["bf16_tflops_sustained"]))
        burst = float(peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
        # The largest launch class: the decoder's full-resolution 64 -> 64 conv (GN + SiLU input),
        # one launch timed by CUDA-graph replay on the device (no host gaps), against the burst peak.
        dom_ms, dom_tflops, dom_prep_ms = _time_conv(DOMINANT_CONV, precision, 5, dev, "norm")
    b_, c_, d_, h_, w_, o_ = DOMINANT_CONV
    vox = b_ * d_ * h_ * w_
    return {"bound": "tensor", "achieved": round(dom_tflops, 1), "peak": burst, "unit": "TFLOP/s",
            "frac": round(dom_tflops / burst, 4), "traffic": round(DOMINANT_TRAFFIC_PER_VOXEL * vox),
            "kernel": "conv3d_khcat_kernel<64,2>: VAE decoder full-resolution 64->64 conv "
                      f"{b_}x{c_}x{d_}x{h_}x{w_} (GN affine + SiLU input), the largest launch class",
            "launch_ms": round(dom_ms, 4), "prepare_ms": round(dom_prep_ms, 4),
            "algorithmic_flop": round(2 * vox * o_ * c_ * 27),
            "algorithmic_bytes": vox * (c_ * 2 + o_ * 4),
            "traffic_source": "ncu dram__bytes_read+write of the same kernel on a 1x64x48x128x128 case, "
                              "scaled by voxels",
            "peak_source": f"{peak_kind} bf16_tflops (burst: one launch timed alone)",
            "all_conv_launches": {"achieved": round(agg, 1), "peak": sustained, "frac": round(agg / sustained, 4),
                                  "peak_source": f"{peak_kind} bf16_tflops_sustained",
                                  "launches_per_volume": STEPS_RFLOW * len(unet_gemm) + len(vae_gemm),
                                  "algorithmic_tflop_per_volume": round(conv_flop / 1e12, 2),
                                  "conv_ms_per_volume": round(conv_ms, 2),
                                  "timing": "CUDA events around each GEMM launch of one eager pass, queued "
                                            "behind a device spin so the host runs ahead of the device: the "
                                            "events bracket device time, not host launch gaps"}}


def main() -> None:
    args = _args()
    if args.case != "volume":
        run_case(args)
        return
    if args.impl == "reference":
        # The reference's CPU arithmetic only (the oracle); rank 0 alone under torchrun.
        run_reference(args, int(os.environ.get("RANK", "0")))
        return
    from ctmr_b200 import distributed as D
    from ctmr_b200 import pipeline as P
    from ctmr_b200 import weights as W

    world_env = int(os.environ.get("WORLD_SIZE", "1"))
    rank, world, local = D.init_from_env() if world_env > 1 else (0, 1, 0)
    if world > 1 and args.mode == "partition" and world not in D.GROUP_SIZES:
        raise SystemExit(f"--mode partition needs N in {D.GROUP_SIZES}")
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    unet_w = W.random_weights(W.unet_shapes(P.PRODUCTION_UNET), seed=0, device=dev)
    vae_w = W.random_weights(W.vae_decoder_shapes(P.PRODUCTION_VAE), seed=1, device=dev)
    common = dict(unet_w=unet_w, vae_w=vae_w, dev=dev, world=world, rank=rank, local=local, no_graph=args.no_graph)

    headline_group = D.VolumeGroup(rank, world, world) if world > 1 and args.mode == "partition" else None
    run = VolumeRun(args.precision, group=headline_group, **common)
    head = run.measure(args.steps, args.warmup, clocks=True)
    run.release()

    # The precision-matched line (the reference's own arithmetic is FP32: split-fp16 "exact" products)
    # and the TF32-input mode's line, beside a 16-bit headline.
    other_modes = {}
    if world == 1 and not args.no_fp32_line:
        for mode, dtype in (("fp32", "fp32 (split-fp16 operands, 3 products)"),
                            ("tf32", "tf32 (TF32-rounded operands, fp32 accumulation)")):
            if mode == args.precision:
                continue
            run_m = VolumeRun(mode, group=None, **common)
            m = run_m.measure(args.steps, args.warmup)
            run_m.release()
            other_modes[mode] = {"value": round(m["value"], 3), "unit": UNIT, "ms_per_step": round(m["ms"], 2),
                                 "e2e": m["e2e"], "gpu_launches": int(m["launches"]), "dtype": dtype}

    # The north-star partition beside the replicas: all N GPUs on one volume.
    partition = None
    if world > 1 and headline_group is None and world in D.GROUP_SIZES:
        # A failure that every rank meets alike (a Python error of the partition's set-up) is
        # reported in the line instead of taking the measured replicas with it.
        prun = None
        try:
            prun = VolumeRun(args.precision, group=D.VolumeGroup(rank, world, world), **common)
            m = prun.measure(args.steps, args.warmup)
            partition = {"value": round(m["value"], 3), "unit": UNIT, "ms_per_volume": round(m["ms"], 2),
                         "ranks_per_volume": world, "e2e": m["e2e"], "parallelism": D.describe_partition(world)}
        except Exception as e:  # noqa: BLE001
            partition = {"error": f"{type(e).__name__}: {e}"[:300], "ranks_per_volume": world}
        finally:
            if prun is not None:
                prun.release()

    roofline = conv_roofline(args.precision, unet_w, vae_w, dev, head["ms"]) if world == 1 else None
    if rank == 0:
        base = None if (world > 1 or args.no_cpu_baseline) else cpu_baseline()
        line = {
            "metric": METRIC, "value": round(head["value"], 3), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(head["ms"], 2), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": args.precision, "data": "synthetic (random-init weights, N(0,1) latent)",
            "config": workload_config(),
            "parallelism": ("single GPU" if world == 1 else D.describe_partition(world) if headline_group else
                            f"{world} replicas (one volume per GPU per step, no data-path collective)"),
            "cuda_graph": not args.no_graph,
            "e2e": head["e2e"], "gpu_launches": int(head["launches"]), "clocks": head["clocks"],
            "roofline": roofline, "cpu_baseline": base,
        }
        line.update(other_modes)
        if partition is not None:
            line["partition"] = partition
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.barrier(device_ids=[local])
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
