"""Encoder-attention benchmark: audio-seconds per second through the attention plugins.

    python bench.py [--gpus N] [--steps K] [--warmup W]
                    [--workload parakeet|parakeet_long|zipformer|zipformer_fused|ragged|
                                parakeet_conv|zipformer_conv]
    python bench.py --impl reference ...   # the reference math on the host cores

A *step* is one encoder forward's worth of attention calls over one batch:
* ``parakeet`` (default): 24 Conformer layers of
  ``parakeet_relative_attention`` on 256 utterances x 375 frames, fp16, 8 x 128 heads,
  each layer with its own inputs (590 MB of QKV per layer, far above the 126 MB L2).
* ``parakeet_long`` (config 4, long-form): the same on 16 utterances x 3000 frames with
  valid lengths U[1500, 3000] (295 MB of QKV per layer).
* ``zipformer``: every layer of the six Zipformer stacks
  (2/2/4/5/4/2 layers at T = 750/375/188/94/188/375), each layer one
  ``zipformer_relative_attention`` call plus three ``zipformer_attention_value`` calls,
  bf16, 256 utterances.
* ``parakeet_conv`` / ``zipformer_conv``: the encoders' convolution modules of one pass
  (Parakeet: 24 ``parakeet_conformer_convolution`` calls at 256 x 375 x 1024, kernel 9,
  f16; Zipformer: two ``zipformer_convolution`` calls per layer of the config-3 stacks,
  kernels 31/31/15/15/15/31, bf16).

The default line also carries the other workloads as sub-objects, each with its own
timed region: ``zipformer``, ``parakeet_long``, ``zipformer_fused``, ``parakeet_conv`` and
``zipformer_conv``.

``value`` = audio seconds of all ranks' batches x K / max-over-ranks device time of the
K steps (CUDA events, inputs resident in HBM). ``e2e`` = the same metric through the
public operator API with host (pinned) inputs copied in and the outputs copied out
inside the timed region. Under torchrun each rank runs its own batches (weak scaling,
no collective on the data path; one barrier and one max-reduction of the timings).
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time
from datetime import timedelta
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
METRIC = "encoder-attention audio-sec/sec (RTFx)"
UNIT = "audio-s/s"


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=("ours", "reference"), default="ours")
    p.add_argument("--workload", choices=("parakeet", "parakeet_long", "zipformer",
                                          "zipformer_fused", "ragged", "parakeet_conv",
                                          "zipformer_conv"),
                   default="parakeet")
    p.add_argument("--batch", type=int, default=None,
                   help="utterances per GPU (default 256; 16 for parakeet_long)")
    p.add_argument("--e2e-steps", type=int, default=2)
    p.add_argument("--deal", choices=("dynamic", "longest_first", "round_robin"),
                   default="dynamic",
                   help="ragged workload: how batches are dealt to ranks (dynamic: taken one at "
                        "a time, longest first, from a counter shared through a TCPStore)")
    p.add_argument("--cpu-seconds", type=float, default=10.0)
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-gpu-reference", action="store_true",
                   help="leave out the reference pipeline timed on this GPU")
    p.add_argument("--no-secondary", action="store_true",
                   help="default workload only: leave out the zipformer, parakeet_long and "
                        "zipformer_fused sub-lines")
    args = p.parse_args()
    if args.batch is None:
        args.batch = 16 if args.workload == "parakeet_long" else 256
    return args


def parakeet_shape(args):
    """(frames, shortest valid length) of the Parakeet workload: config 2 or config 4."""
    return (3000, 1500) if args.workload == "parakeet_long" else (375, 60)


def is_parakeet(args) -> bool:
    return args.workload in ("parakeet", "parakeet_long")


def load_peaks() -> dict:
    path = REPO / "MEASURED_PEAKS.json"
    if path.is_file():
        d = json.loads(path.read_text())
        return dict(hbm_gbs=d["hbm_gbs"], bf16_tflops=d["bf16_tflops"],
                    bf16_tflops_sustained=d.get("bf16_tflops_sustained", d["bf16_tflops"]),
                    source="measured")
    return dict(hbm_gbs=6650.0, bf16_tflops=1590.0, bf16_tflops_sustained=1400.0,
                source="fallback")


def load_traffic(kernel_key: str, algorithmic_bytes: float):
    """DRAM bytes per launch of ``kernel_key``, scaled from the committed ncu capture.

    ``profiles/dram_traffic.txt`` holds, per kernel, the ``dram__bytes_read.sum +
    dram__bytes_write.sum`` of one captured launch and that launch's algorithmic bytes.
    The capture is a smaller case than the benchmark's; traffic grows with the units
    processed, so it is scaled by the ratio of algorithmic bytes. None if absent.
    """
    path = REPO / "profiles" / "dram_traffic.txt"
    if not path.is_file():
        return None
    for line in path.read_text().splitlines():
        parts = line.split()
        if len(parts) >= 3 and parts[0] == kernel_key and not line.startswith("#"):
            try:
                return float(parts[1]) / float(parts[2]) * algorithmic_bytes
            except (ValueError, ZeroDivisionError):
                return None
    return None


# ---- clocks sampling ------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("pci.bus_id,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, bus_id: str | None):
        self.bus_id = (bus_id or "").lower()
        self.proc = None
        self.path = Path(os.environ.get("TMPDIR", "/tmp")) / f"fga_clocks_{os.getpid()}.csv"

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self) -> dict | None:
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        for line in self.path.read_text().splitlines():
            parts = [s.strip() for s in line.split(",")]
            if len(parts) < 9:
                continue
            rows.append(parts)
        if self.bus_id:
            mine = [r for r in rows if r[0].lower() == self.bus_id]
            rows = mine or [r for r in rows if r[0] == rows[0][0]]
        elif rows:
            rows = [r for r in rows if r[0] == rows[0][0]]
        self.path.unlink(missing_ok=True)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": float(rows[0][2]) if rows[0][2].replace(".", "").isdigit() else None,
                "samples": len(rows), "reasons": reasons}


# ---- distributed plumbing -----------------------------------------------------------------
def init_dist(args):
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "ours":
        torch.cuda.set_device(local)
    if world > 1 and args.impl == "ours":
        import torch.distributed as dist

        dist.init_process_group(backend="nccl", timeout=timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def allreduce_max(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def allgather_floats(x: float, world: int) -> list:
    """Every rank's value of ``x``, in rank order (one collective, all ranks call it)."""
    if world == 1:
        return [x]
    import torch
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    out = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(out, t)
    return [float(o.item()) for o in out]


def barrier(world: int):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


# ---- workloads -----------------------------------------------------------------------------
def build_parakeet(args, rank):
    import torch

    from fast_gpu_asr_b200 import workloads as wl

    frames, low = parakeet_shape(args)
    layers = []
    for i in range(wl.PARAKEET_LAYERS):
        lens = wl.parakeet_lengths(args.batch, frames, low, seed=1000 * rank + 7)
        layers.append(wl.make_parakeet_layer(args.batch, frames, 8, 128, torch.float16, "cuda",
                                             seed=1000 * rank + i, lengths=lens))
    torch.cuda.synchronize()
    audio = wl.parakeet_audio_seconds(layers[0].valid_lengths)
    flops = wl.parakeet_flops(layers[0].valid_lengths, frames, 8, 128)
    nbytes = wl.parakeet_bytes(args.batch, frames, 8, 128, 2)
    outs = [torch.empty((args.batch, frames, 1024), dtype=torch.float16, device="cuda")
            for _ in range(2)]
    return layers, outs, audio, flops, nbytes


def run_parakeet_step(layers, outs, stream, events=None):
    from fast_gpu_asr_b200.attention import parakeet_relative_attention

    for i, L in enumerate(layers):
        if events is not None:
            events[i][0].record(stream)
        parakeet_relative_attention(L.qkv, L.position, L.content_bias, L.position_bias,
                                    L.valid_lengths, L.scale, out=outs[i % 2], stream=stream)
        if events is not None:
            events[i][1].record(stream)


def build_zipformer(args, rank, fused=False):
    import torch

    from fast_gpu_asr_b200 import workloads as wl

    input_lengths = wl.zipformer_input_lengths(args.batch, seed=1000 * rank + 1)
    stacks = []
    total_bytes = 0.0
    seed = 1000 * rank
    for ds, t, embed, heads, nlayers in wl.ZIPFORMER_STACKS:
        lens = wl.zipformer_stack_lengths(input_lengths, ds)
        weights = torch.empty((args.batch, heads, t, t), dtype=torch.bfloat16, device="cuda")
        layers = []
        for _ in range(nlayers):
            seed += 1
            L = wl.make_zipformer_layer(args.batch, t, embed, heads, torch.bfloat16, "cuda",
                                        seed, lens)
            layers.append(L)
            total_bytes += wl.zipformer_layer_bytes(args.batch, t, embed, heads, 2)
        outs = (torch.empty_like(layers[0].value_a), torch.empty_like(layers[0].nonlin_value))
        if fused:
            # The fused entry point writes head 0's weights only, and both self outputs.
            weights = torch.empty((args.batch, 1, t, t), dtype=torch.bfloat16, device="cuda")
            outs = outs + (torch.empty_like(layers[0].value_b),)
        stacks.append((heads, weights, layers, outs))
    torch.cuda.synchronize()
    return stacks, wl.zipformer_audio_seconds(input_lengths), total_bytes


def zipformer_fused_launch_bytes(stacks):
    """(call, algorithmic bytes, kernels) of every call of one fused step, in call order."""
    out = []
    for heads, weights0, layers, (out_a, out_nl, out_b) in stacks:
        for L in layers:
            n, t = L.projection.shape[:2]
            w0 = n * t * t * 2
            out.append(("zipformer_attention_fused",
                        L.projection.numel() * 2 + L.position.numel() * 2 + L.mask.numel()
                        + 2 * L.value_a.numel() * 2 + 2 * out_a.numel() * 2 + w0, 1))
            out.append(("zipformer_attention_value",
                        w0 + L.nonlin_value.numel() * 2 + out_nl.numel() * 2, 1))
    return out


def run_zipformer_fused_step(stacks, stream, events=None):
    from fast_gpu_asr_b200.attention import zipformer_attention_fused, zipformer_attention_value

    j = 0
    for heads, weights0, layers, (out_a, out_nl, out_b) in stacks:
        for L in layers:
            if events is not None:
                events[j][0].record(stream)
            zipformer_attention_fused(L.projection, L.position, L.mask, L.value_a, L.value_b,
                                      out1=out_a, out2=out_b, weights0=weights0, stream=stream)
            if events is not None:
                events[j][1].record(stream)
                events[j + 1][0].record(stream)
            zipformer_attention_value(weights0, L.nonlin_value, 1, out=out_nl, stream=stream)
            if events is not None:
                events[j + 1][1].record(stream)
            j += 2


def zipformer_launch_bytes(stacks):
    """(kernel, algorithmic bytes) of every launch of one step, in launch order."""
    out = []
    for heads, weights, layers, (out_self, out_nl) in stacks:
        for L in layers:
            n, t = L.projection.shape[:2]
            nhtt = weights.numel() * 2
            out.append(("zipformer_relative_attention",
                        L.projection.numel() * 2 + L.position.numel() * 2 + L.mask.numel()
                        + nhtt))
            for v, o, h in ((L.value_a, out_self, heads), (L.value_b, out_self, heads),
                            (L.nonlin_value, out_nl, 1)):
                used = nhtt if h > 1 else n * t * t * 2
                out.append(("zipformer_attention_value", used + v.numel() * 2 + o.numel() * 2))
    return out


def run_zipformer_step(stacks, stream, events=None):
    from fast_gpu_asr_b200.attention import zipformer_attention_value, zipformer_relative_attention

    j = 0

    def mark(i):
        if events is not None:
            events[j][i].record(stream)

    for heads, weights, layers, (out_self, out_nl) in stacks:
        for L in layers:
            mark(0)
            zipformer_relative_attention(L.projection, L.position, L.mask, out=weights,
                                         stream=stream)
            mark(1)
            j += 1
            for v, o, h in ((L.value_a, out_self, heads), (L.value_b, out_self, heads),
                            (L.nonlin_value, out_nl, 1)):
                mark(0)
                zipformer_attention_value(weights, v, h, out=o, stream=stream)
                mark(1)
                j += 1


# ---- CPU legs (oracle port of the reference math) -----------------------------------------
def cpu_parakeet(seconds: float, frames: int = 375, low: int = 60, per_call: int = 4):
    """Time the oracle (reference math restated on torch CPU) on config-2 (or, with
    frames=3000, config-4) utterances."""
    import torch

    from fast_gpu_asr_b200 import workloads as wl
    from oracle import parakeet_relative_attention as oracle

    torch.set_num_threads(os.cpu_count() or 1)
    layer = wl.make_parakeet_layer(per_call, frames, 8, 128, torch.float16, "cpu", seed=11,
                                   length_low=low)
    args = dict(qkv=layer.qkv.float().numpy(), position=layer.position.float().numpy(),
                content_bias=layer.content_bias.float().numpy(),
                position_bias=layer.position_bias.float().numpy(),
                valid_lengths=layer.valid_lengths.numpy())
    oracle(**args, scale=layer.scale, dtype="float16")  # warm-up
    audio = wl.parakeet_audio_seconds(layer.valid_lengths)
    calls, t0 = 0, time.perf_counter()
    while True:
        oracle(**args, scale=layer.scale, dtype="float16")
        calls += 1
        elapsed = time.perf_counter() - t0
        if elapsed >= seconds:
            break
    value = audio * calls / (elapsed * wl.PARAKEET_LAYERS)
    sample = (f"{calls} calls x {per_call} utterances x {frames} frames (8x128 heads, fp16 "
              f"rounding) = {calls} of the 24 per-forward layer calls on a {per_call}-utterance "
              f"slice; scaled to a 24-layer forward")
    return value, torch.get_num_threads(), sample


def cpu_zipformer(seconds: float):
    import torch

    from fast_gpu_asr_b200 import workloads as wl
    from oracle import zipformer_attention_value, zipformer_relative_attention

    torch.set_num_threads(os.cpu_count() or 1)
    per_call = 2
    input_lengths = wl.zipformer_input_lengths(per_call, seed=3)
    layers = []
    for ds, t, embed, heads, nlayers in wl.ZIPFORMER_STACKS:
        lens = wl.zipformer_stack_lengths(input_lengths, ds)
        L = wl.make_zipformer_layer(per_call, t, embed, heads, torch.bfloat16, "cpu", 3, lens)
        layers.append((heads, nlayers, {k: getattr(L, k).float().numpy() if k != "mask"
                                        else L.mask.numpy() for k in
                                        ("projection", "position", "mask", "value_a", "value_b",
                                         "nonlin_value")}))
    t0 = time.perf_counter()
    forwards = 0.0
    while True:
        for heads, nlayers, x in layers:
            w = zipformer_relative_attention(x["projection"], x["position"], x["mask"], "bfloat16")
            zipformer_attention_value(w, x["value_a"], heads, "bfloat16")
            zipformer_attention_value(w, x["value_b"], heads, "bfloat16")
            zipformer_attention_value(w, x["nonlin_value"], 1, "bfloat16")
        # One pass covers one layer of each stack; a forward has 2/2/4/5/4/2 layers.
        forwards += 6.0 / sum(s[4] for s in wl.ZIPFORMER_STACKS)
        elapsed = time.perf_counter() - t0
        if elapsed >= seconds:
            break
    value = wl.zipformer_audio_seconds(input_lengths) * forwards / elapsed
    sample = (f"{per_call}-utterance slice, one layer of each of the 6 stacks per pass "
              f"(weights + 2 self AV + nonlin AV, bf16 rounding), scaled to a 19-layer forward")
    return value, torch.get_num_threads(), sample


def cpu_convolution(kind: str, seconds: float, per_call: int | None = None):
    """Time the convolution oracle (the reference plugin arithmetic restated in numpy,
    storage-precision rounding per tap) on a slice of the conv workload's utterances."""
    from fast_gpu_asr_b200 import workloads as wl
    from oracle.convolution_oracle import depthwise_convolution

    if per_call is None:
        per_call = 2 if kind == "parakeet" else 4
    rng = np.random.default_rng(5)
    if kind == "parakeet":
        lengths = wl.parakeet_lengths(per_call, 375, 60, seed=7)
        calls = [(rng.normal(0, 1, (per_call, 375, 1024)).astype(np.float32), lengths,
                  wl.PARAKEET_CONV_KERNEL, 1024, "float16", wl.PARAKEET_LAYERS)]
        audio = float(lengths.sum()) * wl.PARAKEET_FRAME_SECONDS
    else:
        in_lengths = wl.zipformer_input_lengths(per_call, seed=1)
        calls = [(rng.normal(0, 1, (per_call, t, embed)).astype(np.float32),
                  wl.zipformer_stack_lengths(in_lengths, ds), wl.ZIPFORMER_CONV_KERNELS[i],
                  embed, "bfloat16", 2 * nl)
                 for i, (ds, t, embed, _, nl) in enumerate(wl.ZIPFORMER_STACKS)]
        audio = float(in_lengths.sum()) * wl.ZIPFORMER_INPUT_FRAME_SECONDS
    weights = [(rng.normal(0, 0.2, (k, c)).astype(np.float32),
                rng.normal(0, 0.1, c).astype(np.float32)) for _, _, k, c, _, _ in calls]
    t0, passes = time.perf_counter(), 0.0
    while True:
        # One call per stack (or one Parakeet layer), scaled to the pass's call count.
        for (x, lens, _, _, dt, reps), (w, b) in zip(calls, weights):
            depthwise_convolution(x, lens, w, b, kind, dt)
        passes += 1.0 / sum(c[5] for c in calls) * len(calls)
        elapsed = time.perf_counter() - t0
        if elapsed >= seconds:
            break
    sample = (f"{per_call}-utterance slice, one conv-module call per "
              + ("layer" if kind == "parakeet" else "stack") + " per pass, scaled to a full pass")
    return audio * passes / elapsed, 1, sample


def cpu_leg(args):
    """The CPU timing function of the workload (seconds -> value, cores, sample)."""
    if args.workload in ("parakeet_conv", "zipformer_conv"):
        return lambda seconds: cpu_convolution(args.workload[:-5], seconds)
    if args.workload == "parakeet_long":
        return lambda seconds: cpu_parakeet(seconds, 3000, 1500, 1)
    return cpu_parakeet if args.workload == "parakeet" else cpu_zipformer


def reference_arm(args, world, rank):
    """`--impl reference`: the reference math (oracle port) on the host cores, rank 0 only."""
    if rank != 0:
        return
    fn = cpu_leg(args)
    per_step = []
    for _ in range(args.warmup):
        fn(min(2.0, args.cpu_seconds))
    for _ in range(args.steps):
        value, cores, sample = fn(args.cpu_seconds / max(1, args.steps) + 0.5)
        per_step.append(value)
    value = statistics.median(per_step)
    config = workload_config(args)
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT,
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": None, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": config["dtype"], "data": "synthetic",
            "config": config,
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port",
                             "sample": sample},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def workload_config(args) -> dict:
    if args.workload in ("parakeet_conv", "zipformer_conv"):
        return {"workload": args.workload, "batch": args.batch,
                "dtype": "f16" if args.workload == "parakeet_conv" else "bf16"}
    if args.workload == "parakeet_long":
        return {"workload": "parakeet_relative_attention (config 4, long-form)",
                "batch": args.batch, "frames": 3000, "heads": 8, "head_dim": 128, "layers": 24,
                "lengths": "U[1500,3000]", "dtype": "f16", "parallelism": f"dp{args.gpus}",
                "l2": "inputs exceed L2 (295 MB QKV per layer, 24 distinct layers)"}
    if args.workload == "parakeet":
        return {"workload": "parakeet_relative_attention (config 2)", "batch": args.batch,
                "frames": 375, "heads": 8, "head_dim": 128, "layers": 24,
                "lengths": "U[60,375]", "dtype": "f16", "parallelism": f"dp{args.gpus}",
                "l2": "inputs exceed L2 (590 MB QKV per layer, 24 distinct layers)"}
    if args.workload == "zipformer_fused":
        return {"workload": "zipformer fused weights + both self-attention values, then the "
                            "nonlinear attention-value call on head 0's weights, per layer "
                            "(config 3 through zipformer_attention_fused: beyond the drop-in "
                            "surface)",
                "batch": args.batch, "stacks_T": [750, 375, 188, 94, 188, 375],
                "layers": [2, 2, 4, 5, 4, 2], "dtype": "bf16", "parallelism": f"dp{args.gpus}",
                "l2": "per-layer inputs of distinct layers; head-0 weights up to 288 MB"}
    if args.workload == "ragged":
        return {"workload": "ragged whole-box run (config 5): 20,000 lognormal utterances, "
                            f"length-sorted batches of 256 dealt {args.deal.replace('_', ' ')}; "
                            "per batch 24 parakeet layers (f16) + 19 zipformer layers (bf16); "
                            "outputs of both models gathered to rank 0",
                "batch": args.batch, "utterances": 20000, "dtype": "f16+bf16",
                "parallelism": f"dp{args.gpus}", "l2": "inputs exceed L2 for all but the "
                "shortest batches; two input sets alternate per layer"}
    return {"workload": "zipformer weights + 3 attention-value calls per layer (config 3)",
            "batch": args.batch, "stacks_T": [750, 375, 188, 94, 188, 375],
            "layers": [2, 2, 4, 5, 4, 2], "dtype": "bf16", "parallelism": f"dp{args.gpus}",
            "l2": "weights tensor up to 1.15 GB per layer exceeds L2"}


# ---- ragged whole-box run (config 5) -------------------------------------------------------
def ragged_arm(args, world, rank, local):
    """Length-sorted batches dealt to ranks (by default dynamically: each rank takes the
    next batch, longest first, from a counter in a TCPStore as soon as it has finished the
    previous one; or longest processing time first by estimated cost; or round-robin); per
    batch the Parakeet stack (24 layers, f16) and the Zipformer stacks (bf16); per-batch
    outputs of both models gathered to rank 0 at the end.

    ``value`` = audio seconds of all utterances / max over ranks of the summed batch time
    (CUDA events around each batch's attention calls, host gaps between the launches
    included; inputs are generated on the device between batches, outside the events).
    ``rank_launch_ms`` sums the events around each launch instead, which leaves the host
    gaps out. One small call of each operator before the first batch loads the kernels.
    The gather is timed separately.
    """
    import torch

    from fast_gpu_asr_b200 import _lib
    from fast_gpu_asr_b200 import workloads as wl
    from fast_gpu_asr_b200.attention import parakeet_relative_attention
    from fast_gpu_asr_b200.sharding import (DynamicDeal, batch_costs, gather_to_rank0,
                                            length_sorted_batches, shard_longest_first,
                                            shard_round_robin)

    _lib.library()
    stream = torch.cuda.Stream()
    durations = wl.ragged_durations()
    plan = length_sorted_batches(durations, args.batch)
    deal = None
    if args.deal == "dynamic":
        import torch.distributed as dist

        if world == 1:
            store = dist.HashStore()
        else:
            store = dist.TCPStore(os.environ.get("MASTER_ADDR", "127.0.0.1"),
                                  int(os.environ.get("MASTER_PORT", "29500")) + 1, world,
                                  rank == 0, timeout=timedelta(seconds=120))
        deal = DynamicDeal(store, np.argsort(-batch_costs(plan), kind="stable"))
        assignment = None
        barrier(world)  # every rank's store client is connected before the first take

        def batches():
            while (b := deal.next()) is not None:
                yield b
        mine_iter = batches()
    else:
        if args.deal == "longest_first":
            assignment = shard_longest_first(batch_costs(plan), world)
        else:
            assignment = [shard_round_robin(len(plan), world, r) for r in range(world)]
        mine_iter = iter(assignment[rank])
    warm_p = wl.make_parakeet_layer(2, 64, 8, 128, torch.float16, "cuda", seed=1,
                                    lengths=np.array([64, 33], np.int32))
    warm_z = wl.make_zipformer_layer(2, 64, 192, 4, torch.bfloat16, "cuda", 1,
                                     np.array([64, 33], np.int64))
    with torch.cuda.stream(stream):
        parakeet_relative_attention(warm_p.qkv, warm_p.position, warm_p.content_bias,
                                    warm_p.position_bias, warm_p.valid_lengths, warm_p.scale,
                                    stream=stream)
        run_zipformer_step([(4, torch.empty((2, 4, 64, 64), dtype=torch.bfloat16, device="cuda"),
                             [warm_z], (torch.empty_like(warm_z.value_a),
                                        torch.empty_like(warm_z.nonlin_value)))], stream)
    stream.synchronize()
    kernel_ms, launch_ms, outputs, z_outputs, launches = 0.0, 0.0, {}, {}, 0
    shapes, z_shapes = {}, {}
    for b in plan:
        lens = np.maximum(1, np.floor(b.lengths / wl.PARAKEET_FRAME_SECONDS)).astype(np.int32)
        shapes[b.index] = (len(lens), int(lens.max()), 1024)
        in_frames = np.maximum(2, np.round(b.lengths / wl.ZIPFORMER_INPUT_FRAME_SECONDS))
        z_shapes[b.index] = []
        for ds, _, embed, heads, _ in wl.ZIPFORMER_STACKS:
            zt = int(wl.zipformer_stack_lengths(in_frames.astype(np.int64), ds).max())
            z_shapes[b.index] += [(len(lens), zt, heads * wl.ZIPFORMER_VALUE_DIM),
                                  (len(lens), zt, 3 * embed // 4)]
    torch.cuda.synchronize()
    wall0 = time.perf_counter()
    for idx in mine_iter:
        b = plan[idx]
        p_lens = np.maximum(1, np.floor(b.lengths / wl.PARAKEET_FRAME_SECONDS)).astype(np.int32)
        t = int(p_lens.max())
        players = [wl.make_parakeet_layer(len(p_lens), t, 8, 128, torch.float16, "cuda",
                                          seed=7919 * idx + i, lengths=p_lens) for i in range(2)]
        in_frames = np.maximum(2, np.round(b.lengths / wl.ZIPFORMER_INPUT_FRAME_SECONDS)).astype(np.int64)
        stacks = []
        for s_i, (ds, _, embed, heads, nlayers) in enumerate(wl.ZIPFORMER_STACKS):
            lens = wl.zipformer_stack_lengths(in_frames, ds)
            zt = int(lens.max())
            layers = [wl.make_zipformer_layer(len(lens), zt, embed, heads, torch.bfloat16, "cuda",
                                              7919 * idx + 100 * s_i + i, lens) for i in range(2)]
            weights = torch.empty((len(lens), heads, zt, zt), dtype=torch.bfloat16, device="cuda")
            outs = (torch.empty_like(layers[0].value_a), torch.empty_like(layers[0].nonlin_value))
            stacks.append((heads, weights, [layers[i % 2] for i in range(nlayers)], outs))
        out = torch.empty((len(p_lens), t, 1024), dtype=torch.float16, device="cuda")
        n_launch = wl.PARAKEET_LAYERS + 4 * sum(len(s[2]) for s in stacks)
        events = [[torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)]
                  for _ in range(n_launch)]
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            start.record(stream)
            for i in range(wl.PARAKEET_LAYERS):
                L = players[i % 2]
                events[i][0].record(stream)
                parakeet_relative_attention(L.qkv, L.position, L.content_bias, L.position_bias,
                                            L.valid_lengths, L.scale, out=out, stream=stream)
                events[i][1].record(stream)
            run_zipformer_step(stacks, stream, events[wl.PARAKEET_LAYERS:])
            end.record(stream)
        end.synchronize()
        kernel_ms += start.elapsed_time(end)
        launch_ms += sum(e[0].elapsed_time(e[1]) for e in events)
        launches += n_launch
        outputs[idx] = out
        # The attention outputs of each stack's last layer (self-attention, nonlinear).
        z_outputs[idx] = [t for s in stacks for t in s[3]]
        del players, stacks
    torch.cuda.synchronize()
    wall_ms = (time.perf_counter() - wall0) * 1000.0
    if deal is not None:
        assignment = deal.assignment(world)
    mine = assignment[rank]
    barrier(world)
    max_ms = allreduce_max(kernel_ms, world)
    rank_ms = allgather_floats(kernel_ms, world)
    rank_launch_ms = allgather_floats(launch_ms, world)
    rank_wall_ms = allgather_floats(wall_ms, world)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    gathered = gather_to_rank0(outputs, shapes, world, rank, "cuda", torch.float16, assignment)
    z_gathered = gather_to_rank0(z_outputs, z_shapes, world, rank, "cuda", torch.bfloat16,
                                 assignment)
    torch.cuda.synchronize()
    gather_s = time.perf_counter() - t0
    if rank == 0:
        assert gathered is not None and len(gathered) == len(plan)
        assert z_gathered is not None and len(z_gathered) == len(plan)
        gathered_bytes = sum(t.numel() * t.element_size() for t in gathered.values()) + sum(
            t.numel() * t.element_size() for ts in z_gathered.values() for t in ts)
        audio = float(durations.sum())
        line = {"metric": METRIC, "value": audio / (max_ms / 1000.0), "unit": UNIT,
                "n_gpus": world, "steps": 1, "warmup": 0, "ms_per_step": max_ms,
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
                "dtype": "f16+bf16", "data": "synthetic", "config": workload_config(args),
                "batches": len(plan), "batches_per_rank": len(mine), "deal": args.deal,
                "rank_busy_ms": rank_ms, "rank_busy_spread": max(rank_ms) / max(min(rank_ms), 1e-9),
                "rank_launch_ms": rank_launch_ms,
                # Host wall time of each rank's batch loop, input generation included: what
                # the dynamic deal balances.
                "rank_wall_ms": rank_wall_ms,
                "rank_wall_spread": max(rank_wall_ms) / max(min(rank_wall_ms), 1e-9),
                "gather_wall_s": gather_s, "gathered_bytes": gathered_bytes,
                "gpu_launches": launches,
                "variant": _lib.last_kernel_variant()}
        print(json.dumps(line), flush=True)


# ---- our arm ---------------------------------------------------------------------------------
def device_bus_id(local: int):
    import torch

    props = torch.cuda.get_device_properties(local)
    bus = getattr(props, "pci_bus_id", None)
    if bus is None:
        return None
    return (f"{getattr(props, 'pci_domain_id', 0):08x}:{bus:02x}:"
            f"{getattr(props, 'pci_device_id', 0):02x}.0")


def sub_args(args, workload: str):
    """The arguments of a secondary workload of the default line (its own default batch)."""
    a = argparse.Namespace(**vars(args))
    a.workload = workload
    a.batch = 16 if workload == "parakeet_long" else 256
    return a


def measure_workload(args, world, rank, local, peaks, *, with_e2e=True, with_cpu=True,
                     with_gpu_reference=False) -> dict:
    """Build one workload, run W warm-up and K timed steps (CUDA events around every launch
    on the launching stream, max over ranks), and return its line fields."""
    import torch

    from fast_gpu_asr_b200 import _lib

    stream = torch.cuda.Stream()
    if is_parakeet(args):
        layers, outs, audio, flops, nbytes = build_parakeet(args, rank)
        launch_kinds = [("parakeet_relative_attention", nbytes)] * len(layers)

        def step(events=None):
            run_parakeet_step(layers, outs, stream, events)
    elif args.workload == "zipformer_fused":
        stacks, audio, _ = build_zipformer(args, rank, fused=True)
        calls = zipformer_fused_launch_bytes(stacks)
        launch_kinds = [(name, nb) for name, nb, _ in calls]
        total_bytes = float(sum(nb for _, nb in launch_kinds))

        def step(events=None):
            run_zipformer_fused_step(stacks, stream, events)
    else:
        stacks, audio, total_bytes = build_zipformer(args, rank)
        launch_kinds = zipformer_launch_bytes(stacks)

        def step(events=None):
            run_zipformer_step(stacks, stream, events)
    n_launch = len(launch_kinds)

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            step()
    stream.synchronize()
    variant = _lib.last_kernel_variant()

    # Timed region: K steps, with events around every launch (on the launching stream).
    events = [[[torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)]
               for _ in range(n_launch)] for _ in range(args.steps)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(device_bus_id(local)) if rank == 0 else None
    barrier(world)
    torch.cuda.synchronize()
    if sampler:
        sampler.start()
        time.sleep(0.3)
    torch.cuda.nvtx.range_push("fga_timed")
    with torch.cuda.stream(stream):
        start.record(stream)
        for k in range(args.steps):
            step(events[k])
        end.record(stream)
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_pop()
    clocks = sampler.stop() if sampler else None
    barrier(world)
    elapsed_ms = start.elapsed_time(end)
    max_ms = allreduce_max(elapsed_ms, world)
    launch_ms = np.array([[e[0].elapsed_time(e[1]) for e in ev] for ev in events])

    total_audio = audio * args.steps * world
    value = total_audio / (max_ms / 1000.0)
    ms_per_step = max_ms / args.steps

    # Per-kernel totals over the timed steps; the roofline is reported for the kernel
    # with the largest share of device time.
    kernels = {}
    for i, (name, nb) in enumerate(launch_kinds):
        k = kernels.setdefault(name, {"ms": 0.0, "bytes": 0.0, "launches": 0})
        k["ms"] += float(launch_ms[:, i].sum())
        k["bytes"] += nb * args.steps
        k["launches"] += args.steps
    busy_ms = sum(k["ms"] for k in kernels.values())
    shares = {name: k["ms"] / busy_ms for name, k in kernels.items()}
    dominant = max(kernels, key=lambda n: kernels[n]["ms"])
    dk = kernels[dominant]
    avg_launch_ms = dk["ms"] / dk["launches"]
    avg_bytes = dk["bytes"] / dk["launches"]

    if is_parakeet(args):
        achieved = flops / (avg_launch_ms / 1000.0) / 1e12
        roofline = {"bound": "tensor", "kernel": dominant, "achieved": achieved,
                    "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                    "frac": achieved / peaks["bf16_tflops"],
                    "traffic": load_traffic(dominant, avg_bytes),
                    "peak_source": f"{peaks['source']} bf16 dense (burst)",
                    "flops_per_launch": flops, "bytes_per_launch": nbytes,
                    "hbm_frac": nbytes / (avg_launch_ms / 1000.0) / 1e9 / peaks["hbm_gbs"],
                    "avg_launch_ms": avg_launch_ms, "variant": variant}
    else:
        achieved = dk["bytes"] / (dk["ms"] / 1000.0) / 1e9
        roofline = {"bound": "hbm", "kernel": dominant, "achieved": achieved,
                    "peak": peaks["hbm_gbs"], "unit": "GB/s",
                    "frac": achieved / peaks["hbm_gbs"],
                    "traffic": load_traffic(dominant, avg_bytes),
                    "peak_source": f"{peaks['source']} HBM copy",
                    "bytes_per_launch": avg_bytes, "avg_launch_ms": avg_launch_ms,
                    "kernel_shares": shares,
                    "kernel_hbm_frac": {n: k["bytes"] / (k["ms"] / 1000.0) / 1e9
                                        / peaks["hbm_gbs"] for n, k in kernels.items()},
                    "step_bytes": total_bytes,
                    "step_hbm_frac": total_bytes / (ms_per_step / 1000.0) / 1e9
                    / peaks["hbm_gbs"],
                    "variant": variant}
    # One kernel per entry point call (the weights and fused calls also queue a 4-byte
    # memset of their work counter, which is not a kernel of this library).
    gpu_launches = args.steps * n_launch

    gpu_ref = None
    if with_gpu_reference and not args.no_gpu_reference:
        if is_parakeet(args):
            gpu_ref = gpu_reference_parakeet(layers, args, world, peaks, ms_per_step)
        else:
            gpu_ref = gpu_reference_zipformer(stacks, audio, world, peaks, ms_per_step)

    e2e = None
    if with_e2e and not args.no_e2e:
        if is_parakeet(args):
            e2e = e2e_parakeet(args, layers, audio, world)
        else:
            e2e = e2e_zipformer(args, stacks, audio, world,
                                fused=args.workload == "zipformer_fused")

    cpu = None
    if with_cpu and rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, cores, sample = cpu_leg(args)(args.cpu_seconds)
        cpu = {"value": v, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample}

    return {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": workload_config(args)["dtype"], "data": "synthetic",
            "config": workload_config(args), "roofline": roofline, "cpu_baseline": cpu,
            "e2e": e2e, "gpu_reference": gpu_ref, "gpu_launches": gpu_launches,
            "clocks": clocks, "audio_seconds_per_step_per_gpu": audio}


# ---- convolution modules ---------------------------------------------------------------------
def build_convolution(kind: str, batch: int, rank: int):
    """Calls of one encoder step's convolution modules, with their inputs resident:
    Parakeet config 2 (24 layers, one Conformer conv module each, 256 x 375 x 1024,
    kernel 9, f16) or Zipformer config 3 (two conv modules per layer, each stack's T,
    embed dim and kernel, bf16). Layers alternate between two input/output buffer sets, so
    consecutive calls do not find their inputs in L2 (stack inputs of 5-75 MB; a call's
    read plus write exceeds the 126 MB L2 for the larger stacks only).
    Returns (calls, audio seconds per step, algorithmic bytes per step)."""
    import torch

    from fast_gpu_asr_b200 import workloads as wl
    from fast_gpu_asr_b200.convolution import parakeet_conformer_convolution, zipformer_convolution

    gen = torch.Generator(device="cuda").manual_seed(4242 + rank)

    def tensors(n, t, c, k, dt, lengths):
        xs = [torch.randn((n, t, c), generator=gen, device="cuda").to(dt) for _ in range(2)]
        ys = [torch.empty_like(xs[0]) for _ in range(2)]
        w = (0.2 * torch.randn((k, c), generator=gen, device="cuda")).to(dt)
        b = (0.1 * torch.randn((c,), generator=gen, device="cuda")).to(dt)
        lens = torch.from_numpy(np.asarray(lengths, np.int32)).cuda()
        return xs, ys, w, b, lens

    calls = []
    if kind == "parakeet":
        lengths = wl.parakeet_lengths(batch, 375, 60, seed=7 + rank)
        xs, ys, w, b, lens = tensors(batch, 375, 1024, wl.PARAKEET_CONV_KERNEL, torch.float16,
                                     lengths)
        for i in range(wl.PARAKEET_LAYERS):
            calls.append((parakeet_conformer_convolution, xs[i % 2], lens, w, b, ys[i % 2]))
        audio = float(lengths.sum()) * wl.PARAKEET_FRAME_SECONDS
    else:
        in_lengths = wl.zipformer_input_lengths(batch, seed=1 + rank)
        for s_i, (ds, t, embed, _, nlayers) in enumerate(wl.ZIPFORMER_STACKS):
            lengths = wl.zipformer_stack_lengths(in_lengths, ds)
            xs, ys, w, b, lens = tensors(batch, t, embed, wl.ZIPFORMER_CONV_KERNELS[s_i],
                                         torch.bfloat16, lengths)
            for i in range(2 * nlayers):
                calls.append((zipformer_convolution, xs[i % 2], lens, w, b, ys[i % 2]))
        audio = float(in_lengths.sum()) * wl.ZIPFORMER_INPUT_FRAME_SECONDS
    nbytes = float(sum(2 * c[1].numel() * c[1].element_size() for c in calls))
    return calls, audio, nbytes


def measure_convolution(args, world, rank, local, peaks, kind: str) -> dict:
    """One step = every conv-module call of an encoder pass; CUDA events around every
    launch on the launching stream, W warm-up and K timed steps, max over ranks."""
    import torch

    cpu = None
    if rank == 0 and not args.no_cpu_baseline:
        value, cores, sample = cpu_convolution(kind, min(3.0, args.cpu_seconds))
        cpu = {"value": value, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample}
    calls, audio, nbytes = build_convolution(kind, 256, rank)
    stream = torch.cuda.Stream()

    def step(events=None):
        for i, (op, x, lens, w, b, y) in enumerate(calls):
            if events is not None:
                events[i][0].record(stream)
            op(x, lens, w, b, out=y, stream=stream)
            if events is not None:
                events[i][1].record(stream)

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            step()
    stream.synchronize()
    events = [[[torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)]
               for _ in calls] for _ in range(args.steps)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(device_bus_id(local)) if rank == 0 else None
    barrier(world)
    torch.cuda.synchronize()
    if sampler:
        sampler.start()
        time.sleep(0.3)
    torch.cuda.nvtx.range_push("fga_timed")
    with torch.cuda.stream(stream):
        start.record(stream)
        for k in range(args.steps):
            step(events[k])
        end.record(stream)
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_pop()
    clocks = sampler.stop() if sampler else None
    barrier(world)
    max_ms = allreduce_max(start.elapsed_time(end), world)
    busy_ms = sum(e[0].elapsed_time(e[1]) for ev in events for e in ev)
    avg_launch_ms = busy_ms / (args.steps * len(calls))
    achieved = nbytes * args.steps / (busy_ms / 1000.0) / 1e9
    name = "parakeet_conformer_convolution" if kind == "parakeet" else "zipformer_convolution"
    return {
        "value": audio * args.steps * world / (max_ms / 1000.0), "unit": UNIT,
        "ms_per_step": max_ms / args.steps,
        "dtype": "f16" if kind == "parakeet" else "bf16",
        "config": {"workload": f"{kind} conv modules of one encoder pass "
                               + ("(24 layers, 256 x 375 x 1024, kernel 9)" if kind == "parakeet"
                                  else "(2 per layer, config-3 stacks, kernels 31,31,15,15,15,31)"),
                   "batch": 256, "l2": "two buffer sets alternate between layers"},
        "roofline": {"bound": "hbm", "kernel": name, "achieved": achieved,
                     "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": achieved / peaks["hbm_gbs"],
                     "traffic": load_traffic(name, nbytes / len(calls)),
                     "peak_source": f"{peaks['source']} HBM copy",
                     "bytes_per_launch": nbytes / len(calls), "avg_launch_ms": avg_launch_ms},
        "cpu_baseline": cpu, "gpu_launches": len(calls) * args.steps, "clocks": clocks,
    }


# Secondary workloads carried in the default line (same K and W, each its own timed region).
SECONDARY = ("zipformer", "parakeet_long", "zipformer_fused")
CONV_SECONDARY = ("parakeet", "zipformer")


def ours_arm(args, world, rank, local):
    import torch

    from fast_gpu_asr_b200 import _lib

    _lib.library()
    peaks = load_peaks()
    if args.workload in ("parakeet_conv", "zipformer_conv"):
        # The convolution modules alone (the same measurement the default line carries).
        sub = measure_convolution(args, world, rank, local, peaks, args.workload[:-5])
        line = {"metric": "encoder-convolution audio-sec/sec (RTFx)", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "data": "synthetic", **sub}
        if rank == 0:
            print(json.dumps(line), flush=True)
        return
    line = measure_workload(args, world, rank, local, peaks,
                            with_gpu_reference=args.workload in ("parakeet", "zipformer"))
    if args.workload == "parakeet" and not args.no_secondary:
        for name in SECONDARY:
            torch.cuda.empty_cache()
            sub = measure_workload(sub_args(args, name), world, rank, local, peaks,
                                   with_e2e=name != "zipformer_fused",
                                   with_cpu=name != "zipformer_fused",
                                   with_gpu_reference=name == "zipformer")
            line[name] = {k: sub[k] for k in ("value", "unit", "ms_per_step", "dtype", "config",
                                              "roofline", "e2e", "cpu_baseline",
                                              "gpu_reference", "gpu_launches", "clocks")}
        for kind in CONV_SECONDARY:
            torch.cuda.empty_cache()
            line[f"{kind}_conv"] = measure_convolution(args, world, rank, local, peaks, kind)
    if rank == 0:
        print(json.dumps(line), flush=True)


# ---- the reference pipeline on this GPU ------------------------------------------------------
def _time_ms(fn, stream, reps: int) -> float:
    import torch

    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        fn()
        torch.cuda.synchronize()
        start.record(stream)
        for _ in range(reps):
            fn()
        end.record(stream)
    torch.cuda.synchronize()
    return start.elapsed_time(end) / reps


def gpu_reference_parakeet(layers, args, world, peaks, our_ms_per_step):
    """The reference plugin's pipeline restated on this B200 (TensorRT and the plugin
    sources cannot run here): per layer and head, the three cuBLAS GEMMs it issues
    (``parakeet_relative_attention_plugin.cu:1052-1133``: (Q+u)K^T and (Q+v)P^T into HBM
    score buffers, then weights x V) timed with CUDA events through torch.matmul, plus its
    softmax pass (``:452-538``: reads both score buffers, writes the weights) and bias pass
    (``:268-281``) counted at the measured HBM copy rate, i.e. at their floor. The sum is a
    lower bound on the reference pipeline's time on this GPU. ``torch_eager_ms`` also times
    the whole pipeline in unfused torch ops (an upper bound)."""
    import torch

    L = layers[0]
    n, t, c3 = L.qkv.shape
    c, heads, d = c3 // 3, 8, 128
    dt = L.qkv.dtype
    qkv = L.qkv.view(n, t, 3, heads, d)
    q = [qkv[:, :, 0, h].contiguous() for h in range(heads)]     # [N, T, D]
    k = [qkv[:, :, 1, h].contiguous() for h in range(heads)]
    v = [qkv[:, :, 2, h].contiguous() for h in range(heads)]
    p = [L.position[0, :, h * d:(h + 1) * d].contiguous() for h in range(heads)]  # [2T-1, D]
    scores = torch.empty((n, t, t), dtype=dt, device="cuda")
    pos_scores = torch.empty((n, t, 2 * t - 1), dtype=dt, device="cuda")
    out = torch.empty((n, t, d), dtype=dt, device="cuda")
    stream = torch.cuda.Stream()

    def gemms():
        for h in range(heads):
            torch.matmul(q[h], k[h].transpose(1, 2), out=scores)
            torch.matmul(q[h], p[h].t(), out=pos_scores)
            torch.matmul(scores, v[h], out=out)

    gemm_ms = _time_ms(gemms, stream, 3)
    elem = 2
    softmax_bytes = heads * n * t * t * elem * 3            # read two score rows, write weights
    bias_bytes = 3 * n * t * c * elem                        # read Q, write Q+u and Q+v
    floor_ms = (softmax_bytes + bias_bytes) / (peaks["hbm_gbs"] * 1e9) * 1e3
    layer_ms = gemm_ms + floor_ms
    lengths = L.valid_lengths.long()

    def eager():
        qf = L.qkv.view(n, t, 3, heads, d).permute(2, 0, 3, 1, 4)
        qu = (qf[0].float() + L.content_bias.float()[None, :, None, :]).to(dt)
        qv = (qf[0].float() + L.position_bias.float()[None, :, None, :]).to(dt)
        pp = L.position[0].view(2 * t - 1, heads, d).permute(1, 0, 2)
        sc = torch.matmul(qu, qf[1].transpose(-1, -2))
        ps = torch.matmul(qv, pp.transpose(-1, -2))
        shifted = ps.as_strided((n, heads, t, t), (ps.stride(0), ps.stride(1), 2 * t - 2, 1),
                                ps.storage_offset() + t - 1)
        logits = (sc.float() + shifted.float()) * L.scale
        mask = torch.arange(t, device="cuda")[None, :] >= lengths[:, None]
        logits.masked_fill_(mask[:, None, None, :], float("-inf"))
        w = torch.softmax(logits, dim=-1).nan_to_num_(0.0).to(dt)
        return torch.matmul(w, qf[2])

    eager_ms = _time_ms(eager, stream, 2)
    nlayers = len(layers)
    ref_step_ms = allreduce_max(layer_ms * nlayers, world)
    audio = wl_audio_parakeet(L)
    return {"value": audio * world / (ref_step_ms / 1000.0), "unit": UNIT,
            "ms_per_step": ref_step_ms,
            "what": "reference plugin pipeline on this GPU: its cuBLAS GEMMs (timed) + its "
                    "softmax and bias passes at the measured HBM copy rate (a lower bound)",
            "gemm_ms_per_layer": gemm_ms, "softmax_floor_ms_per_layer": floor_ms,
            "torch_eager_ms_per_layer": eager_ms,
            "speedup_of_ours": ref_step_ms / our_ms_per_step}


def wl_audio_parakeet(layer) -> float:
    from fast_gpu_asr_b200 import workloads as wl

    return wl.parakeet_audio_seconds(layer.valid_lengths)


def gpu_reference_zipformer(stacks, audio, world, peaks, our_ms_per_step):
    """The reference plugins' pipeline restated on this B200, per layer: the weights plugin's
    per-head cuBLAS GEMM writing the content scores into the [N, H, T, T] output
    (``zipformer_relative_attention_plugin.cu:490-566``) and the three attention-value
    calls (``zipformer_attention_value_plugin.cu:438-572``, cuBLAS GEMMs here) timed with CUDA
    events through torch.matmul, plus the weights plugin's in-place softmax pass (reads the
    scores and positional queries, writes the weights) counted at the measured HBM copy
    rate. The sum is a lower bound on the reference pipeline's time on this GPU."""
    import torch

    stream = torch.cuda.Stream()
    total_ms = 0.0
    per_stack = []
    for heads, weights, layers, (out_self, out_nl, *_) in stacks:
        L = layers[0]
        n, t = L.projection.shape[:2]
        dt = L.projection.dtype
        proj = L.projection.view(n, t, heads, 68)
        q = [proj[:, :, h, :32].contiguous() for h in range(heads)]
        k = [proj[:, :, h, 32:64].contiguous() for h in range(heads)]
        scores = torch.empty((n, t, t), dtype=dt, device="cuda")
        w = weights.view(n, heads, t, t)
        va = L.value_a.view(n, t, heads, 12).permute(0, 2, 1, 3).contiguous()
        vb = L.value_b.view(n, t, heads, 12).permute(0, 2, 1, 3).contiguous()
        vn = L.nonlin_value
        oa = torch.empty_like(va)
        on = torch.empty_like(vn)

        def gemms():
            for h in range(heads):
                torch.matmul(q[h], k[h].transpose(1, 2), out=scores)
            torch.matmul(w, va, out=oa)
            torch.matmul(w, vb, out=oa)
            torch.matmul(w[:, 0], vn, out=on)

        gemm_ms = _time_ms(gemms, stream, 3)
        softmax_bytes = n * heads * t * t * 2 * 2 + n * t * heads * 8
        floor_ms = softmax_bytes / (peaks["hbm_gbs"] * 1e9) * 1e3
        per_stack.append({"T": t, "gemm_ms": gemm_ms, "softmax_floor_ms": floor_ms,
                          "layers": len(layers)})
        total_ms += (gemm_ms + floor_ms) * len(layers)
    ref_step_ms = allreduce_max(total_ms, world)
    return {"value": audio * world / (ref_step_ms / 1000.0), "unit": UNIT,
            "ms_per_step": ref_step_ms,
            "what": "reference plugins' pipeline on this GPU: content-score GEMMs and the "
                    "attention-value GEMMs (timed) + the softmax pass at the measured HBM "
                    "copy rate (a lower bound)",
            "per_stack": per_stack, "speedup_of_ours": ref_step_ms / our_ms_per_step}


def _pipelined(nlayers_total, h2d, compute, d2h):
    """Run one step of ``nlayers_total`` layer calls as a three-stream pipeline.

    Layer i copies its inputs in on the copy-in stream, runs on the compute stream and
    copies its outputs back on the copy-out stream, with device buffers double-buffered
    by i % 2 and CUDA events ordering the reuse: PCIe carries the inputs of layer i+1
    and the outputs of layer i-1 (full duplex) while layer i computes. Returns the step
    function, the stream its first operation runs on and the stream its last one runs
    on."""
    import torch

    s_in, s_c, s_out = torch.cuda.Stream(), torch.cuda.Stream(), torch.cuda.Stream()
    h2d_done = [torch.cuda.Event() for _ in range(2)]
    comp_done = [torch.cuda.Event() for _ in range(2)]
    d2h_done = [torch.cuda.Event() for _ in range(2)]
    used = [False, False]

    def step():
        for i in range(nlayers_total):
            b = i % 2
            if used[b]:
                s_in.wait_event(comp_done[b])   # inputs of buffer b were read
            with torch.cuda.stream(s_in):
                h2d(i, b, s_in)
                h2d_done[b].record(s_in)
            s_c.wait_event(h2d_done[b])
            if used[b]:
                s_c.wait_event(d2h_done[b])     # outputs of buffer b were copied out
            with torch.cuda.stream(s_c):
                compute(i, b, s_c)
                comp_done[b].record(s_c)
            s_out.wait_event(comp_done[b])
            with torch.cuda.stream(s_out):
                d2h(i, b, s_out)
                d2h_done[b].record(s_out)
            used[b] = True

    return step, s_in, s_out


def _time_pipeline(step, s_first, s_last, n, world):
    import torch

    step()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    start.record(s_first)
    for _ in range(n):
        step()
    # The last copy-out depends on every earlier operation of the step.
    end.record(s_last)
    torch.cuda.synchronize()
    return allreduce_max(start.elapsed_time(end), world)


def e2e_parakeet(args, layers, audio, world):
    """Same metric through the public API with pinned host inputs and outputs, copies
    overlapped with compute across layers (three-stream pipeline)."""
    import torch

    from fast_gpu_asr_b200.attention import parakeet_relative_attention

    names = ("qkv", "position", "content_bias", "position_bias", "valid_lengths")
    host_in = [{k: getattr(L, k).cpu().pin_memory() for k in names} for L in layers[:2]]
    dev = [{k: torch.empty_like(getattr(layers[0], k)) for k in names} for _ in range(2)]
    outs = [torch.empty((args.batch, layers[0].qkv.shape[1], 1024), dtype=torch.float16,
                        device="cuda") for _ in range(2)]
    host_out = [torch.empty(o.shape, dtype=o.dtype).pin_memory() for o in outs]
    h2d_bytes = sum(t.numel() * t.element_size() for t in host_in[0].values()) * len(layers)
    d2h_bytes = outs[0].numel() * outs[0].element_size() * len(layers)

    def h2d(i, b, s):
        for k, t in host_in[i % 2].items():
            dev[b][k].copy_(t, non_blocking=True)

    def compute(i, b, s):
        d = dev[b]
        parakeet_relative_attention(d["qkv"], d["position"], d["content_bias"],
                                    d["position_bias"], d["valid_lengths"], layers[0].scale,
                                    out=outs[b], stream=s)

    def d2h(i, b, s):
        host_out[b].copy_(outs[b], non_blocking=True)

    step, s_first, s_last = _pipelined(len(layers), h2d, compute, d2h)
    n = max(1, args.e2e_steps)
    ms = _time_pipeline(step, s_first, s_last, n, world)
    return {"value": audio * n * world / (ms / 1000.0), "unit": UNIT,
            "h2d_bytes_per_step": h2d_bytes, "d2h_bytes_per_step": d2h_bytes, "steps": n,
            "ms_per_step": ms / n, "overlap": "copy-in, compute and copy-out streams"}


def e2e_zipformer(args, stacks, audio, world, fused=False):
    """Same metric through the public API with pinned host inputs and outputs.

    Per layer the step copies in the projection, positions, mask and the three value
    inputs, runs the weights call and the three attention-value calls (fused: the fused
    call and the nonlinear attention-value call), and copies the three attention outputs
    back. The weights stay on the device, as between two plugins of an engine. Copies
    overlap compute across layers (three-stream pipeline).
    """
    import torch

    from fast_gpu_asr_b200.attention import (
        zipformer_attention_fused,
        zipformer_attention_value,
        zipformer_relative_attention,
    )

    names = ("projection", "position", "mask", "value_a", "value_b", "nonlin_value")
    plan = []  # one entry per layer call: (heads, weights, host, dev[2], outs[2], host_outs[2])
    h2d_bytes = d2h_bytes = 0
    for heads, weights, layers, (out_self, out_nl, *_) in stacks:
        L0 = layers[0]
        host = {k: getattr(L0, k).cpu().pin_memory() for k in names}
        dev = [{k: torch.empty_like(getattr(L0, k)) for k in names} for _ in range(2)]
        outs = [[torch.empty_like(out_self), torch.empty_like(out_self),
                 torch.empty_like(out_nl)] for _ in range(2)]
        host_outs = [[torch.empty(o.shape, dtype=o.dtype).pin_memory() for o in outs[0]]
                     for _ in range(2)]
        for _ in range(len(layers)):
            plan.append((heads, weights, host, dev, outs, host_outs))
        h2d_bytes += sum(t.numel() * t.element_size() for t in host.values()) * len(layers)
        d2h_bytes += sum(o.numel() * o.element_size() for o in outs[0]) * len(layers)

    def h2d(i, b, s):
        heads, weights, host, dev, outs, host_outs = plan[i]
        for k in names:
            dev[b][k].copy_(host[k], non_blocking=True)

    def compute(i, b, s):
        heads, weights, host, dev, outs, host_outs = plan[i]
        d, o = dev[b], outs[b]
        if fused:
            zipformer_attention_fused(d["projection"], d["position"], d["mask"], d["value_a"],
                                      d["value_b"], out1=o[0], out2=o[1], weights0=weights,
                                      stream=s)
            zipformer_attention_value(weights, d["nonlin_value"], 1, out=o[2], stream=s)
            return
        zipformer_relative_attention(d["projection"], d["position"], d["mask"], out=weights,
                                     stream=s)
        zipformer_attention_value(weights, d["value_a"], heads, out=o[0], stream=s)
        zipformer_attention_value(weights, d["value_b"], heads, out=o[1], stream=s)
        zipformer_attention_value(weights, d["nonlin_value"], 1, out=o[2], stream=s)

    def d2h(i, b, s):
        heads, weights, host, dev, outs, host_outs = plan[i]
        for o, ho in zip(outs[b], host_outs[b]):
            ho.copy_(o, non_blocking=True)

    step, s_first, s_last = _pipelined(len(plan), h2d, compute, d2h)
    n = max(1, args.e2e_steps)
    ms = _time_pipeline(step, s_first, s_last, n, world)
    return {"value": audio * n * world / (ms / 1000.0), "unit": UNIT,
            "h2d_bytes_per_step": h2d_bytes, "d2h_bytes_per_step": d2h_bytes, "steps": n,
            "ms_per_step": ms / n, "overlap": "copy-in, compute and copy-out streams"}


def main():
    args = parse_args()
    sys.path.insert(0, str(REPO))
    world, rank, local = init_dist(args)
    try:
        if args.impl == "reference":
            reference_arm(args, world, rank)
        elif args.workload == "ragged":
            ragged_arm(args, world, rank, local)
        else:
            ours_arm(args, world, rank, local)
    finally:
        if world > 1 and args.impl == "ours":
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
