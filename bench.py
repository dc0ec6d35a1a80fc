#!/usr/bin/env python3
"""Throughput benchmark of the B200 FP16 conv-stack backend.

Default workload (the configuration the metric is
quoted on): 1920x1088 decode on the MLVC-shaped decoder stand-in (the
upstream MLVC network is absent; mlvc_b200.graph.build_mlvc_decoder_standin
assembles one from the reference's documented decoder I/O, plane sizes and
depth-conv block), 8 independent streams, each a sequence of 64-frame GOPs
with its own recurrent feature state (I-frame = state reset), split 8/N per
GPU, one backend instance per stream.  One step = one frame of every stream
a GPU serves.  Random-init FP16 weights and seeded integer-valued latents
(synthetic: no checkpoints exist here).

Other workloads: `block_stack` (configs[1], the 8-block depthwise residual
stack), `conv3x3`, `mlvc_dec_1080p` / `mlvc_dec_640` /
`mlvcs_dec_640` (one stream of a stand-in), single-operator graphs `op_*`
for kernel work, `entropy_1080p` (scale extraction + FP16 -> int32 symbols).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

N>1 runs under torchrun, one process per GPU; streams and replicas are
independent (no data-path collective), timed on the device, max over ranks.
`--impl reference` times the reference's own CPU backend (compiled from its
sources into oracle/_ref) on the host cores.  Prints one JSON line (rank 0).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
for p in (ROOT, ROOT / "mlvc.cpp_b200"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

from mlvc_b200.graph import (build_block_stack, build_conv3x3, build_mlvc_decoder_standin,  # noqa: E402
                             build_mlvc_encoder_standin, build_mlvcs_decoder_standin)

METRIC = "conv-stack frames/s (config 2 block stack; stand-in for 1080p MLVC decode frames/s)"
UNIT = "frames/s"
FLUSH_BYTES = 256 << 20  # > 126 MB L2


def single_op(name):
    """Single-operator graphs at 544x960 (inputs larger than L2) for kernel
    tuning and ncu captures: dw3x3 (256 ch), conv1x1 (128->256 + LeakyReLU),
    ffn (the block's feed-forward half), dwconv (depthwise + 1x1 + residual),
    mbconv (the block's first half: expand, depthwise, projection + residual)."""
    from mlvc_b200.graph import GraphBuilder, kaiming_normal, small_bias
    rng = np.random.default_rng(0)
    gb = GraphBuilder()
    if name == "op_dw3x3":
        x = gb.input("x", [1, 256, 544, 960])
        w = gb.weight("w", kaiming_normal(rng, (256, 1, 3, 3), 1.0))
        b = gb.weight("b", small_bias(rng, 256))
        gb.output(gb.conv(x, w, b, (1, 1), (1, 1), groups=256), "y")
        inputs = [rng.standard_normal((1, 256, 544, 960), dtype=np.float32).astype(np.float16)]
        desc = "single op: depthwise 3x3 s1 p1, 256 ch @544x960 (NCHW boundary conversion included)"
    elif name == "op_dwconv":
        x = gb.input("x", [1, 256, 1024, 316])
        d = gb.conv(x, gb.weight("dw", kaiming_normal(rng, (256, 1, 3, 3), 1.0)), gb.weight("db", small_bias(rng, 256)),
                    (1, 1), (1, 1), groups=256)
        y = gb.conv(d, gb.weight("w", kaiming_normal(rng, (128, 256, 1, 1), 1.0)), gb.weight("b", small_bias(rng, 128)))
        r = gb.input("r", [1, 128, 1024, 316])
        gb.output(gb.add(y, r), "y")
        inputs = [rng.standard_normal((1, 256, 1024, 316), dtype=np.float32).astype(np.float16),
                  rng.standard_normal((1, 128, 1024, 316), dtype=np.float32).astype(np.float16)]
        desc = ("single op: depthwise 3x3 256 -> 1x1 256->128 + residual @1024x316 (widest image the fused "
                "kernel takes; NCHW boundary conversion included)")
    elif name == "op_mbconv":
        x = gb.input("x", [1, 128, 544, 960])
        t = gb.leaky_relu(gb.conv(x, gb.weight("w1", kaiming_normal(rng, (256, 128, 1, 1))),
                                  gb.weight("b1", small_bias(rng, 256))), 0.01)
        d = gb.conv(t, gb.weight("dw", kaiming_normal(rng, (256, 1, 3, 3), 1.0)), gb.weight("db", small_bias(rng, 256)),
                    (1, 1), (1, 1), groups=256)
        y = gb.conv(d, gb.weight("w2", kaiming_normal(rng, (128, 256, 1, 1), 1.0)), gb.weight("b2", small_bias(rng, 128)))
        gb.output(gb.add(y, x), "y")
        inputs = [rng.standard_normal((1, 128, 544, 960), dtype=np.float32).astype(np.float16)]
        desc = ("single op: inverted residual 1x1 128->256 + LeakyReLU -> depthwise 3x3 -> 1x1 256->128 + residual "
                "@544x960 (the block stack's first half; NCHW boundary conversion included)")
    elif name == "op_ffn":
        x = gb.input("x", [1, 128, 544, 960])
        t = gb.conv(x, gb.weight("w1", kaiming_normal(rng, (512, 128, 1, 1))), gb.weight("b1", small_bias(rng, 512)))
        gate, lin = gb.slice(t, 1, 0, 256), gb.slice(t, 1, 256, 512)
        h = gb.mul(gb.clip(gate, 0.0, 1.0), lin)
        y = gb.conv(h, gb.weight("w2", kaiming_normal(rng, (128, 256, 1, 1), 1.0)), gb.weight("b2", small_bias(rng, 128)))
        gb.output(gb.add(y, x), "y")
        inputs = [rng.standard_normal((1, 128, 544, 960), dtype=np.float32).astype(np.float16)]
        desc = ("single op: FFN 1x1 128->512 -> ReGLU -> 1x1 256->128 + residual @544x960 "
                "(NCHW boundary conversion included)")
    else:
        x = gb.input("x", [1, 128, 544, 960])
        w = gb.weight("w", kaiming_normal(rng, (256, 128, 1, 1)))
        b = gb.weight("b", small_bias(rng, 256))
        gb.output(gb.leaky_relu(gb.conv(x, w, b), 0.01), "y")
        inputs = [rng.standard_normal((1, 128, 544, 960), dtype=np.float32).astype(np.float16)]
        desc = "single op: 1x1 conv 128->256 + LeakyReLU @544x960 (NCHW boundary conversion included)"
    graph, weights = gb.finish()
    return graph, weights, inputs, desc, METRIC.replace("config 2 block stack", desc), []


def workload(name):
    if name.startswith("op_"):
        return single_op(name)
    if name.startswith("mlvc_dec_"):
        width, height = {"mlvc_dec_1080p": (1920, 1088), "mlvc_dec_640": (640, 368)}[name]
        gb, inputs = build_mlvc_decoder_standin(0, width, height)
        desc = (f"MLVC-shaped decoder stand-in @{width}x{height} (the upstream MLVC architecture is absent): documented "
                "decoder I/O (z_raw 1/128, y_raw_0/1 1/16, ref_feature 256ch 1/8, q_index int32 -> x_hat, feature), "
                "hyperprior x8 pixel-shuffle up-sampling, QP-indexed dequantisation, 2+2+2 depth-conv blocks at 256 ch "
                "(the profile's block: 1x1 +LeakyReLU, dw3x3, 1x1 +residual, ReGLU FFN +residual), x8 pixel-shuffle "
                "reconstruction; Kaiming-normal weights, seed 0")
        desc += ("; ref_feature <- feature bound as recurrent state (as the codec pipeline binds decoder input 3 to "
                 "output 1), so it stays on the device between frames")
        metric = f"MLVC-shaped decoder stand-in frames/s @{width}x{height} (stand-in for MLVC decode frames/s)"
        graph, weights = gb.finish()
        return graph, weights, inputs, desc, metric, [(3, 1)]
    if name.startswith("mlvc_enc_"):
        width, height = {"mlvc_enc_1080p": (1920, 1088), "mlvc_enc_640": (640, 368)}[name]
        gb, inputs = build_mlvc_encoder_standin(0, width, height)
        desc = (f"MLVC-shaped encoder stand-in @{width}x{height} (the upstream MLVC architecture is absent): "
                "documented encoder I/O (x [1,3,H,W], ref_feature 256ch 1/8, q_index int32 -> feature, z_raw 1/128, "
                "y_raw_0/1 1/16), pixel-unshuffle x8 analysis with 3x3 s2 down-sampling, hyperprior encoder and "
                "decoder, the y0 / y1 latent quantisation tails, the recurrent feature update; Kaiming-normal "
                "weights, seed 0; ref_feature <- feature bound as recurrent state (input 1 <- output 0)")
        metric = f"MLVC-shaped encoder stand-in frames/s @{width}x{height} (stand-in for MLVC encode frames/s)"
        graph, weights = gb.finish()
        return graph, weights, inputs, desc, metric, [(1, 0)]
    if name == "mlvcs_dec_640":
        gb, inputs = build_mlvcs_decoder_standin(0, 640, 368)
        desc = ("MLVC-S-shaped decoder stand-in @640x368 (the upstream MLVC-S architecture is absent): documented "
                "small-profile sizes (feature 96, y/z 48 ch, hidden/recon 192, y_scale_repeat 4, mini hyperprior "
                "z 1/64 with 2 blocks), x4 hyperprior up-sampling, QP-indexed dequantisation, 2+2+2 depth-conv "
                "blocks (192 / 96 / 192 ch), x8 pixel-shuffle reconstruction; Kaiming-normal weights, seed 0; "
                "ref_feature <- feature bound as recurrent state")
        metric = "MLVC-S-shaped decoder stand-in frames/s @640x368 (stand-in for MLVC-S P-frame decode frames/s)"
        graph, weights = gb.finish()
        return graph, weights, inputs, desc, metric, [(3, 1)]
    if name == "conv3x3":
        gb, inputs = build_conv3x3(0)
        desc = ("config1-conv3x3: one FP16 3x3 s1 p1 conv 64->64 @184x320, W~N(0,sqrt(2/576)), b~U(-0.1,0.1), "
                "x~N(0,1), seed 0")
        metric = METRIC.replace("config 2 block stack", "config 1 single 3x3 conv")
    else:
        gb, inputs = build_block_stack(0)
        desc = ("config2-block-stack: pixel_unshuffle(2) -> 8 x [1x1 128->256 +LeakyReLU(0.01); dw3x3 256; "
                "1x1 256->128 +residual; 1x1 128->512 -> ReGLU(clip[0,1]) -> 1x1 256->128 +residual] -> "
                "pixel_shuffle(2); input [1,32,184,320] fp16 ~N(0,1); Kaiming-normal weights, seed 0")
        metric = METRIC
    graph, weights = gb.finish()
    return graph, weights, inputs, desc, metric, []


def measured_peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        d = json.loads(path.read_text())
        return d.get("hbm_gbs"), d.get("bf16_tflops"), "measured"
    return 6650.0, 1590.0, "fallback"


def ncu_traffic():
    """Per-launch DRAM traffic of the dominant kernel from the committed ncu summary."""
    path = ROOT / "profiles" / "ncu_traffic.json"
    if path.exists():
        try:
            return json.loads(path.read_text())
        except ValueError:
            return {}
    return {}


class ClockSampler:
    """Samples nvidia-smi clocks and throttle reasons while the timed region runs."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu_index = gpu_index
        self.proc = None
        self.path = tempfile.mktemp(prefix="clocks_", suffix=".csv")

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                                          "-lms", "200", "-i", str(self.gpu_index)],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        rows = []
        try:
            for line in open(self.path):
                f = [x.strip() for x in line.split(",")]
                if len(f) >= 9 and f[1].replace(".", "").isdigit():
                    rows.append(f)
        except OSError:
            pass
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"], "samples": 0}
        sm = [float(r[1]) for r in rows]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": float(rows[0][2]), "reasons": reasons,
                "samples": len(rows), "power_w_max": max(float(r[3]) for r in rows if r[3].replace(".", "").isdigit())}


def pin_host_cores(local_rank, local_world):
    """Gives each rank of a multi-GPU run its own contiguous share of the host
    cores this process may use, so the ranks' host threads (slot copies,
    submits, waits) neither migrate nor contend for the same cores.  Returns
    the cores kept, or None when there are fewer cores than ranks."""
    try:
        cores = sorted(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        return None
    share = len(cores) // max(1, local_world)
    if share < 1:
        return None
    mine = cores[local_rank * share:(local_rank + 1) * share]
    os.sched_setaffinity(0, mine)
    return mine


def replica_throughput(local_ms, steps, world, device="cpu"):
    """Whole-job frames/s of `world` independent replicas that each ran `steps`
    frames in `local_ms` device milliseconds: the slowest rank bounds the job
    (max over ranks; needs an initialised process group when world > 1)."""
    import torch
    t = torch.tensor([float(local_ms)], dtype=torch.float64, device=device)
    if world > 1:
        import torch.distributed as dist
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    return world * steps / (ms_max / 1000.0), ms_max


# ------------------------------------------------ entropy-coder inputs
# One frame of the reference's encode prelude (core/src/entropy.cpp:389-394):
# extract_scales(z_raw) and integer_values of y_raw_1, y_raw_0 and z_raw, at
# the 1920x1088 plane sizes (latent 128 -> two 64 x 68 x 120 halves, z 128 x
# 9 x 15; scale table 128 levels).
ENTROPY_CFG = dict(model_width=1920, model_height=1088, latent_channels=128)
ENTROPY_DESC = ("entropy-coder inputs of one 1920x1088 frame: extract_scales(z_raw [1,128,9,15]) -> 2 x int32 "
                "[64,68,120], integer_values(y_raw_1, y_raw_0 [1,64,68,120], z_raw) -> int32; integer-valued FP16 "
                "latents rint(N(0,1)*3), z rint(N(0,1)*4), seed 0")
ENTROPY_METRIC = "entropy-coder input frames/s @1920x1088 (scale extraction + symbol conversion)"


def entropy_inputs():
    rng = np.random.default_rng(0)
    z = np.rint(rng.standard_normal((1, 128, 9, 15)) * 4).astype(np.float16)
    y1 = np.rint(rng.standard_normal((1, 64, 68, 120)) * 3).astype(np.float16)
    y0 = np.rint(rng.standard_normal((1, 64, 68, 120)) * 3).astype(np.float16)
    return z, y1, y0


def entropy_cpu_frames_per_s(frames):
    """The CPU prelude: the reference's compiled extract_scales (oracle/_ref)
    and the numpy restatement of integer_values (entropy.cpp needs the absent
    rANS coder).  One thread."""
    from oracle import scales_oracle  # CPU baseline only
    from oracle.ref_backend import ref_extract_scales
    z, y1, y0 = entropy_inputs()
    times = []
    for _ in range(frames + 1):
        t0 = time.perf_counter()
        ref_extract_scales(z, **ENTROPY_CFG)
        for v in (y1, y0, z):
            scales_oracle.integer_values(v)
        times.append(time.perf_counter() - t0)
    times = times[1:]
    return frames / sum(times), times


def run_entropy_arm(args, rank, world, local_rank):
    import torch
    from mlvc_b200 import Backend

    torch.cuda.set_device(local_rank)
    dev = torch.device(f"cuda:{local_rank}")
    z, y1, y0 = entropy_inputs()
    be = Backend(local_rank)
    stream = torch.cuda.ExternalStream(be.stream)
    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=dev)
    zt, y1t, y0t = (torch.from_numpy(a).to(dev) for a in (z, y1, y0))
    s0 = torch.empty((64, 68, 120), dtype=torch.int32, device=dev)
    s1 = torch.empty_like(s0)
    sy1, sy0 = (torch.empty(a.shape, dtype=torch.int32, device=dev) for a in (y1, y0))
    sz = torch.empty(z.shape, dtype=torch.int32, device=dev)
    flag = torch.zeros(1, dtype=torch.int32, device=dev)
    torch.cuda.synchronize()

    def scales():
        be.extract_scales_device(zt.data_ptr(), 128, 1920, 1088, 128, s0.data_ptr(), s1.data_ptr())

    def symbols(src, dst):
        be.integer_values_device(src.data_ptr(), src.numel(), dst.data_ptr(), flag.data_ptr())

    def frame():
        scales()
        symbols(y1t, sy1)
        symbols(y0t, sy0)
        symbols(zt, sz)

    def flush_l2():
        with torch.cuda.stream(stream):
            flush.fill_(1)

    for _ in range(args.warmup):
        flush_l2()
        frame()
    torch.cuda.synchronize()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    gpu_index = vis.split(",")[local_rank] if vis else local_rank
    with ClockSampler(gpu_index) as clocks:
        for i in range(args.steps):
            flush_l2()  # cold L2 at the start of every frame (untimed)
            starts[i].record(stream)
            frame()
            ends[i].record(stream)
        torch.cuda.synchronize()
    ms = sum(a.elapsed_time(b) for a, b in zip(starts, ends))
    value, ms_max = replica_throughput(ms, args.steps, world, f"cuda:{local_rank}")
    if int(flag.item()) != 0:
        raise RuntimeError("symbol conversion reported an out-of-range value")
    want0, want1 = be.extract_scales(z, **ENTROPY_CFG)
    if not (np.array_equal(s0.cpu().numpy(), want0) and np.array_equal(s1.cpu().numpy(), want1)
            and np.array_equal(sy1.cpu().numpy(), be.integer_values(y1))):
        raise RuntimeError("device-pointer results differ from the host-buffer calls")

    # per-kernel cold-L2 launch times (events around each launch)
    def timed(fn, n=20):
        total = 0.0
        for _ in range(n):
            flush_l2()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            fn()
            b.record(stream)
            torch.cuda.synchronize()
            total += a.elapsed_time(b)
        return total / n
    t_scales = timed(scales)
    t_sym = timed(lambda: symbols(y1t, sy1))
    n_out = s0.numel()
    kernels = {
        "mlvc_extract_scales": {"launches": 1, "us_cold_l2": 1e3 * t_scales,
                                "algorithmic_bytes": z.nbytes + 8 * n_out},
        "mlvc_integer_values_f16": {"launches": 3, "us_cold_l2_y_half": 1e3 * t_sym,
                                    "algorithmic_bytes": 6 * (y1.size + y0.size + z.size)},
    }
    hbm, _, peak_kind = measured_peaks()
    sym_bytes = 6.0 * y1.size
    achieved = sym_bytes / (t_sym / 1e3) / 1e9
    roof = {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
            "peak_kind": peak_kind, "kernel": "mlvc_integer_values_f16",
            "algorithmic_bytes_per_launch": sym_bytes, "avg_launch_us_cold_l2": 1e3 * t_sym,
            "traffic": ncu_traffic().get(args.workload, {}).get("mlvc_integer_values_f16")}

    # end to end through the public host-buffer calls (the reference's call shape)
    def host_frame():
        be.extract_scales(z, **ENTROPY_CFG)
        for v in (y1, y0, z):
            be.integer_values(v)
    for _ in range(args.warmup):
        host_frame()
    e_st, e_en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e_st.record(stream)
    for _ in range(args.steps):
        host_frame()
    e_en.record(stream)
    torch.cuda.synchronize()
    e2e_value, _ = replica_throughput(e_st.elapsed_time(e_en), args.steps, world, f"cuda:{local_rank}")
    h2d = 2 * z.nbytes + y1.nbytes + y0.nbytes
    d2h = 8 * n_out + 4 * (y1.size + y0.size + z.size) + 3 * 4

    line = None
    if rank == 0:
        line = {
            "metric": ENTROPY_METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f16->int32", "data": "synthetic",
            "config": {"workload": ENTROPY_DESC, "global_batch": world,
                       "parallelism": f"replicas x{world} (no collective)",
                       "l2": "flushed before every timed frame (256 MiB fill, untimed)"},
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d * world,
                    "d2h_bytes_per_step": d2h * world,
                    "path": "mlvc_b200_extract_scales + 3 x mlvc_b200_integer_values on pageable host buffers "
                            "(each call copies in, launches, copies out and waits)"},
            "gpu_launches": 4 * args.steps,
            "roofline": roof,
            "kernels": kernels,
            "clocks": clocks.summary(),
        }
        if world == 1 and not args.no_cpu_baseline:
            fps, times = entropy_cpu_frames_per_s(1000)  # ~10 s of CPU work
            line["cpu_baseline"] = {"value": fps, "unit": UNIT, "cores": 1, "kind": "port",
                                    "sample": f"{len(times)} frames: reference extract_scales compiled from "
                                              "core/src/scales.cpp (oracle/_ref) + numpy restatement of "
                                              f"integer_values, {sum(times):.2f} s"}
    be.close()
    return line


# ------------------------------------------------------------------ CPU
def reference_backend_frames_per_s(graph, weights, inputs, frames, warmup, threads):
    """Times the reference CPU backend (oracle/_ref) running the same graph."""
    from oracle.ref_backend import RefCpuBackend  # reference arm / CPU baseline only
    with tempfile.TemporaryDirectory() as d:
        part = Path(d) / "aot" / "stack"
        part.mkdir(parents=True)
        (part / "graph.pb").write_bytes(graph)
        (part / "weights.bin").write_bytes(weights)
        ref = RefCpuBackend(d, "stack", threads)
        for _ in range(warmup):
            ref.run(inputs)
        times = []
        for _ in range(frames):
            t0 = time.perf_counter()
            ref.run(inputs)
            times.append(time.perf_counter() - t0)
        ref.close()
    return frames / sum(times), times


def run_reference_arm(args, rank, world):
    if args.workload == "entropy_1080p":
        if rank != 0:
            return 0
        fps, times = entropy_cpu_frames_per_s(args.steps)
        line = {
            "impl": "reference", "metric": ENTROPY_METRIC, "value": fps, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * sum(times) / len(times),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16->int32",
            "data": "synthetic", "config": {"workload": ENTROPY_DESC, "global_batch": 1, "parallelism": "cpu"},
            "cpu_baseline": {"value": fps, "unit": UNIT, "cores": 1, "kind": "port",
                             "sample": f"{args.steps} frames: reference extract_scales (oracle/_ref) + numpy "
                                       "restatement of integer_values"},
            "e2e": {"value": fps, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        }
        print(json.dumps(line), flush=True)
        return 0
    if args.workload == STREAMS_WORKLOAD:
        if rank != 0:
            return 0
        graph, weights, inputs = streams_graph()
        threads = os.cpu_count() or 1
        fps, times = reference_stream_frames_per_s(graph, weights, inputs, args.steps, args.warmup, threads)
        line = {
            "impl": "reference", "metric": STREAMS_METRIC, "value": fps, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * sum(times) / len(times),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "fp16", "data": "synthetic",
            "config": {"workload": STREAMS_DESC, "global_batch": STREAMS, "parallelism": "cpu-threads",
                       "step": "one frame of one stream (a bounded sample: the CPU decodes the 8 streams' frames one "
                               "after another, so frames/s is the per-frame rate)"},
            "cpu_baseline": {"value": fps, "unit": UNIT, "cores": threads, "kind": "reference",
                             "sample": f"{args.steps} frames (streams in turn, recurrent state carried) on the "
                                       "reference backends/cpu (AVX2, fusion on)"},
            "e2e": {"value": fps, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        }
        print(json.dumps(line), flush=True)
        return 0
    graph, weights, inputs, desc, metric, _ = workload(args.workload)
    if rank != 0:
        return 0
    threads = os.cpu_count() or 1
    fps, times = reference_backend_frames_per_s(graph, weights, inputs, args.steps, args.warmup, threads)
    line = {
        "impl": "reference", "metric": metric, "value": fps, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1000.0 * sum(times) / len(times), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp16", "data": "synthetic",
        "config": {"workload": desc, "global_batch": 1, "parallelism": "cpu-threads"},
        "cpu_baseline": {"value": fps, "unit": UNIT, "cores": threads, "kind": "reference",
                         "sample": f"{args.steps} frames of the workload, reference backends/cpu (AVX2, fusion on)"},
        "e2e": {"value": fps, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0



# ------------------------------------------------------------ roofline
def kernel_roofline(be, workload_name, frame_ms=None):
    """Per-kernel device times of one backend's schedule and the roofline line
    of the kernel with the largest in-frame time.

    In a replayed frame consecutive kernels overlap (programmatic dependent
    launch: a kernel's prologue runs while its predecessor drains), so CUDA
    events recorded between steps could only time them by removing that
    overlap.  Two measurements are therefore taken:
      * in-frame span (the roofline's time): the frame replayed with every
        tensor-core kernel writing %globaltimer stamps; span = last CTA exit -
        first CTA passing griddepcontrol.wait, mean over 10 replays, each after
        a 256 MiB L2 flush (Backend.trace_spans);
      * isolated launches timed with CUDA events on the backend's stream, back
        to back (warm) and after a 256 MiB flush (cold); these include each
        launch's own start-up, which the frame hides.
    Kernels without stamps (the bandwidth kernels) enter the in-frame total
    with their warm isolated time.  Algorithmic work per launch is the
    planner's count: one HBM read of each distinct input and weight tensor,
    one write of each output, FP16 = 2 B; FLOPs = 2 * MACs.  Both roofs are
    reported; `bound` is the one the kernel's intensity puts it under (the
    measured ridge = bf16 peak / copy bandwidth)."""
    steps = be.steps()
    warm = be.time_steps(20, 0)
    cold = be.time_steps(10, FLUSH_BYTES)
    spans = be.trace_spans(10, FLUSH_BYTES)
    per_kernel = {}
    for st, w_ms, c_ms, s_ms in zip(steps, warm, cold, spans):
        k = per_kernel.setdefault(st["kernel"], {"launches": 0, "warm_ms": 0.0, "cold_ms": 0.0, "frame_ms": 0.0,
                                                 "spanned": False, "bytes": 0.0, "flops": 0.0})
        k["launches"] += 1
        k["warm_ms"] += w_ms
        k["cold_ms"] += c_ms
        k["frame_ms"] += s_ms if s_ms > 0 else w_ms
        k["spanned"] = k["spanned"] or s_ms > 0
        k["bytes"] += st["bytes"]
        k["flops"] += st["flops"]
    total_frame = sum(v["frame_ms"] for v in per_kernel.values())
    dom_name, dom = max(per_kernel.items(), key=lambda kv: kv[1]["frame_ms"])
    hbm, tflops_peak, peak_kind = measured_peaks()
    ridge = tflops_peak * 1e12 / (hbm * 1e9)
    intensity = dom["flops"] / max(dom["bytes"], 1.0)
    tensor_achieved = dom["flops"] / (dom["frame_ms"] / 1e3) / 1e12
    hbm_achieved = dom["bytes"] / (dom["frame_ms"] / 1e3) / 1e9
    if intensity >= ridge:
        roof = {"bound": "tensor", "achieved": tensor_achieved, "peak": tflops_peak, "unit": "TFLOP/s"}
    else:
        roof = {"bound": "hbm", "achieved": hbm_achieved, "peak": hbm, "unit": "GB/s"}
    roof["frac"] = roof["achieved"] / roof["peak"]
    roof["peak_kind"] = peak_kind
    roof["kernel"] = dom_name
    roof["time_source"] = ("in-frame span from the kernel's %globaltimer stamps (frame replayed after an L2 flush)"
                           if dom["spanned"] else "isolated warm launches, CUDA events")
    roof["intensity_flop_per_byte"] = intensity
    roof["ridge_flop_per_byte"] = ridge
    roof["tensor_roof"] = {"achieved_tflops": tensor_achieved, "peak_tflops": tflops_peak,
                           "frac": tensor_achieved / tflops_peak}
    roof["hbm_roof"] = {"achieved_gbs": hbm_achieved, "peak_gbs": hbm, "frac": hbm_achieved / hbm}
    roof["launches_per_step"] = dom["launches"]
    roof["algorithmic_bytes_per_launch"] = dom["bytes"] / dom["launches"]
    roof["algorithmic_flops_per_launch"] = dom["flops"] / dom["launches"]
    roof["avg_launch_us_in_frame"] = 1e3 * dom["frame_ms"] / dom["launches"]
    roof["avg_launch_us_isolated_events"] = 1e3 * dom["warm_ms"] / dom["launches"]
    roof["avg_launch_us_isolated_cold_l2_events"] = 1e3 * dom["cold_ms"] / dom["launches"]
    roof["share_in_frame"] = dom["frame_ms"] / total_frame
    roof["sum_in_frame_us"] = 1e3 * total_frame
    if frame_ms is not None:
        roof["frame_us_timed_region"] = 1e3 * frame_ms  # device time per frame of the timed region
    roof["traffic"] = ncu_traffic().get(workload_name, {}).get(dom_name)
    kernels = {k: {"launches": v["launches"], "share_in_frame": v["frame_ms"] / total_frame,
                   "us_in_frame": 1e3 * v["frame_ms"], "in_frame_from_stamps": v["spanned"],
                   "us_isolated_events": 1e3 * v["warm_ms"], "us_isolated_cold_l2_events": 1e3 * v["cold_ms"],
                   "tflops_in_frame": v["flops"] / (v["frame_ms"] / 1e3) / 1e12 if v["flops"] else 0.0,
                   "gbs_in_frame": v["bytes"] / (v["frame_ms"] / 1e3) / 1e9}
               for k, v in per_kernel.items()}
    return roof, kernels


# ------------------------------------------- config 5: 8 streams at 1080p
STREAMS = 8
GOP = 64
# frames of different streams in flight on one GPU at a time (--concurrency)
STREAM_LANES = 2
STREAMS_WORKLOAD = "mlvc_dec_1080p_8s"
STREAMS_Q = 21
STREAMS_DESC = ("BASELINE config 5 on the MLVC-shaped decoder stand-in @1920x1088 (the upstream MLVC architecture is "
                "absent): 8 independent streams of 64-frame GOPs, each with its own recurrent feature state (bound "
                "ref_feature <- feature on the device, reset at every I-frame), split 8/N per GPU with one backend "
                "instance per stream; one step = one frame of every stream on that GPU; decoder I/O z_raw 1/128, "
                "y_raw_0/1 1/16, q_index 21 -> x_hat (8-bit YUV420 1920x1080 through the codec output conversion "
                "on the e2e path); 2+2+2 depth-conv blocks at 256 ch, x8 pixel-shuffle reconstruction; "
                "Kaiming-normal weights, seed 0; integer-valued latents seeded per stream and frame")
STREAMS_METRIC = ("1080p decode frames/s, 8 independent streams (MLVC-shaped decoder stand-in for the 1080p MLVC "
                  "decode of BASELINE config 5)")


def streams_graph():
    gb, inputs = build_mlvc_decoder_standin(0, 1920, 1088, q_index=STREAMS_Q)
    graph, weights = gb.finish()
    return graph, weights, inputs


def stream_latents(inputs, stream, frame):
    """Seeded integer-valued latents (z_raw, y_raw_0, y_raw_1) of one frame of one stream."""
    rng = np.random.default_rng((stream << 20) + frame)
    return [np.rint(rng.standard_normal(inputs[k].shape) * scale).astype(np.float16)
            for k, scale in zip(range(3), (4, 3, 3))]


def reference_stream_frames_per_s(graph, weights, inputs, frames, warmup, threads):
    """The reference CPU backend decoding frames of the streams in turn, its
    recurrent feature state carried (ref_feature <- feature) and reset at
    every GOP start."""
    from oracle.ref_backend import RefCpuBackend  # reference arm / CPU baseline only
    q = np.array([STREAMS_Q], np.int32)
    with tempfile.TemporaryDirectory() as d:
        part = Path(d) / "aot" / "MLVCDecoder"
        part.mkdir(parents=True)
        (part / "graph.pb").write_bytes(graph)
        (part / "weights.bin").write_bytes(weights)
        ref = RefCpuBackend(d, "MLVCDecoder", threads, state_bindings=[(3, 1, list(inputs[3].shape))])
        times = []
        for f in range(warmup + frames):
            lat = stream_latents(inputs, f % STREAMS, f // STREAMS)
            if f % (STREAMS * GOP) == 0:
                ref.reset_state()
            t0 = time.perf_counter()
            ref.run(lat + [q])
            if f >= warmup:
                times.append(time.perf_counter() - t0)
        ref.close()
    return frames / sum(times), times


def run_streams_arm(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    from mlvc_b200 import Backend

    if STREAMS % world:
        raise SystemExit(f"--gpus must divide the {STREAMS} streams")
    torch.cuda.set_device(local_rank)
    dev = torch.device(f"cuda:{local_rank}")
    n_local = STREAMS // world
    stream_ids = list(range(rank * n_local, (rank + 1) * n_local))
    graph, weights, inputs = streams_graph()
    q = np.array([STREAMS_Q], np.int32)
    backends = []
    for sid in stream_ids:
        be = Backend(local_rank)
        be.load_memory(graph, weights, [(3, 1)])
        be.reset_state()
        outs = be.run(stream_latents(inputs, sid, 0) + [q])  # inputs now resident on the device
        if not all(np.isfinite(o.astype(np.float32)).all() for o in outs):
            raise RuntimeError("non-finite output")
        be.reset_state()
        backends.append(be)
    cstreams = [torch.cuda.ExternalStream(be.stream, device=dev) for be in backends]
    s0 = cstreams[0]
    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=dev)

    # The local streams run in `lanes` lanes: stream j starts after the L2
    # flush (j < lanes) or after stream j - lanes finished its frame, so at
    # most `lanes` frames are in flight on the GPU.  Fewer concurrent frames
    # keep more of each one's producer -> consumer tensors in the 126 MB L2.
    lanes = max(1, min(args.concurrency, n_local))

    def chain(j, cs, after_flush, done):
        if j < lanes:
            if cs is not s0:
                cs.wait_event(after_flush)
        else:
            cs.wait_event(done[j - lanes])

    def step(i):
        """One frame of every local stream, each on its own CUDA stream, in
        lanes after an L2 flush on stream 0, joined back into stream 0."""
        with torch.cuda.stream(s0):
            flush.fill_(1)
        start = torch.cuda.Event(enable_timing=True)
        start.record(s0)
        done = []
        for j, (cs, be) in enumerate(zip(cstreams, backends)):
            chain(j, cs, start, done)
            be.enqueue()
            ev = torch.cuda.Event()
            ev.record(cs)
            done.append(ev)
        for j in range(max(1, n_local - lanes), n_local):
            s0.wait_event(done[j])
        end = torch.cuda.Event(enable_timing=True)
        end.record(s0)
        return start, end

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    gpu_index = vis.split(",")[local_rank] if vis else local_rank
    with ClockSampler(gpu_index) as clocks:
        marks = [step(i) for i in range(args.steps)]
        torch.cuda.synchronize()
    ms = sum(a.elapsed_time(b) for a, b in marks)
    frames_local = args.steps * n_local
    t = torch.tensor([ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    value = STREAMS * args.steps / (ms_max / 1e3)

    # ---- end to end through the public slot API: per stream two slots,
    # latents in from pinned host memory, submit(slot, shifted_q), the decoded
    # frame out as 8-bit YUV420 through the codec output conversion
    width, height = 1920, 1080
    for be in backends:
        be.reset_state()
        be.configure_codec_io(width, height, 1920, 1088, 1.0, slots=2, output_index=0)
    lat_cache = {}

    def frame_inputs(sid, f):
        key = (sid, f % 4)  # four distinct latent sets per stream, cycled
        if key not in lat_cache:
            lat_cache[key] = stream_latents(inputs, sid, f % 4)
        return lat_cache[key]

    for sid in stream_ids:  # every latent set the run cycles through, made before any timing
        for f in range(4):
            frame_inputs(sid, f)

    def pipeline(first, n):
        for i in range(first, first + n):
            slot = i % 2
            with torch.cuda.stream(s0):
                flush.fill_(1)  # cold L2 before every step, inside the timed region
            fl = torch.cuda.Event()
            fl.record(s0)
            done = []
            for j, (sid, cs, be) in enumerate(zip(stream_ids, cstreams, backends)):
                if i >= 2:
                    be.wait_slot(slot)
                if i % GOP == 0 and i > 0:
                    be.reset_state()  # I-frame: a new GOP starts from a zeroed feature
                for k, a in enumerate(frame_inputs(sid, i)):
                    be.slot_input(slot, k)[...] = a
                chain(j, cs, fl, done)  # the same lanes as the device-timed steps
                be.submit(slot, shifted_q=STREAMS_Q)
                ev = torch.cuda.Event()
                ev.record(cs)
                done.append(ev)
        for be in backends:
            for slot in range(min(first + n, 2)):
                be.wait_slot(slot)

    pipeline(0, max(2, args.warmup))
    for be in backends:
        be.reset_state()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    # whole GOPs per stream (at least K frames): the window the codec decodes
    # between two I-frames, long enough that host jitter of one rank does not
    # set the max over ranks
    e2e_frames = GOP * max(1, -(-args.steps // GOP))
    e_st, e_en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_st.record(s0)
    pipeline(0, e2e_frames)
    e_en.record(s0)
    torch.cuda.synchronize()
    e2e_local = e_st.elapsed_time(e_en)
    t = torch.tensor([e2e_local], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_value = STREAMS * e2e_frames / (float(t.item()) / 1e3)
    # per-rank device times (value path, e2e path) for the line's diagnostics
    per_rank = torch.tensor([[ms, e2e_local]], dtype=torch.float64, device=dev)
    if world > 1:
        gathered = [torch.zeros_like(per_rank) for _ in range(world)]
        dist.all_gather(gathered, per_rank)
        per_rank = torch.cat(gathered)
    per_rank_ms = per_rank.cpu().tolist()
    try:
        host_cores = len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        host_cores = os.cpu_count()
    h2d = sum(a.nbytes for a in inputs[:3]) + 4
    d2h = width * height * 3 // 2
    # the slot path still decodes after the timed run (first frame of a fresh GOP, stream 0)
    be = backends[0]
    be.reset_state()
    for k, a in enumerate(frame_inputs(stream_ids[0], 0)):
        be.slot_input(0, k)[...] = a
    be.submit(0, shifted_q=STREAMS_Q)
    be.wait_slot(0)
    got = np.concatenate([pl.reshape(-1) for pl in be.slot_output_yuv(0)])
    if got.size != d2h or float(got.std()) == 0.0:
        raise RuntimeError("slot path produced no decoded frame")

    roof, kernels = kernel_roofline(backends[0], args.workload, ms_max / args.steps / n_local)
    line = None
    if rank == 0:
        line = {
            "metric": STREAMS_METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "fp16", "data": "synthetic",
            "config": {"workload": STREAMS_DESC, "global_batch": STREAMS, "streams_per_gpu": n_local, "concurrent_streams_per_gpu": lanes,
                       "parallelism": f"{STREAMS} independent streams over {world} GPU(s), {n_local} per GPU "
                                      "(no collective)",
                       "step": f"one frame of each of the {n_local} streams on a GPU ({STREAMS} frames per step "
                               "job-wide)",
                       "l2": "flushed before every timed step (256 MiB fill; untimed on the device path, inside "
                             "the timed region on the e2e path)"},
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d * STREAMS,
                    "d2h_bytes_per_step": d2h * STREAMS,
                    "path": ("mlvc_b200 slot API per stream, 2 slots: latents (z_raw, y_raw_0, y_raw_1) from pinned "
                             "host memory, submit(slot, shifted_q), schedule, x_hat -> 8-bit YUV420 1920x1080 on the "
                             "GPU, pinned D2H; GOP reset every 64 frames; timed on the device over whole 64-frame GOPs "
                             "(at least K frames) per stream"),
                    "frames_per_stream": e2e_frames,
                    "per_rank_ms": [r[1] for r in per_rank_ms],
                    "host_cores_per_rank": host_cores},
            "per_rank_ms": [r[0] for r in per_rank_ms],
            "gpu_launches": sum(b.kernel_launches for b in backends) * args.steps,
            "roofline": roof,
            "kernels": kernels,
            "clocks": clocks.summary(),
        }
        if world == 1 and not args.no_cpu_baseline:
            threads = os.cpu_count() or 1
            try:
                fps, times = reference_stream_frames_per_s(graph, weights, inputs, args.cpu_frames, 1, threads)
                line["cpu_baseline"] = {"value": fps, "unit": UNIT, "cores": threads, "kind": "reference",
                                        "sample": f"{args.cpu_frames} frames (streams in turn, state carried) on "
                                                  f"the reference backends/cpu (AVX2, fusion on), {sum(times):.1f} s"}
            except Exception as e:  # reported, never silently replaced
                line["cpu_baseline"] = {"value": None, "unit": UNIT, "cores": threads, "kind": "reference",
                                        "sample": f"unavailable: {e}"}
    for be in backends:
        be.close()
    return line


# ------------------------------------------------------------------ GPU
def run_b200_arm(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    from mlvc_b200 import Backend

    torch.cuda.set_device(local_rank)
    graph, weights, all_inputs, desc, metric, bindings = workload(args.workload)
    be = Backend(local_rank)
    be.load_memory(graph, weights, bindings)
    if bindings:  # state-bound inputs live on the device; the CPU baseline gets all inputs
        be.reset_state()
    bound = {i for i, _ in bindings}
    inputs = [a for k, a in enumerate(all_inputs) if k not in bound]
    outs = be.run(inputs)  # inputs now resident on the device
    if not all(np.isfinite(o.astype(np.float32)).all() for o in outs):
        raise RuntimeError("non-finite output")
    stream = torch.cuda.ExternalStream(be.stream)
    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=f"cuda:{local_rank}")

    def flush_l2():
        with torch.cuda.stream(stream):
            flush.fill_(1)

    for _ in range(args.warmup):
        flush_l2()
        be.enqueue()
    be.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    be.synchronize()

    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    gpu_index = vis.split(",")[local_rank] if vis else local_rank
    with ClockSampler(gpu_index) as clocks:
        for i in range(args.steps):
            flush_l2()  # cold L2 at the start of every frame (untimed)
            starts[i].record(stream)
            be.enqueue()
            ends[i].record(stream)
        be.synchronize()
    torch.cuda.synchronize()
    ms = sum(s.elapsed_time(e) for s, e in zip(starts, ends))
    value, ms_max = replica_throughput(ms, args.steps, world, f"cuda:{local_rank}")

    # ---- end to end through the public slot API: H2D + replay + D2H per frame
    be.configure_slots(2)
    in_bytes = sum(int(np.prod(s)) * np.dtype(d).itemsize for _, d, s in be.inputs)
    out_bytes = sum(int(np.prod(s)) * np.dtype(d).itemsize for _, d, s in be.outputs)
    for slot in range(2):
        for k, arr in enumerate(inputs):
            be.slot_input(slot, k)[...] = arr
    def pipeline(n):
        # frame i: wait for slot i % 2 to come back, flush L2 (on the compute
        # stream, ahead of the frame's schedule), submit; the slot pipeline
        # overlaps frame i's schedule with frame i-1's device->host copy and
        # frame i+1's host->device copy
        for i in range(n):
            slot = i % 2
            if i >= 2:
                be.wait_slot(slot)
            flush_l2()
            be.submit(slot)
        for slot in range(min(n, 2)):
            be.wait_slot(slot)

    pipeline(max(2, args.warmup))
    e_st = torch.cuda.Event(enable_timing=True)
    e_en = torch.cuda.Event(enable_timing=True)
    be.synchronize()
    if world > 1:
        dist.barrier()
    # The start event is recorded while the device is idle and the end event
    # after the last slot came back, so the interval covers every copy.
    e_st.record(stream)
    pipeline(args.steps)
    e_en.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e_st.elapsed_time(e_en)
    e2e_value, _ = replica_throughput(e2e_ms, args.steps, world, f"cuda:{local_rank}")
    # output still correct after the slot loop (with recurrent state: one frame
    # each way from a reset state)
    if bindings:
        be.reset_state()
        want = be.run(inputs)[0]
        be.reset_state()
        be.submit(0)
        be.wait_slot(0)
        first = be.slot_output(0, 0)
    else:
        want = outs[0]
        first = be.slot_output((args.steps - 1) % 2, 0)
    if not np.array_equal(first.view(np.uint16), want.view(np.uint16)):
        raise RuntimeError("slot path output differs from run()")

    roof, kernels = kernel_roofline(be, args.workload, ms_max / args.steps)

    line = None
    if rank == 0:
        line = {
            "metric": metric, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "fp16", "data": "synthetic",
            "config": {"workload": desc, "global_batch": world, "parallelism": f"replicas x{world} (no collective)",
                       "l2": "flushed before every timed frame (256 MiB fill, untimed)"},
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": in_bytes * world,
                    "d2h_bytes_per_step": out_bytes * world,
                    "path": ("mlvc_b200 slot API, 2 slots: pinned H2D, schedule, pinned D2H per frame on three "
                             "streams; timed over the whole run, including a 256 MiB L2 flush before every frame")},
            "gpu_launches": be.kernel_launches * args.steps,
            "roofline": roof,
            "kernels": kernels,
            "clocks": clocks.summary(),
        }
        if world == 1 and not args.no_cpu_baseline:
            threads = os.cpu_count() or 1
            try:
                fps, times = reference_backend_frames_per_s(graph, weights, all_inputs, args.cpu_frames, 1, threads)
                line["cpu_baseline"] = {"value": fps, "unit": UNIT, "cores": threads, "kind": "reference",
                                        "sample": f"{args.cpu_frames} frames of the same workload on the reference "
                                                  f"backends/cpu (AVX2, fusion on), {sum(times):.1f} s"}
            except Exception as e:  # reported, never silently replaced
                line["cpu_baseline"] = {"value": None, "unit": UNIT, "cores": threads, "kind": "reference",
                                        "sample": f"unavailable: {e}"}
    be.close()
    return line


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--workload", choices=["block_stack", "conv3x3", "op_dw3x3", "op_conv1x1", "op_ffn", "op_dwconv",
                                                   "op_mbconv", "mlvc_dec_1080p", "mlvc_dec_640", "mlvcs_dec_640",
                                                   "mlvc_enc_1080p", "mlvc_enc_640", "entropy_1080p",
                                                   STREAMS_WORKLOAD],
                    default=STREAMS_WORKLOAD)
    ap.add_argument("--concurrency", type=int, default=STREAM_LANES,
                    help="streams of one GPU decoding at the same time (the others queue behind them)")
    ap.add_argument("--cpu-frames", type=int, default=16)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference_arm(args, rank, world)
    if world > 1:
        import datetime

        pin_host_cores(local_rank, int(os.environ.get("LOCAL_WORLD_SIZE", world)))
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device(f"cuda:{local_rank}"))
    arm = {"entropy_1080p": run_entropy_arm, STREAMS_WORKLOAD: run_streams_arm}.get(args.workload, run_b200_arm)
    line = arm(args, rank, world, local_rank)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()
    if line is not None:
        print(json.dumps(line), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
