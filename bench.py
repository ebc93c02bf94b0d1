#!/usr/bin/env python3
"""Benchmark of the B200 MiniMax-H3 transformer step: seconds per 768p x 124-frame step (d 5120,
40 heads of 128, SwiGLU 13824, 48 blocks; 32 latent frames x 24 x 42 = 32256 video rows + 512 text + 256 audio rows),
random-init bf16 weights, synthetic inputs, one denoising step at t = 0.7. One JSON line on rank 0.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload dense|sparse|int8|long|long-sparse|c1]
    python -m torch.distributed.run --nproc-per-node N ... bench.py --gpus N        (sequence-parallel, Ulysses)
    python bench.py --impl reference                                                (the CPU restatement arm)

value: device time per step (inputs already in HBM, CUDA events on the library's stream, max over ranks).
e2e:   the same through h3_step with pinned host buffers (host->device copies and the velocities' readback inside).
"""
import argparse
import ctypes
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "mako-video_b200"))
sys.path.insert(0, REPO)

import numpy as np  # noqa: E402

METRIC = "s per 768p x 124f transformer step"
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}

WORKLOADS = {
    # name: (config, layout, sparse ratio, sparse local, int8 mask, description)
    "dense": ("c2", "c2", 0.0, 1, 0, "C2: 768p dense, 48 blocks, S = 33024"),
    "sparse": ("c2", "c2", 0.1, 1, 0, "C3: C2 + block-sparse attention, ratio 0.1, local 1, 528 padded cubes"),
    "int8": ("c2", "c2", 0.0, 1, 15, "C4: C2 with int8 W8A8 qkv, out, fc1, fc2"),
    "long": ("c2", "c5", 0.0, 1, 0, "C5: 15 s clip, 92736 video + 1008 keyframe + 512 text + 640 audio rows, dense"),
    "long-sparse": ("c2", "c5", 0.1, 3, 0, "C5 sparse, ratio 0.1, local 3"),
    "c1": ("c1", "c1", 0.0, 1, 0, "C1: one d=1024 block, 576 rows"),
    "vae": (None, None, 0.0, 1, 0, "MiniMax-H3's video VAE decoder on 768p latents"),
    "h3": ("h3", "h3", 0.0, 1, 0, "MiniMax-H3 itself: d 5376, 56 heads, SwiGLU 14336, 50 blocks, 1344x768x124 frames = 37296 video "
                                  "+ 512 text + 414 audio rows, dense"),
}



_json_out = None


def emit(line):
    out = _json_out if _json_out is not None else sys.stdout
    out.write(json.dumps(line) + "\n")
    out.flush()

def load_traffic(kernel, workload):
    """DRAM bytes per launch of the dominant kernel from the committed ncu summary (null when not captured)."""
    p = os.path.join(REPO, "profiles", "traffic.json")
    try:
        with open(p) as f:
            return json.load(f)[kernel][workload]["bytes_per_launch"]
    except (OSError, KeyError, ValueError):
        return None


def load_peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d, "measured"
    return PEAKS_FALLBACK, "fallback"


# ---------------------------------------------------------------------------------------------- FLOP counts

def step_flops(cfg, S, layout, sparse_ratio=0.0):
    """Algorithmic FLOPs of one step: the block GEMMs (2 M N K each) and attention (4 S^2 inner dense)."""
    d, inner, F, L = cfg["dim"], cfg["heads"] * 128, cfg["ffn"], cfg["blocks"]
    gemm = L * 2 * S * (d * 3 * inner + inner * d + d * 2 * F + F * d)
    attn_launch = attention_flops(cfg, S, layout, sparse_ratio)
    return gemm, L * attn_launch


def attention_flops(cfg, S, layout, sparse_ratio=0.0):
    """One block's attention: 4 S^2 inner dense; sparse: 4 inner (V (k 64 + D) + D S) (selected cubes of 64 rows and
    the D dense rows for every video query; every key for the dense queries)."""
    inner = cfg["heads"] * 128
    if not sparse_ratio:
        return 4 * S * S * inner
    ph, pw = layout["h"] // 2, layout["w"] // 2
    V = layout["frames"] * ph * pw
    D = S - V
    cubes = ((layout["frames"] + 3) // 4) * ((ph + 3) // 4) * ((pw + 3) // 4)
    k = max(1, min(cubes, math.ceil(sparse_ratio * cubes - 1e-6)))
    return 4 * inner * (V * (k * 64 + D) + D * S)


# ------------------------------------------------------------------------------------------------- clocks

class ClockSampler:
    """nvidia-smi samples (every 200 ms) of the SM clock and throttle reasons while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except (FileNotFoundError, OSError):
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        rows = []
        if self.path and os.path.exists(self.path):
            for line in open(self.path):
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
            os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(rows)}


# ----------------------------------------------------------------------------------------------- CPU sample

def _inputs(layout, cfg, seed=0):
    rng = np.random.default_rng(seed)
    text = rng.standard_normal((layout.d["text"], cfg["text_dim"]), dtype=np.float32)
    video = rng.standard_normal((layout.video_rows, 96), dtype=np.float32)
    audio = rng.standard_normal((layout.audio_rows, 32), dtype=np.float32)
    return text, video, audio


def cpu_step_sample(cfg, layout, threads=None, weights=None):
    """The oracle's own step (oracle/h3_oracle.py: step, torch fp32 with bf16-valued weights) with ONE block of the
    configuration's width over ALL of the workload's rows, on `threads` host threads. The probes time the block (from
    the packed input to block 0's output); the rest of the step (text projection and token refiner, time embedding,
    patch projections, final norm and heads) runs once. Returns (extrapolated s per step = rest + blocks x block,
    block s, rest s, description, weights)."""
    import torch
    from oracle import h3_oracle as O

    threads = threads or os.cpu_count() or 1
    torch.set_num_threads(threads)
    one = dict(cfg, blocks=1)
    w = weights if weights is not None else O.make_weights(one, 0)
    text, video, audio = _inputs(layout, cfg)
    marks = {}

    def probe(name, layer, _a):
        marks[name if layer < 0 else f"{name}{layer}"] = time.perf_counter()

    t0 = time.perf_counter()
    O.step(one, w, layout.d, text, video, audio, 0.7, 0.7, probes=probe)
    t1 = time.perf_counter()
    block = marks["block0"] - marks["x0"]
    rest = (t1 - t0) - block
    L = cfg["blocks"]
    desc = (f"oracle step (oracle/h3_oracle.py: step, torch fp32) with one full-width block (d {cfg['dim']}, {cfg['heads']} heads, "
            f"SwiGLU {cfg['ffn']}) over all {layout.rows} rows: the block timed ({block:.1f} s) x{L} blocks + the step's "
            f"other work once ({rest:.1f} s); {threads} host threads")
    return rest + L * block, block, rest, desc, w


# ---------------------------------------------------------------------------------------------------- arms

def run_reference(args, rank, world):
    """The reference's host-side path for the step. The reference's own step is Metal code inside an absent
    submodule, so the CPU arm is the oracle's restatement of it: one full step of the oracle with one full-width
    block over all of the workload's rows per timed sample, the block scaled to the stack's block count. Samples run
    until K are timed or ~2 minutes have passed (at least one), so the run stays within a few minutes."""
    if rank != 0:
        return
    import h3b200 as H
    if args.workload == "vae":
        emit(reference_vae(H))
        return
    cfg_name, lay_name, ratio, local, int8, wdesc = WORKLOADS[args.workload]
    cfg = dict(H.CONFIGS[cfg_name])
    layout = H.Layout.named(lay_name)
    threads = os.cpu_count() or 1
    # warm-up: the same step on an eighth of the frames (threads and allocator spun up; weights generated)
    small = dict(layout.d)
    small["frames"] = max(1, small["frames"] // 8)
    w = None
    for _ in range(min(args.warmup, 1)):
        _, _, _, _, w = cpu_step_sample(cfg, H.Layout(**small), threads, w)
    vals, blocks, rests, desc = [], [], [], ""
    t_start = time.perf_counter()
    while len(vals) < max(1, args.steps) and (not vals or time.perf_counter() - t_start < 120.0):
        v, b, r, desc, w = cpu_step_sample(cfg, layout, threads, w)
        vals.append(v)
        blocks.append(b)
        rests.append(r)
    value = statistics.mean(vals)
    sample_s = statistics.mean(b + r for b, r in zip(blocks, rests))
    note = ""
    if ratio or int8:
        note = " (dense bf16-valued fp32 attention and projections: the CPU restatement has no sparse or int8 fast path)"
    line = {"metric": METRIC, "value": value, "unit": "s", "n_gpus": args.gpus, "steps": len(vals), "warmup": min(args.warmup, 1),
            "steps_requested": args.steps, "warmup_requested": args.warmup,
            "ms_per_step": sample_s * 1e3,
            "ms_per_step_is": "one timed sample: the oracle's step with one full-width block over all rows",
            "extrapolated_from": f"1 full-S block x{cfg['blocks']} + the step's other work once",
            "higher_is_better": False, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded normal inputs, hash-generated ~N(0, 0.02) weights)", "impl": "reference",
            "config": {"workload": wdesc, "rows": layout.rows, "dim": cfg["dim"], "heads": cfg["heads"], "ffn": cfg["ffn"],
                       "blocks": cfg["blocks"]},
            "cpu_baseline": {"value": value, "unit": "s", "cores": threads, "kind": "port", "sample": desc + note,
                             "block_s": statistics.mean(blocks), "rest_s": statistics.mean(rests)},
            "e2e": {"value": value, "unit": "s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    emit(line)


class Runner:
    """One model on this rank's GPU and the workload inputs; measures device time (inputs resident) and the end-to-end
    time through h3_step (host buffers)."""

    def __init__(self, H, torch, dist, model, layout, cfg, rank, world, local_rank):
        self.H, self.torch, self.dist = H, torch, dist
        self.model, self.layout, self.cfg = model, layout, cfg
        self.rank, self.world, self.local_rank = rank, world, local_rank
        self.dev = torch.device("cuda", local_rank)
        self.text, video, audio = _inputs(layout, cfg)
        model.begin(self.text, layout)
        self.dv, self.da = torch.from_numpy(video).to(self.dev), torch.from_numpy(audio).to(self.dev)
        self.ov, self.oa = torch.empty_like(self.dv), torch.empty_like(self.da)
        pin = lambda a: torch.from_numpy(a).pin_memory().numpy()
        self.pv, self.pa = pin(video), pin(audio)
        self.hv = torch.empty(video.shape, dtype=torch.float32).pin_memory().numpy()
        self.ha = torch.empty(audio.shape, dtype=torch.float32).pin_memory().numpy()
        self.ext = torch.cuda.ExternalStream(model.stream, device=self.dev)
        self.t = (0.7, 0.7)

    def step_dev(self):
        L = self.layout
        self.model.step_device(self.dv.data_ptr(), L.video_rows, self.da.data_ptr() if self.da.numel() else None, L.audio_rows,
                               *self.t, self.ov.data_ptr(), self.oa.data_ptr() if self.oa.numel() else None)

    def step_host(self):
        H, pv, pa, hv, ha = self.H, self.pv, self.pa, self.hv, self.ha
        H.check(H.lib().h3_step(self.model.h, pv.ctypes.data, pv.shape[0], pa.ctypes.data if pa.size else None, pa.shape[0], *self.t,
                                hv.ctypes.data, ha.ctypes.data if ha.size else None))

    def barrier(self):
        if self.world > 1:
            self.dist.barrier()

    def maxed(self, vals):
        if self.world == 1:
            return vals
        t = self.torch.tensor(vals, device=self.dev, dtype=self.torch.float64)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return [float(x) for x in t]

    def measure(self, steps, warmup, pairs, clocks_gpu=None):
        torch = self.torch
        for _ in range(warmup):
            self.step_dev()
        self.model.synchronize()
        # value: K steps back to back with the inputs in HBM, CUDA events on the library's stream
        self.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        clk = ClockSampler(clocks_gpu) if clocks_gpu is not None else None
        if clk:
            clk.__enter__()
        with torch.cuda.stream(self.ext):
            e0.record()
            for _ in range(steps):
                self.step_dev()
            e1.record()
        self.model.synchronize()
        torch.cuda.synchronize()
        if clk:
            clk.__exit__()
        self.barrier()
        ms = e0.elapsed_time(e1) / steps
        launches = self.model.last_launches()
        # end to end, interleaved with device-resident steps so that both see the same clocks: each pair is one
        # h3_step (pinned host buffers in and out, wall clock) and one step_device (CUDA events), in alternating order
        # so that neither always follows the other (under the power cap the clock drifts between consecutive steps)
        e2e, dev = [], []

        def host_step():
            self.barrier()
            t0 = time.perf_counter()
            self.step_host()
            e2e.append(time.perf_counter() - t0)

        def device_step():
            self.barrier()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with torch.cuda.stream(self.ext):
                a.record()
                self.step_dev()
                b.record()
            self.model.synchronize()
            dev.append(a.elapsed_time(b) * 1e-3)

        for i in range(pairs):
            for f in ((host_step, device_step) if i % 2 == 0 else (device_step, host_step)):
                f()
        if not np.isfinite(self.hv).all():
            raise RuntimeError("non-finite velocities")
        # per-kernel-class device times (events after each class in every block) through h3_step: the copies too
        self.model.set_timing(True)
        self.step_host()
        classes = self.model.timing_by_class()
        self.model.set_timing(False)
        ms, e2e_s, dev_s = self.maxed([ms, statistics.mean(e2e), statistics.mean(dev)])
        diffs = [(a - b) * 1e3 for a, b in zip(e2e, dev)]
        return {"ms": ms, "e2e_s": e2e_s, "paired_dev_s": dev_s, "launches": launches, "classes": classes,
                "pair_diff_ms": {"mean": statistics.mean(diffs), "stdev": statistics.stdev(diffs) if len(diffs) > 1 else None,
                                 "pairs": len(diffs)},
                "clocks": clk.summary() if clk else None}


def _line_part(m, cfg, layout, ratio, world, peaks, args_workload_key, int8):
    """The metric, e2e, the attention roofline and the HBM-bound kernels' bandwidth of one measured workload."""
    S = layout.rows
    classes = m["classes"]
    attn_ms, attn_n = classes.get("attn", (0.0, 0))
    attn_launch = attention_flops(cfg, S, layout.d, ratio) / world
    achieved = attn_launch / (attn_ms / max(attn_n, 1) * 1e-3) / 1e12 if attn_ms else None
    peak = peaks.get("bf16_tflops_sustained", peaks.get("bf16_tflops"))
    gemm_flops, attn_flops = step_flops(cfg, S, layout.d, ratio)
    gemm_ms = sum(classes.get(c, (0.0, 0))[0] for c in ("qkv", "out", "fc1", "fc2"))
    gemm_tflops = (gemm_flops / world) / (gemm_ms * 1e-3) / 1e12 if gemm_ms else None
    if int8:
        # no int8 GEMM peak is measured on this pool: B200's dense int8 rate is twice its bf16 rate
        gemm_peak, gemm_peak_kind = 2 * peak, "2 x measured bf16 sustained (int8 TOPS)"
    else:
        gemm_peak, gemm_peak_kind = peak, "measured bf16 sustained"
    h2d_ms = classes.get("h2d", (0.0, 0))[0]
    d2h_ms = classes.get("d2h", (0.0, 0))[0]
    vb, ab = layout.video_rows * 96 * 4, layout.audio_rows * 32 * 4
    # HBM-bound kernels: modulated RMS norms (fp32 rows in, bf16 or int8 + row scale out) and the AdaLN GEMV (weights)
    S_l = -(-S // world)
    d, td, L = cfg["dim"], cfg["time_dim"], cfg["blocks"]
    norm_ms, norm_n = classes.get("norm", (0.0, 0))
    norm_bytes = S_l * d * (4 + (1 if int8 else 2)) + (S_l * 4 if int8 else 0)
    norm_gbs = norm_bytes / (norm_ms / norm_n * 1e-3) / 1e9 if norm_ms else None
    ada_ms = classes.get("adaln", (0.0, 0))[0]
    ada_bytes = (-(-L // world) * 18 * d + 2 * d) * td * 2
    ada_gbs = ada_bytes / (ada_ms * 1e-3) / 1e9 if ada_ms else None
    hbm = peaks.get("hbm_gbs")
    return {
        "value": m["ms"] / 1e3, "unit": "s", "ms_per_step": m["ms"],
        "e2e": {"value": m["e2e_s"], "unit": "s", "h2d_bytes_per_step": int(vb + ab), "d2h_bytes_per_step": int(vb + ab),
                "paired_device_s": m["paired_dev_s"], "h2d_ms": h2d_ms, "d2h_ms": d2h_ms,
                "e2e_minus_device_ms": m.get("pair_diff_ms"),
                "note": "each timed h3_step (pinned host buffers, wall clock) is paired with a device-resident step "
                        "(CUDA events), in alternating order, so both see the same clocks; h2d_ms / d2h_ms are the copy "
                        "stages' CUDA-event times inside h3_step (d2h includes the gather of the video rows back to the "
                        "layout's order); e2e_minus_device_ms is the per-pair difference, whose spread (the step's clock "
                        "drift under the power cap) exceeds the copies' ~0.6 ms"},
        "roofline": {"bound": "tensor", "kernel": "attention (attn3_kernel, tcgen05)" if ratio else "attention (attn2_kernel, tcgen05)",
                     "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": (achieved / peak) if achieved else None,
                     "traffic": load_traffic("attention", args_workload_key) if world == 1 else None,
                     "peak_kind": "measured bf16 sustained (MEASURED_PEAKS.json)",
                     "launch_flops": attn_launch, "launch_ms": attn_ms / max(attn_n, 1) if attn_n else None,
                     "gemm_tflops": gemm_tflops, "gemm_frac": gemm_tflops / (gemm_peak) if gemm_tflops else None,
                     "gemm_peak": gemm_peak, "gemm_peak_kind": gemm_peak_kind},
        "hbm_kernels": {
            "rms_mod_kernel": {"achieved_gbs": norm_gbs, "frac": norm_gbs / hbm if norm_gbs and hbm else None,
                               "bytes_per_launch": norm_bytes, "launch_ms": norm_ms / norm_n if norm_n else None},
            "adaln_kernel": {"achieved_gbs": ada_gbs, "frac": ada_gbs / hbm if ada_gbs and hbm else None, "bytes_per_step": ada_bytes,
                             "ms": ada_ms},
            "peak_gbs": hbm, "peak_kind": "measured copy bandwidth (MEASURED_PEAKS.json)"},
        "step_tflops": (gemm_flops + attn_flops) / world / (m["ms"] * 1e-3) / 1e12 * world,
        "stage_ms": {k: round(v[0], 3) for k, v in sorted(classes.items(), key=lambda kv: -kv[1][0])},
    }


def vae_flops(cfg, h, w):
    """One clip of the video decoder: its blocks' GEMMs (2 M N K) and attention (4 T^2 d per tile), M = tiles x T rows,
    plus the token embedding and the pixel projection."""
    import h3b200 as H
    ty, tx = len(H.vae_tile_starts(h)), len(H.vae_tile_starts(w))
    th, tw = min(16, h), min(16, w)
    T = cfg["clip"] * th * tw + cfg["registers"] + 1
    M, d, F = ty * tx * T, cfg["dim"], cfg["ffn"]
    gemm = cfg["blocks"] * 2 * M * d * (3 * d + d + 2 * F + F) + 2 * M * d * (64 + 3 * 4 * 16 * 16)
    attn = cfg["blocks"] * ty * tx * 4 * T * T * d
    return gemm, attn, ty * tx, T


def reference_vae(H):
    """The decoder's CPU restatement (oracle/vae_oracle.py) on one 16 x 16-latent tile of a clip with ONE block of
    MiniMax-H3's decoder width, the block scaled to 36 and the tile to the 28 tiles of a 768p clip."""
    import torch
    from oracle import vae_oracle as V

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    cfg = dict(H.VAE_CONFIGS["h3"])
    one, none = dict(cfg, blocks=1), dict(cfg, blocks=0)
    w1 = V.make_weights(one, 0)
    w0 = dict(w1, blocks=[])
    lat = np.random.default_rng(0).standard_normal((cfg["clip"], 16, 16, cfg["channels"]), dtype=np.float32)
    t0 = time.perf_counter()
    V.decode_clip(none, w0, lat)
    rest = time.perf_counter() - t0
    t0 = time.perf_counter()
    V.decode_clip(one, w1, lat)
    block = time.perf_counter() - t0 - rest
    clip_s = 28 * (rest + cfg["blocks"] * block)
    return {"metric": "s per 768p clip of the video VAE decoder (7 latent frames -> 28 frames)", "value": clip_s, "unit": "s",
            "impl": "reference", "n_gpus": 0, "steps": 1, "warmup": 0, "ms_per_step": (rest + block) * 1e3,
            "ms_per_step_is": "one timed sample: one tile with one block, plus one tile without blocks",
            "extrapolated_from": "1 tile x 28, 1 block x 36", "higher_is_better": False, "scaling": "strong", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic",
            "cpu_baseline": {"value": clip_s, "unit": "s", "cores": threads, "kind": "port",
                             "sample": f"oracle/vae_oracle.py decode_clip on one 16 x 16-latent tile, d 2048, one block ({block:.2f} s) "
                                       f"and the rest ({rest:.2f} s); {threads} host threads"},
            "e2e": {"value": clip_s, "unit": "s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def run_vae(args, rank):
    """--workload vae: the decoder alone (one line with its metric; --profile: warm-up + steps clip decodes, nothing
    timed, for ncu)."""
    import torch
    import h3b200 as H

    if rank != 0:
        return
    if args.profile:
        cfg = H.VAE_CONFIGS["h3"]
        m = H.VideoDecoder(cfg, seed=0)
        lat = torch.randn(cfg["clip"], 48, 84, cfg["channels"], device="cuda")
        canvas = torch.empty((cfg["clip"] * 4, 48 * 16, 84 * 16, 3), device="cuda")
        for _ in range(args.warmup + args.steps):
            m.decode_clip_device(lat.data_ptr(), 48, 84, canvas.data_ptr())
        m.close()
        return
    peaks, _ = load_peaks()
    r = measure_vae(torch, H, peaks, clips=args.steps, warmup=max(args.warmup, 1))
    r.update({"n_gpus": 1, "ms_per_step": r["value"] * 1e3, "higher_is_better": False, "scaling": "strong", "vs_baseline": None,
              "dtype": "bf16", "data": "synthetic (seeded normal latents, hash-generated weights)"})
    emit(r)


def measure_vae(torch, H, peaks, clips=3, warmup=2):
    """The video VAE decoder at MiniMax-H3's size on 768p latents: device seconds per clip (latents and canvas in
    HBM), and a whole 1344 x 768 x 124-frame video (37 latent frames, 7 clips) through h3vae_decode from host latents
    to host frames (the reference's 69 s on an M5 Max, docs/performance.md:19)."""
    cfg = H.VAE_CONFIGS["h3"]
    h, w = 48, 84
    m = H.VideoDecoder(cfg, seed=0)
    rng = np.random.default_rng(0)
    lat = torch.from_numpy(rng.standard_normal((cfg["clip"], h, w, cfg["channels"]), dtype=np.float32)).cuda()
    canvas = torch.empty((cfg["clip"] * 4, h * 16, w * 16, 3), dtype=torch.float32, device="cuda")
    ext = torch.cuda.ExternalStream(m.stream, device=canvas.device)
    for _ in range(warmup):
        m.decode_clip_device(lat.data_ptr(), h, w, canvas.data_ptr())
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    with torch.cuda.stream(ext):
        e0.record()
        for _ in range(clips):
            m.decode_clip_device(lat.data_ptr(), h, w, canvas.data_ptr())
        e1.record()
    torch.cuda.synchronize()
    clip_s = e0.elapsed_time(e1) / clips * 1e-3
    launches = m.last_launches()
    video = rng.standard_normal((37, h, w, cfg["channels"]), dtype=np.float32)
    count = [0]
    t0 = time.perf_counter()
    m.decode(video, sink=lambda i, a: count.__setitem__(0, count[0] + 1))
    e2e = time.perf_counter() - t0
    m.close()
    gemm, attn, tiles, T = vae_flops(cfg, h, w)
    peak = peaks.get("bf16_tflops_sustained", peaks.get("bf16_tflops"))
    tflops = (gemm + attn) / clip_s / 1e12
    return {"metric": "s per 768p clip of the video VAE decoder (7 latent frames -> 28 frames)", "value": clip_s, "unit": "s",
            "config": {"model": "MiniMax-H3 video VAE decoder: d 2048, 32 heads of 64, SwiGLU 8192, 36 blocks (random-init bf16)",
                       "latents": [cfg["clip"], h, w, cfg["channels"]], "tiles": tiles, "tokens_per_tile": T},
            "roofline": {"bound": "tensor", "achieved": tflops, "peak": peak, "unit": "TFLOP/s", "frac": tflops / peak,
                         "flops_per_clip": gemm + attn, "peak_kind": "measured bf16 sustained (MEASURED_PEAKS.json)"},
            "e2e": {"value": e2e, "unit": "s per 1344x768x124 video (37 latent frames, 7 clips)", "frames": count[0],
                    "h2d_bytes": int(video.nbytes), "d2h_bytes": int(count[0] * h * 16 * w * 16 * 3 * 4),
                    "reference_m5max_s": 69.0},
            "gpu_launches_per_clip": launches, "steps": clips, "warmup": warmup}


def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    import h3b200 as H

    torch.cuda.set_device(local_rank)
    cfg_name, lay_name, ratio, local, int8, wdesc = WORKLOADS[args.workload]
    cfg = dict(H.CONFIGS[cfg_name])
    if args.blocks:
        cfg["blocks"] = args.blocks  # a shorter stack of the same blocks (profiling cases)
    layout = H.Layout.named(lay_name)

    def new_model(int8_mask, sparse_ratio, sparse_local, config=None):
        nccl_id = None
        if world > 1:
            obj = [H.nccl_unique_id() if rank == 0 else None]
            dist.broadcast_object_list(obj, src=0)
            nccl_id = obj[0]
        return H.Model(config or cfg, seed=0, int8_mask=int8_mask, sparse_ratio=sparse_ratio, sparse_local=sparse_local, rank=rank,
                       world=world, nccl_id=nccl_id, device=local_rank)

    model = new_model(int8, ratio, local)
    run = Runner(H, torch, dist, model, layout, cfg, rank, world, local_rank)
    if args.profile:
        # profiling runs (ncu): just the steps, no timing extras
        for _ in range(args.warmup + args.steps):
            run.step_dev()
        model.synchronize()
        model.close()
        return
    peaks, _ = load_peaks()
    m = run.measure(args.steps, args.warmup, max(4, min(args.steps, 10)), clocks_gpu=local_rank)
    head = _line_part(m, cfg, layout, ratio, world, peaks, args.workload, int8)
    line = {
        "metric": METRIC, "value": head["value"], "unit": "s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": head["ms_per_step"], "higher_is_better": False, "scaling": "strong", "vs_baseline": None,
        "dtype": "int8" if int8 else "bf16", "data": "synthetic (seeded normal inputs, hash-generated ~N(0, 0.02) weights)",
        "config": {"workload": wdesc, "rows": layout.rows, "dim": cfg["dim"], "heads": cfg["heads"], "ffn": cfg["ffn"],
                   "blocks": cfg["blocks"], "parallelism": f"ulysses-sp{world}" if world > 1 else "single-gpu",
                   "l2": "no flush: each step streams ~54 GB of weights, far past the 126 MB L2"},
        "roofline": head["roofline"], "hbm_kernels": head["hbm_kernels"], "step_tflops": head["step_tflops"],
        "stage_ms": head["stage_ms"], "e2e": head["e2e"], "gpu_launches": m["launches"] * args.steps, "clocks": m["clocks"],
    }
    if world > 1:
        line["exchange"] = ("Ulysses all-to-all fused into the q/k/v GEMM and attention epilogues as NVLink peer stores "
                            "(CUDA IPC mappings); NCCL carries a 4-byte barrier per exchange, the AdaLN all-gather and the heads' "
                            "all-gather")
    # the other BASELINE configurations, on the same weights where the workload allows, fewer steps
    ks, kw = min(args.steps, 5), 3
    # int8 last: it needs its own model (int8 weights); the others run on the dense model's weights
    extras = [] if args.extras == "none" or args.workload != "dense" else (
        ["sparse"] + (["long", "long-sparse"] if world > 1 else []) + ["int8", "h3"])
    run_layout = lay_name
    for name in extras:
        c2name, lname, r2, l2, i2, d2 = WORKLOADS[name]
        lay2 = H.Layout.named(lname)
        cfg2 = dict(H.CONFIGS[c2name])
        if i2 or cfg2 != cfg:
            model.close()
            model = new_model(i2, r2, l2, cfg2)
            run = Runner(H, torch, dist, model, lay2, cfg2, rank, world, local_rank)
        else:
            model.set_sparse(r2, l2)
            if lname != run_layout:
                run = Runner(H, torch, dist, model, lay2, cfg, rank, world, local_rank)
        run_layout = lname
        m2 = run.measure(ks, kw, ks)
        part = _line_part(m2, cfg2, lay2, r2, world, peaks, name, i2)
        part.update({"workload": d2, "rows": lay2.rows, "steps": ks, "warmup": kw, "gpu_launches": m2["launches"] * ks})
        line[name.replace("-", "_")] = part
    if "sparse" in line:
        line["sparse"]["dense_over_sparse"] = line["value"] / line["sparse"]["value"]
    if "long" in line and "long_sparse" in line:
        line["long_sparse"]["dense_over_sparse"] = line["long"]["value"] / line["long_sparse"]["value"]
    model.close()
    if rank != 0:
        return
    if world == 1 and args.extras == "all" and args.workload == "dense":
        line["vae_decode"] = measure_vae(torch, H, peaks)
    if world == 1 and not args.no_cpu_baseline and cfg_name == "c2":
        v, b, r, desc, _ = cpu_step_sample(cfg, layout)
        line["cpu_baseline"] = {"value": v, "unit": "s", "cores": os.cpu_count(), "kind": "port", "sample": desc,
                                "block_s": b, "rest_s": r}
    emit(line)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="dense", choices=sorted(WORKLOADS))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--blocks", type=int, default=0, help="override the block count (profiling cases only)")
    ap.add_argument("--profile", action="store_true", help="run warmup + steps and exit (for ncu captures)")
    ap.add_argument("--extras", default="all", choices=["all", "none"],
                    help="with the dense workload: also measure sparse (C3), int8 (C4) and, on 2+ GPUs, the long clip (C5)")
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))
    # The JSON line is the only thing on stdout: everything else written to file descriptor 1 (NCCL's version banner
    # and other native messages included) goes to stderr.
    global _json_out
    _json_out = os.fdopen(os.dup(1), "w")
    sys.stdout.flush()
    os.dup2(2, 1)
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if args.workload == "vae":
        import torch

        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", 0)))
        run_vae(args, rank)
        return
    if world > 1:
        import datetime

        # NCCL's communicator set-up lines (ranks, transports) on stderr: the library's own communicator carries the
        # barriers and all-gathers; the all-to-all data moves as NVLink peer stores from the kernels' epilogues
        if os.environ.get("NCCL_DEBUG", "").upper() not in ("INFO", "TRACE"):
            os.environ["NCCL_DEBUG"] = "INFO"
            os.environ["NCCL_DEBUG_SUBSYS"] = "INIT"
        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local_rank))
    try:
        run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
