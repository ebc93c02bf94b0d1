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
    """Algorithmic FLOPs of one step: the block GEMMs and attention (the SURVEY's per-unit figures)."""
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

def cpu_sample(cfg, S, n_q=4096, n_k=16384, threads=None):
    """The CPU restatement (the oracle's block arithmetic, fp32 with bf16-valued weights) on one full-width block:
    q/k/v for n_k rows, attention of n_q queries over those n_k keys, the out projection and the FFN for n_q rows;
    each part scaled to all S rows (work per row is uniform) and to every block. Returns (s per step, description)."""
    import torch
    from oracle import h3_oracle as O

    threads = threads or os.cpu_count() or 1
    torch.set_num_threads(threads)
    d, H, F, L = cfg["dim"], cfg["heads"], cfg["ffn"], cfg["blocks"]
    inner = H * 128
    g = torch.Generator().manual_seed(0)
    w = lambda *s: (torch.randn(*s, generator=g) * 0.02).bfloat16().float()
    Wqkv, Wout, W1, W2 = w(3 * inner, d), w(d, inner), w(2 * F, d), w(d, F)
    Wada = w(18 * d, cfg["time_dim"])
    n_k, n_q = min(n_k, S), min(n_q, S)
    x = torch.randn(n_k, d, generator=g)
    mod = torch.randn(6, d, generator=g) * 0.1
    pos = np.stack([np.arange(n_k, dtype=np.float64)] * 3, 1)
    cs = torch.from_numpy(O.rope_table(pos))
    t0 = time.perf_counter()
    s = torch.randn(1, cfg["time_dim"], generator=g)
    _ = s @ Wada.T
    t_ada = time.perf_counter() - t0
    t0 = time.perf_counter()
    h = O.rms(x, 1e-6) * (1 + mod[1]) + mod[0]
    qkv = (h @ Wqkv.T).reshape(n_k, 3, H, 128)
    q = O.rope(O.rms(qkv[:n_q, 0], 1e-6), cs[:n_q])
    k = O.rope(O.rms(qkv[:, 1], 1e-6), cs)
    v = qkv[:, 2]
    t_qkv = time.perf_counter() - t0
    t0 = time.perf_counter()
    qh, kh, vh = q.permute(1, 0, 2), k.permute(1, 0, 2), v.permute(1, 0, 2)
    o = torch.empty_like(qh)
    for hh in range(H):  # one head at a time keeps the score matrix to n_q x n_k
        o[hh] = torch.softmax(qh[hh] @ kh[hh].T / math.sqrt(128.0), -1) @ vh[hh]
    t_attn = time.perf_counter() - t0
    t0 = time.perf_counter()
    xr = x[:n_q] + mod[2] * (o.permute(1, 0, 2).reshape(n_q, inner) @ Wout.T)
    h2 = O.rms(xr, 1e-6) * (1 + mod[4]) + mod[3]
    gv = h2 @ W1.T
    a = torch.nn.functional.silu(gv[:, :F]) * gv[:, F:]
    xr = xr + mod[5] * (a @ W2.T)
    t_rest = time.perf_counter() - t0
    block = t_qkv * (S / n_k) + t_attn * (S / n_q) * (S / n_k) + t_rest * (S / n_q) + t_ada
    desc = (f"one full-width block (d {d}, {H} heads, SwiGLU {F}): q/k/v for {n_k} rows, attention of {n_q} queries over "
            f"{n_k} keys, out + FFN for {n_q} rows, each part scaled to S = {S} rows and x{L} blocks; torch fp32 on "
            f"{threads} threads")
    return block * L, desc, t_qkv + t_attn + t_rest + t_ada


# ---------------------------------------------------------------------------------------------------- arms

def run_reference(args, rank, world):
    """The reference's host-side path for the step: the CPU restatement (the reference's own step is Metal inside
    an absent submodule), all host threads, a bounded sample per step scaled to the full step."""
    if rank != 0:
        return
    import h3b200 as H
    cfg_name, lay_name, ratio, local, int8, wdesc = WORKLOADS[args.workload]
    cfg = H.CONFIGS[cfg_name]
    S = H.Layout.named(lay_name).rows
    vals = []
    desc = ""
    for i in range(args.warmup + args.steps):
        v, desc, _ = cpu_sample(cfg, S)
        if i >= args.warmup:
            vals.append(v)
    value = statistics.mean(vals)
    threads = os.cpu_count()
    line = {"metric": METRIC, "value": value, "unit": "s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": value * 1e3, "higher_is_better": False, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "impl": "reference",
            "config": {"workload": wdesc, "rows": S, "dim": cfg["dim"], "heads": cfg["heads"], "blocks": cfg["blocks"]},
            "cpu_baseline": {"value": value, "unit": "s", "cores": threads, "kind": "port", "sample": desc},
            "e2e": {"value": value, "unit": "s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    emit(line)


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
    nccl_id = None
    if world > 1:
        obj = [H.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        nccl_id = obj[0]
    model = H.Model(cfg, seed=0, int8_mask=int8, sparse_ratio=ratio, sparse_local=local, rank=rank, world=world,
                    nccl_id=nccl_id, device=local_rank)
    rng = np.random.default_rng(0)
    text = rng.standard_normal((layout.d["text"], cfg["text_dim"]), dtype=np.float32)
    video = rng.standard_normal((layout.video_rows, 96), dtype=np.float32)
    audio = rng.standard_normal((layout.audio_rows, 32), dtype=np.float32)
    model.begin(text, layout)
    dev = torch.device("cuda", local_rank)
    dv, da = torch.from_numpy(video).to(dev), torch.from_numpy(audio).to(dev)
    ov, oa = torch.empty_like(dv), torch.empty_like(da)
    ext = torch.cuda.ExternalStream(model.stream, device=dev)
    t_v, t_a = 0.7, 0.7

    def step_dev():
        model.step_device(dv.data_ptr(), layout.video_rows, da.data_ptr() if da.numel() else None, layout.audio_rows, t_v, t_a,
                          ov.data_ptr(), oa.data_ptr() if oa.numel() else None)

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(args.warmup):
        step_dev()
    model.synchronize()
    if args.profile:
        # profiling runs (ncu): just the steps, no timing extras
        for _ in range(args.steps):
            step_dev()
        model.synchronize()
        model.close()
        return

    # ---- value: device time per step, inputs resident
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clk:
        with torch.cuda.stream(ext):
            e0.record()
            for _ in range(args.steps):
                step_dev()
            e1.record()
        model.synchronize()
    torch.cuda.synchronize()
    barrier()
    ms = e0.elapsed_time(e1) / args.steps
    launches = model.last_launches()
    clocks = clk.summary()

    # ---- per-kernel-class device times (events after each kernel class of every block), one more step
    model.set_timing(True)
    step_dev()
    model.synchronize()
    classes = model.timing_by_class()
    model.set_timing(False)

    # ---- e2e through h3_step with pinned host buffers
    pin = lambda a: torch.from_numpy(a).pin_memory().numpy()
    pv, pa = pin(video), pin(audio)
    hv = torch.empty(video.shape, dtype=torch.float32).pin_memory().numpy()
    ha = torch.empty(audio.shape, dtype=torch.float32).pin_memory().numpy()
    barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        H.check(H.lib().h3_step(model.h, pv.ctypes.data, pv.shape[0], pa.ctypes.data if pa.size else None, pa.shape[0], t_v, t_a,
                                hv.ctypes.data, ha.ctypes.data if ha.size else None))
    e2e_s = (time.perf_counter() - t0) / args.steps
    barrier()

    # ---- max over ranks
    if world > 1:
        t = torch.tensor([ms, e2e_s], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, e2e_s = float(t[0]), float(t[1])
    if not np.isfinite(hv).all():
        raise RuntimeError("non-finite velocities")
    model.close()
    if rank != 0:
        return

    S = layout.rows
    gemm_flops, attn_flops = step_flops(cfg, S, layout.d, ratio)
    peaks, peak_kind = load_peaks()
    L = cfg["blocks"]
    attn_ms, attn_n = classes.get("attn", (0.0, 0))
    attn_launch = attention_flops(cfg, S, layout.d, ratio) / world
    achieved = attn_launch / (attn_ms / max(attn_n, 1) * 1e-3) / 1e12 if attn_ms else None
    peak = peaks.get("bf16_tflops_sustained", peaks.get("bf16_tflops"))
    gemm_ms = sum(classes.get(c, (0.0, 0))[0] for c in ("qkv", "out", "fc1", "fc2"))
    gemm_tflops = (gemm_flops / world) / (gemm_ms * 1e-3) / 1e12 if gemm_ms else None
    breakdown = {k: round(v[0], 3) for k, v in sorted(classes.items(), key=lambda kv: -kv[1][0])}
    line = {
        "metric": METRIC, "value": ms / 1e3, "unit": "s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms, "higher_is_better": False, "scaling": "strong", "vs_baseline": None,
        "dtype": "int8" if int8 else "bf16", "data": "synthetic (seeded normal inputs, hash-generated ~N(0, 0.02) weights)",
        "config": {"workload": wdesc, "rows": S, "dim": cfg["dim"], "heads": cfg["heads"], "ffn": cfg["ffn"], "blocks": L,
                   "parallelism": f"ulysses-sp{world}" if world > 1 else "single-gpu",
                   "l2": "no flush: each step streams ~54 GB of weights, far past the 126 MB L2"},
        "roofline": {"bound": "tensor", "kernel": "attention (flash_attn, tcgen05)", "achieved": achieved, "peak": peak,
                     "unit": "TFLOP/s", "frac": (achieved / peak) if achieved else None,
                     "traffic": load_traffic("attention", args.workload) if world == 1 else None,
                     "peak_kind": f"{peak_kind} bf16 sustained",
                     "launch_flops": attn_launch, "launch_ms": attn_ms / max(attn_n, 1) if attn_n else None,
                     "gemm_tflops": gemm_tflops, "gemm_frac": gemm_tflops / peak if gemm_tflops else None},
        "step_tflops": (gemm_flops + attn_flops) / (ms * 1e-3) / 1e12,
        "stage_ms": breakdown,
        "e2e": {"value": e2e_s, "unit": "s", "h2d_bytes_per_step": int(video.nbytes + audio.nbytes),
                "d2h_bytes_per_step": int(hv.nbytes + ha.nbytes)},
        "gpu_launches": launches * args.steps,
        "clocks": clocks,
    }
    if world == 1 and not args.no_cpu_baseline:
        v, desc, spent = cpu_sample(cfg, S)
        line["cpu_baseline"] = {"value": v, "unit": "s", "cores": os.cpu_count(), "kind": "port", "sample": desc,
                                "sample_seconds": spent}
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
    if world > 1:
        import datetime

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
