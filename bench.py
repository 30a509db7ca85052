#!/usr/bin/env python
"""Throughput of the two-view inference hot path on B200: MASt3R ViT-L, 512x384 image
pairs (patch 16, 24x32 = 768 tokens), global batch 64 pairs sharded over the GPUs of
one node (one process per GPU), synthetic seeded images and trunc-normal weights.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...

Prints one JSON line (rank 0).  `value` = pairs/s of the whole job from device time
(CUDA events on the engine's stream, max over ranks, inputs resident in HBM);
`e2e` = the same through the public batch API with pinned host buffers, every step
including the H2D copy of the images and the D2H copy of every output.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "image pairs/sec/GPU at MASt3R ViT-L 512 (1/2/4/8 B200); attention TFLOPS vs peak"
VARIANT = "mast3r_vit_large"
IMAGE_HW = (384, 512)
GLOBAL_PAIRS = 64
WEIGHT_SEED = 0
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def env_rank():
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("LOCAL_RANK", "0")),
            int(os.environ.get("WORLD_SIZE", "1")))


# DRAM bytes (read + write) per token row of the encoder fc1 launch (K 1024 -> N 4096, GELU,
# 16-bit output), from an ncu capture of that launch at 16 pairs (24576 rows: 58.8 MB read +
# 147.7 MB written); traffic grows with the rows, so a launch moves this many bytes per row.
FC1_DRAM_BYTES_PER_ROW = (58836992 + 147696128) / 24576


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d, "measured"
    return FALLBACK_PEAKS, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self):
        self.proc = None
        self.lines = []
        self.t = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                                          "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
            return
        self.t = threading.Thread(target=self._read, daemon=True)
        self.t.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        if self.t:
            self.t.join(timeout=2)
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


def make_inputs(first_pair: int, n: int, hw):
    """Seeded synthetic uint8 image pairs (uniform [0, 255]); pair p depends only on p."""
    img1 = np.empty((n, *hw, 3), np.uint8)
    img2 = np.empty((n, *hw, 3), np.uint8)
    for i in range(n):
        rng = np.random.default_rng(1000 + first_pair + i)
        img1[i] = rng.integers(0, 256, (*hw, 3), dtype=np.uint8)
        img2[i] = rng.integers(0, 256, (*hw, 3), dtype=np.uint8)
    return img1, img2


def weights_file(dims, rank, dist):
    from mast3r_runtime_b200 import make_weights, save_safetensors

    path = Path(os.environ.get("M3R_BENCH_WEIGHTS", f"/tmp/m3r_bench_{dims.name}_seed{WEIGHT_SEED}.safetensors"))
    if rank == 0 and not path.exists():
        tmp = path.with_suffix(".tmp")
        save_safetensors(tmp, make_weights(dims, seed=WEIGHT_SEED))
        tmp.rename(path)
    if dist is not None:
        dist.barrier()
    return path


def flops_per_pair(d, hw):
    """Algorithmic FLOP of one pair (2 per multiply-add; GEMM/conv contractions + attention 4*N^2*dh)."""
    H, W = hw
    p = d.patch
    hg, wg = H // p, W // p
    n = hg * wg
    e, c = d.enc_dim, d.dec_dim
    enc = 2 * n * (3 * p * p * e + d.enc_depth * (3 * e * e + e * e + 2 * e * d.enc_mlp)) + d.enc_depth * 4 * n * n * e
    dec = 2 * n * e * c + d.dec_depth * (2 * n * (3 * c * c + c * c + 4 * c * c + 2 * c * d.dec_mlp) + 2 * 4 * n * n * c)
    lf = 2 * n * (d.lf_in * d.lf_hidden + d.lf_hidden * d.desc_dim * p * p)
    h0, w0 = 4 * hg, 4 * wg
    dpt = 2 * n * (e * 96 + 96 * 16 * 96 + c * 192 + 192 * 4 * 192 + c * 384 + c * 768) \
        + 2 * (hg // 2) * (wg // 2) * 768 * 9 * 768 \
        + 2 * 9 * 256 * (h0 * w0 * 96 + (h0 // 2) * (w0 // 2) * 192 + hg * wg * 384 + (hg // 2) * (wg // 2) * 768) \
        + 2 * 9 * (2 * h0) * (2 * w0) * 256 * 128 + 2 * 9 * (4 * h0) * (4 * w0) * 128 * 128 + 2 * (4 * h0) * (4 * w0) * 128 * 4
    return 2 * (enc + dec + lf + dpt)  # per view, two views


def cpu_baseline_port(dims, hw, n_pairs=1, budget_s=60.0):
    """The oracle (numpy float32, all host cores) on one pair: a bounded sample of the workload."""
    from mast3r_runtime_b200 import make_weights
    from oracle.model import Model
    import oracle

    w = make_weights(dims, seed=WEIGHT_SEED)
    m = Model(w, dims, dtype=np.float32)
    img1, img2 = make_inputs(0, n_pairs, hw)
    times = []
    t_start = time.perf_counter()
    for i in range(n_pairs):
        t0 = time.perf_counter()
        m.forward(img1[i], img2[i])
        times.append(time.perf_counter() - t0)
        if time.perf_counter() - t_start > budget_s:
            break
    return {"value": len(times) / sum(times), "unit": "pairs/s", "cores": oracle.cpu_count(), "kind": "port",
            "sample": f"{len(times)} pair(s) of the 64-pair workload through oracle/model.py (numpy float32, "
                      f"all host cores), {sum(times):.1f} s"}


def run_reference(args):
    rank, _, world = env_rank()
    if rank != 0:
        return 0
    from mast3r_runtime_b200.weights import VARIANTS
    from mast3r_runtime_b200 import make_weights
    from oracle.model import Model
    import oracle

    d = VARIANTS[VARIANT]
    m = Model(make_weights(d, seed=WEIGHT_SEED), d, dtype=np.float32)
    img1, img2 = make_inputs(0, 1, IMAGE_HW)
    budget = float(os.environ.get("M3R_REFERENCE_BUDGET_S", "240"))
    t_all = time.perf_counter()
    warm = 0
    for _ in range(args.warmup):
        m.forward(img1[0], img2[0])
        warm += 1
        if time.perf_counter() - t_all > budget / 3:
            break
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        m.forward(img1[0], img2[0])
        times.append(time.perf_counter() - t0)
        if time.perf_counter() - t_all > budget:
            break
    v = 1.0 / statistics.mean(times)
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": "pairs/s", "n_gpus": args.gpus,
        "steps": len(times), "warmup": warm, "ms_per_step": 1000.0 * statistics.mean(times),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "MASt3R ViT-L 512x384 two-view inference, one pair per step (CPU)",
                   "global_batch": 1, "image": "384x512"},
        "cpu_baseline": {"value": v, "unit": "pairs/s", "cores": oracle.cpu_count(), "kind": "port",
                         "sample": "one pair per step through the reference algorithm restated in numpy "
                                   "(oracle/model.py, float32; the reference's own numpy model cannot travel "
                                   "to this host)"},
        "e2e": {"value": v, "unit": "pairs/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_ours(args):
    import ctypes  # noqa: F401

    rank, local_rank, world = env_rank()
    dist = None
    if world > 1:
        import datetime

        import torch
        import torch.distributed as tdist

        torch.cuda.set_device(local_rank)
        tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                 device_id=torch.device("cuda", local_rank))
        dist = tdist

    def allmax(x: float) -> float:
        if dist is None:
            return x
        import torch

        t = torch.tensor([x], dtype=torch.float64, device=f"cuda:{local_rank}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def barrier():
        if dist is not None:
            dist.barrier()

    from mast3r_runtime_b200 import NativeEngine, _lib
    from mast3r_runtime_b200.weights import VARIANTS

    d = VARIANTS[VARIANT]
    total_pairs = args.pairs
    per = total_pairs // world
    assert per * world == total_pairs, "global batch must divide over the GPUs"
    path = weights_file(d, rank, dist)
    eng = NativeEngine(d, IMAGE_HW, [local_rank], per)
    eng.load(str(path))
    img1, img2 = make_inputs(rank * per, per, IMAGE_HW)

    # ---------------- device-resident throughput (value)
    eng.stage(img1, img2)
    for _ in range(args.warmup):
        eng.run_resident(per)
    barrier()
    clocks = ClockSampler() if rank == 0 else None
    if clocks:
        clocks.start()
    dev_ms = []
    t0 = time.perf_counter()
    for _ in range(args.steps):
        dev_ms.append(eng.run_resident(per))
    wall = time.perf_counter() - t0
    barrier()
    clk = clocks.stop() if clocks else None
    total_ms = allmax(sum(dev_ms))
    wall = allmax(wall)
    value = total_pairs * args.steps / (total_ms / 1000.0)

    # ---------------- end to end through the public batch API (pinned host buffers)
    e2e_line = None
    if not args.no_e2e:
        p1 = _lib.pinned_empty(img1.shape, np.uint8)
        p2 = _lib.pinned_empty(img2.shape, np.uint8)
        p1[...] = img1
        p2[...] = img2
        outs = eng._out_arrays(per, alloc=_lib.pinned_empty)
        for _ in range(2):  # direct launches, then CUDA-graph capture of the sub-batch passes
            eng.infer_batch(p1, p2, out=outs)
        barrier()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            eng.infer_batch(p1, p2, out=outs)
        e2e_s = allmax(time.perf_counter() - t0)
        e2e_line = {"value": total_pairs * args.steps / e2e_s, "unit": "pairs/s",
                    "h2d_bytes_per_step": int(p1.nbytes + p2.nbytes) * world,
                    "d2h_bytes_per_step": int(sum(o.nbytes for o in outs.values())) * world}

    # ---------------- per-kernel-family device time (untimed run, events around every launch)
    eng.set_profiling(True)
    eng.run_resident(per)
    prof = eng.profile()
    ops = eng.profile_ops()
    eng.set_profiling(False)
    launches_per_step = int(prof["gemm_launches"] + prof["attn_launches"] + prof["other_launches"])

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and total_pairs == GLOBAL_PAIRS:
        cpu = cpu_baseline_port(d, IMAGE_HW)

    if rank == 0:
        pk, src = peaks()
        gemm_tf = prof["gemm_flop"] / (prof["gemm_ms"] * 1e-3) / 1e12 if prof["gemm_ms"] > 0 else 0.0
        attn_tf = prof["attn_flop"] / (prof["attn_ms"] * 1e-3) / 1e12 if prof["attn_ms"] > 0 else 0.0
        peak_tc = float(pk["bf16_tflops_sustained"])
        fc1 = ops.get("enc.fc1", {"ms": 0.0, "flop": 0.0, "launches": 1})
        fc1_tf = (fc1["flop"] / fc1["launches"]) / (fc1["ms"] / fc1["launches"] * 1e-3) / 1e12 if fc1["ms"] > 0 else 0.0
        fc1_rows = 2 * per * (IMAGE_HW[0] // d.patch) * (IMAGE_HW[1] // d.patch)
        fpp = flops_per_pair(d, IMAGE_HW)
        line = {
            "metric": METRIC, "value": value, "unit": "pairs/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": total_ms / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": eng.dtype_name, "data": "synthetic",
            "config": {"workload": "MASt3R ViT-L 512x384 two-view inference (enc 1024x24, dec 768x12, DPT + 24-d "
                                   "local-feature heads)", "global_batch": total_pairs, "pairs_per_gpu": per,
                       "image": "384x512", "parallelism": f"dp{world} (pairs sharded, no collectives)",
                       "l2": f"working set per step >> L2 (activations of {per} pairs, several GB)"},
            "per_gpu": value / world,
            # the dominant kernel's largest launch: encoder fc1 (one launch per block)
            "roofline": {"bound": "tensor", "kernel": f"gemm_tc_kernel enc.fc1 (M={fc1_rows}, N={d.enc_mlp}, "
                                                      f"K={d.enc_dim}, GELU, CTA pairs)",
                         "achieved": fc1_tf, "peak": peak_tc, "unit": "TFLOP/s", "frac": fc1_tf / peak_tc,
                         "peak_source": f"{src} bf16_tflops_sustained",
                         "traffic": FC1_DRAM_BYTES_PER_ROW * fc1_rows,
                         "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one fc1 launch at "
                                           "16 pairs, scaled by rows"},
            "gemm_family": {"kernel": "gemm_tc_kernel (all GEMM/conv launches of a step)", "achieved": gemm_tf,
                            "peak": peak_tc, "unit": "TFLOP/s", "frac": gemm_tf / peak_tc,
                            "ms_per_step": prof["gemm_ms"], "launches_per_step": int(prof["gemm_launches"])},
            "attention": {"achieved": attn_tf, "peak": peak_tc, "unit": "TFLOP/s", "frac": attn_tf / peak_tc,
                          "ms_per_step": prof["attn_ms"], "launches_per_step": int(prof["attn_launches"])},
            "model_tflops": fpp * total_pairs * args.steps / (total_ms / 1000.0) / 1e12,
            "kernel_ms_per_step": {"gemm": prof["gemm_ms"], "attention": prof["attn_ms"], "other": prof["other_ms"]},
            # per operation of the model: [device ms per step, TFLOP/s (0 for non-contractions)]
            "ops": {k: [round(o["ms"], 3), round(o["flop"] / (o["ms"] * 1e-3) / 1e12, 1) if o["ms"] > 0 else 0.0]
                    for k, o in ops.items()},
            "e2e": e2e_line,
            "wall_ms_per_step": 1000.0 * wall / args.steps,
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clk,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    eng.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--pairs", type=int, default=GLOBAL_PAIRS,
                    help="global batch (default: the 64 pairs of the benchmark; smaller for profiling runs)")
    ap.add_argument("--no-e2e", action="store_true", help="skip the end-to-end pass (profiling runs)")
    args = ap.parse_args()
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
