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


# ---------------------------------------------------------------------------- matcher (config 4)
MATCH_HW = (384, 512)       # one 512x384 descriptor map per set: N = 196,608
MATCH_D = 24
MATCH_TOP_K = 512
MATCH_THR = 0.5
FP32_LANES_PER_SM = 128     # FP32 lanes per SM per clock (B200: 148 SMs)
N_SMS = 148


def matcher_inputs(h, w, d, seed, dup_frac=0.3, sigma=0.05):
    """Two [h, w, d] descriptor maps: set B has `dup_frac` of its rows as noisy (sigma)
    copies of set-A rows at random positions, the rest fresh Gaussian (the matcher's
    synthetic workload)."""
    rng = np.random.default_rng(seed)
    n = h * w
    a = rng.standard_normal((n, d)).astype(np.float32)
    b = rng.standard_normal((n, d)).astype(np.float32)
    m = int(dup_frac * n)
    dst = rng.permutation(n)[:m]
    src = rng.permutation(n)[:m]
    b[dst] = a[src] + np.float32(sigma) * rng.standard_normal((m, d)).astype(np.float32)
    return a.reshape(h, w, d), b.reshape(h, w, d)


def run_matcher(devices, steps, sm_mhz):
    """engine.match at N = 196,608 x 24 (rows sharded over `devices`): device time per
    phase (median over steps), host wall time, and a checksum of the result."""
    import hashlib

    from mast3r_runtime_b200 import NativeEngine, tiny_dims

    a, b = matcher_inputs(*MATCH_HW, MATCH_D, 4)
    eng = NativeEngine(tiny_dims(), (32, 32), devices, 1)  # the matcher needs no weights
    r = eng.match(a, b, top_k=MATCH_TOP_K, reciprocal=True, confidence_threshold=MATCH_THR)  # warm-up
    ph = {"normalize_ms": [], "argmax_ms": [], "select_ms": [], "kernel_ms": [], "wall_ms": []}
    for _ in range(max(steps, 3)):
        t0 = time.perf_counter()
        r = eng.match(a, b, top_k=MATCH_TOP_K, reciprocal=True, confidence_threshold=MATCH_THR)
        ph["wall_ms"].append(1000.0 * (time.perf_counter() - t0))
        for k in ("normalize_ms", "argmax_ms", "select_ms", "kernel_ms"):
            ph[k].append(r.timing[k])
    eng.close()
    med = {k: statistics.median(v) for k, v in ph.items()}
    n = MATCH_HW[0] * MATCH_HW[1]
    lane_ops = 2.0 * n * n * MATCH_D          # one multiply and one add per term, issued separately
    peak = N_SMS * FP32_LANES_PER_SM * 1965e6 * len(devices)
    argmax_rate = lane_ops / (med["argmax_ms"] * 1e-3)
    norm_bytes = 2 * 2 * n * MATCH_D * 4       # both sets read and written
    digest = hashlib.sha256(r.idx_1.tobytes() + r.idx_2.tobytes() + r.confidence.tobytes()).hexdigest()[:16]
    return {
        "workload": f"reciprocal top-{MATCH_TOP_K} matcher, N = {n} x {MATCH_D} fp32 per set, 30% noisy copies, "
                    f"threshold {MATCH_THR}; rows of set A sharded over {len(devices)} GPU(s)",
        "devices": len(devices), "matches": int(len(r.idx_1)), "checksum": digest,
        "ms": med["kernel_ms"], "wall_ms": med["wall_ms"],
        "phase_ms": {k[:-3]: med[k] for k in ("normalize_ms", "argmax_ms", "select_ms")},
        "argmax": {"bound": "fp32 pipe", "achieved": argmax_rate / 1e12, "unit": "T lane-ops/s",
                   "peak": peak / 1e12, "frac": argmax_rate / peak,
                   "work": f"{lane_ops:.4g} lane-ops (N^2 D multiplies + N^2 D adds, not fused: the "
                           f"reference's rounding)",
                   "peak_source": f"nominal {N_SMS} SMs x {FP32_LANES_PER_SM} FP32 lanes x 1965 MHz per GPU"
                                  + (f"; median SM clock under load {sm_mhz:.0f} MHz" if sm_mhz else "")},
        "normalize": {"bound": "hbm", "bytes": norm_bytes,
                      "achieved_gbs": norm_bytes / (med["normalize_ms"] * 1e-3) / 1e9},
    }


def cpu_baseline_matcher(rows=32768):
    """The oracle's matcher (oracle/matcher.c, OpenMP on all host cores) on `rows` rows of
    set A against all of set B, extrapolated to the full N x N arg-max."""
    import oracle

    a, b = matcher_inputs(*MATCH_HW, MATCH_D, 4)
    n = MATCH_HW[0] * MATCH_HW[1]
    an = oracle.normalize(a.reshape(n, MATCH_D))
    bn = oracle.normalize(b.reshape(n, MATCH_D))
    t0 = time.perf_counter()
    oracle.argmax(an, bn, 0, rows)
    t = time.perf_counter() - t0
    return {"value": t * n / rows * 1000.0, "unit": "ms per match (arg-max, extrapolated)", "cores": oracle.cpu_count(),
            "kind": "port", "sample": f"oracle/matcher.c arg-max of {rows} of {n} rows against all {n} columns "
                                      f"({t:.1f} s), scaled by {n / rows:.0f}"}


# ---------------------------------------------------------------------------- isolated attention (config 1)
ATT_SEQS, ATT_HEADS, ATT_TOK = 128, 12, 576   # 64 pairs x 2 views, 24 x 24 grid, head dim 64


def run_attention(dtype, iters=20):
    """m3r_attention_fwd on [128 seqs, 12 heads, 576, 64] Q/K/V ~ N(0, 1): self (K, V of the
    same view) and cross (K, V of the other view of the pair); mean kernel time per launch."""
    import ctypes

    from mast3r_runtime_b200 import _lib

    lib = _lib.load()
    rng = np.random.default_rng(9)
    shape = (ATT_SEQS, ATT_HEADS, ATT_TOK, 64)

    def bits(x):
        if dtype == _lib.DTYPE_F16:
            return x.astype(np.float16).view(np.uint16)
        u = x.astype(np.float32).view(np.uint32).astype(np.uint64)
        return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)

    q = bits(rng.standard_normal(shape, dtype=np.float32))
    k = bits(rng.standard_normal(shape, dtype=np.float32))
    v = bits(rng.standard_normal(shape, dtype=np.float32))
    other = np.concatenate([np.arange(64, 128), np.arange(0, 64)])  # view 1 <-> view 2 of each pair
    kc, vc = np.ascontiguousarray(k[other]), np.ascontiguousarray(v[other])
    out = np.empty((ATT_SEQS, ATT_TOK, ATT_HEADS * 64), np.uint16)
    flop = 4.0 * ATT_TOK * ATT_TOK * 64 * ATT_SEQS * ATT_HEADS
    res = {}
    for name, kk, vv in (("self", k, v), ("cross", kc, vc)):
        ms = ctypes.c_float(0)
        _lib.check(lib.m3r_attention_fwd(0, dtype, _lib.ptr(q), _lib.ptr(kk), _lib.ptr(vv), _lib.ptr(out), ATT_SEQS,
                                         ATT_HEADS, ATT_TOK, ATT_TOK, 0.125, iters, ctypes.byref(ms)))
        res[name] = {"ms": ms.value, "tflops": flop / (ms.value * 1e-3) / 1e12}
    return flop, res


def cpu_baseline_attention(slices=384):
    """The reference's own multi_head_attention (csrc/cpu/attention.cpp, OpenMP, compiled into
    oracle/_ref) on `slices` of the 1536 (sequence, head) slices; GFLOP/s of that sample."""
    import oracle

    L = oracle.ref_lib()
    if L is None:
        return None
    rng = np.random.default_rng(9)
    q, k, v = (rng.standard_normal((1, slices, ATT_TOK, 64), dtype=np.float32) for _ in range(3))
    o = np.empty_like(q)
    t0 = time.perf_counter()
    L.ref_multi_head_attention(q, k, v, o, 1, slices, ATT_TOK, 64)
    t = time.perf_counter() - t0
    flop = 4.0 * ATT_TOK * ATT_TOK * 64 * slices
    return {"value": flop / t / 1e9, "unit": "GFLOP/s", "cores": oracle.cpu_count(), "kind": "reference",
            "sample": f"{slices} of 1536 (sequence, head) slices through the reference's multi_head_attention "
                      f"(oracle/_ref), {t:.2f} s"}


def run_small_config(variant, hw, pairs, dtype_name, device, steps, warmup):
    """Device-resident pairs/s of another model configuration on one GPU (rank 0 only)."""
    from mast3r_runtime_b200 import NativeEngine, _lib
    from mast3r_runtime_b200.weights import VARIANTS

    d = VARIANTS[variant]
    path = weights_file(d, 0, None)
    img1, img2 = make_inputs(0, pairs, hw)
    dt = {"fp16": _lib.DTYPE_F16, "bf16": _lib.DTYPE_BF16}[dtype_name]
    eng = NativeEngine(d, hw, [device], pairs, dt)
    eng.load(str(path))
    eng.stage(img1, img2)
    for _ in range(warmup):
        eng.run_resident(pairs)
    ms = [eng.run_resident(pairs) for _ in range(steps)]
    eng.close()
    total = sum(ms)
    return {"value": pairs * steps / (total / 1000.0), "unit": "pairs/s", "pairs_per_pass": pairs,
            "ms_per_pass": total / steps, "dtype": dtype_name,
            "model_tflops": flops_per_pair(d, hw) * pairs * steps / (total / 1000.0) / 1e12}


def cpu_baseline_port(dims, hw, n_pairs=1, budget_s=60.0, workload="the 64-pair workload"):
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
            "sample": f"{len(times)} pair(s) of {workload} through oracle/model.py (numpy float32, "
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


def shard_pairs(total_pairs: int, world: int, rank: int):
    """(first pair, pairs) of this rank: the global batch split evenly, in rank order."""
    per = total_pairs // world
    assert per * world == total_pairs, "global batch must divide over the GPUs"
    return rank * per, per


def all_max(dist, x: float, device=None) -> float:
    """Maximum of x over the ranks of the default group (x itself without one)."""
    if dist is None:
        return x
    import torch

    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def run_ours(args):
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
        # host-side waits while rank 0 drives every GPU (the sharded matcher): an NCCL
        # barrier would leave a spinning kernel on each waiting rank's GPU, time-sliced
        # against rank 0's kernels there
        host_group = tdist.new_group(backend="gloo", timeout=datetime.timedelta(seconds=600))

    def allmax(x: float) -> float:
        return all_max(dist, x, f"cuda:{local_rank}")

    def barrier():
        if dist is not None:
            dist.barrier()

    def host_barrier():
        if dist is not None:
            dist.barrier(group=host_group)

    from mast3r_runtime_b200 import NativeEngine, _lib
    from mast3r_runtime_b200.weights import VARIANTS

    d = VARIANTS[VARIANT]
    total_pairs = args.pairs
    first, per = shard_pairs(total_pairs, world, rank)
    dtypes = {"fp16": _lib.DTYPE_F16, "bf16": _lib.DTYPE_BF16}
    main_dt = dtypes[args.dtype]
    path = weights_file(d, rank, dist)
    img1, img2 = make_inputs(first, per, IMAGE_HW)

    def resident(eng, sample_clocks):
        """W warm-up + K timed resident passes; (device ms summed over K, max over ranks), wall s, clocks."""
        eng.stage(img1, img2)
        for _ in range(args.warmup):
            eng.run_resident(per)
        barrier()
        clocks = ClockSampler() if sample_clocks else None
        if clocks:
            clocks.start()
        dev_ms = []
        t0 = time.perf_counter()
        for _ in range(args.steps):
            dev_ms.append(eng.run_resident(per))
        wall = time.perf_counter() - t0
        barrier()
        clk = clocks.stop() if clocks else None
        return allmax(sum(dev_ms)), allmax(wall), clk

    def profiled(eng):
        """One untimed resident pass with CUDA events around every launch."""
        eng.set_profiling(True)
        eng.run_resident(per)
        prof, ops = eng.profile(), eng.profile_ops()
        eng.set_profiling(False)
        return prof, ops

    # ---------------- device-resident throughput (value), operand type of the headline
    eng = NativeEngine(d, IMAGE_HW, [local_rank], per, main_dt)
    eng.load(str(path))
    total_ms, wall, clk = resident(eng, rank == 0)
    value = total_pairs * args.steps / (total_ms / 1000.0)

    # ---------------- end to end through the public batch API
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
        h2d, d2h = [], []
        t0 = time.perf_counter()
        for _ in range(args.steps):
            _, tm = eng.infer_batch(p1, p2, out=outs)
            h2d.append(tm["h2d_ms"])
            d2h.append(tm["d2h_ms"])
        e2e_s = allmax(time.perf_counter() - t0)
        out_bytes = int(sum(o.nbytes for o in outs.values()))
        d2h_max_ms = allmax(statistics.median(d2h))  # every rank copies at once: the host's aggregate rate
        e2e_line = {"value": total_pairs * args.steps / e2e_s, "unit": "pairs/s",
                    "h2d_bytes_per_step": int(p1.nbytes + p2.nbytes) * world,
                    "d2h_bytes_per_step": out_bytes * world,
                    "host_buffers": "pinned (m3r_host_alloc)",
                    "rank0_h2d_ms": statistics.median(h2d), "rank0_d2h_ms": statistics.median(d2h),
                    "rank0_d2h_gbs": out_bytes / (statistics.median(d2h) * 1e-3) / 1e9 if d2h[0] > 0 else None,
                    "all_ranks_d2h_gbs": out_bytes * world / (d2h_max_ms * 1e-3) / 1e9 if d2h_max_ms > 0 else None}
        # the call the drop-in engine makes: ordinary numpy images in, outputs from the
        # engine's recycled page-locked buffers (the previous step's are released first)
        del outs
        res, _ = eng.infer_batch(img1, img2)  # the pool's first set is allocated (and pinned) here
        res = None
        barrier()
        t0 = time.perf_counter()
        for _ in range(max(1, args.steps // 2)):
            res = None
            res, _ = eng.infer_batch(img1, img2)
        del res
        pg_s = allmax(time.perf_counter() - t0)
        e2e_line["drop_in"] = {"value": total_pairs * max(1, args.steps // 2) / pg_s, "unit": "pairs/s",
                               "host_buffers": "numpy images; outputs in recycled pinned buffers (infer_batch)"}
    prof, ops = profiled(eng)
    eng.close()
    launches_per_step = int(prof["gemm_launches"] + prof["attn_launches"] + prof["other_launches"])

    # ---------------- the other 16-bit operand type (same weights file, same workload)
    other = None
    if not args.no_other_dtype:
        oname = "bf16" if args.dtype == "fp16" else "fp16"
        eng = NativeEngine(d, IMAGE_HW, [local_rank], per, dtypes[oname])
        eng.load(str(path))
        o_ms, _, _ = resident(eng, False)
        o_prof, o_ops = profiled(eng)
        eng.close()
        o_attn = o_prof["attn_flop"] / (o_prof["attn_ms"] * 1e-3) / 1e12 if o_prof["attn_ms"] > 0 else 0.0
        other = {"dtype": oname, "value": total_pairs * args.steps / (o_ms / 1000.0), "unit": "pairs/s",
                 "ms_per_step": o_ms / args.steps, "attention_tflops": o_attn,
                 "ops": {k: [round(o["ms"], 3), round(o["flop"] / (o["ms"] * 1e-3) / 1e12, 1) if o["ms"] > 0 else 0.0]
                         for k, o in o_ops.items()}}

    # ---------------- one pair per call through the object NativeEngineWrapper drives
    latency = None
    if rank == 0 and not args.no_e2e:
        from mast3r_runtime_b200 import CUDAEngine

        ce = CUDAEngine(variant=VARIANT, precision=args.dtype, image_size=IMAGE_HW, devices=[local_rank])
        ce.load(str(path))
        ce.warmup(3)
        lat = []
        for i in range(10):
            t0 = time.perf_counter()
            r = ce.infer(img1[i % per], img2[i % per])
            lat.append(1000.0 * (time.perf_counter() - t0))
        t0 = time.perf_counter()
        m = ce.match(r.desc_1, r.desc_2, top_k=MATCH_TOP_K, reciprocal=True, confidence_threshold=MATCH_THR)
        match_ms = 1000.0 * (time.perf_counter() - t0)
        latency = {"infer_ms_per_pair": statistics.median(lat), "match_ms": match_ms, "matches": int(len(m.idx_1)),
                   "path": "CUDAEngine.infer(img1, img2) -> numpy (the call NativeEngineWrapper.infer makes, "
                           "native_wrapper.py:84-97), one 384x512 pair, host wall time, median of 10"}
        for e in list(ce._engines.values()) + ([ce._matcher] if ce._matcher is not None else []):
            e.close()
    barrier()

    # ---------------- matcher at N = 196,608 (rank 0 drives all N GPUs; the others wait)
    matcher = None
    barrier()
    host_barrier()
    if rank == 0 and not args.no_matcher:
        matcher = run_matcher(list(range(world)), args.steps, clk["sm_mhz"] if clk else None)
    host_barrier()

    # ---------------- isolated attention (128 seqs x 12 heads x 576 x 64), one GPU
    attention_iso = None
    if rank == 0 and not args.no_matcher:
        flop, res = run_attention(main_dt)
        attention_iso = {"workload": f"{ATT_SEQS} seqs (64 pairs x 2 views) x {ATT_HEADS} heads x {ATT_TOK} tokens "
                                     f"(24x24 grid) x 64, {args.dtype}, Q/K/V ~ N(0,1) (RoPE is applied by the "
                                     f"producing QKV GEMM's epilogue in this design)", "flop_per_launch": flop, **res}
        # the operand type the configuration states (bf16) beside the headline's
        oname = "bf16" if args.dtype == "fp16" else "fp16"
        attention_iso[oname] = run_attention(dtypes[oname])[1]

    # ---------------- the smaller configurations, device-resident on rank 0's GPU
    small = None
    if rank == 0 and not args.no_matcher:
        small = {
            "config0": {"workload": "DUNE ViT-S/14 encoder + MASt3R decoder and heads, 336x336, 1 pair per pass "
                                    "(precision fp32 runs fp16 operands with fp32 accumulation)",
                        **run_small_config("dune_vit_small_336", (336, 336), 1, "fp16", local_rank, args.steps,
                                           args.warmup)},
            "config2": {"workload": "DUNE ViT-B/14 encoder + MASt3R decoder and heads, 336x336, bf16: the 4-pair "
                                    "share of one GPU when 32 pairs are sharded over 8, and the whole 32-pair "
                                    "batch on one GPU",
                        "per_gpu_share": run_small_config("dune_vit_base_336", (336, 336), 4, "bf16", local_rank,
                                                          args.steps, args.warmup),
                        "whole_batch": run_small_config("dune_vit_base_336", (336, 336), 32, "bf16", local_rank,
                                                        args.steps, args.warmup)},
        }
    barrier()

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and total_pairs == GLOBAL_PAIRS:
        cpu = cpu_baseline_port(d, IMAGE_HW)
        if matcher is not None:
            matcher["cpu_baseline"] = cpu_baseline_matcher()
        if attention_iso is not None:
            attention_iso["cpu_baseline"] = cpu_baseline_attention()
        if small is not None:
            from mast3r_runtime_b200.weights import VARIANTS

            small["config0"]["cpu_baseline"] = cpu_baseline_port(VARIANTS["dune_vit_small_336"], (336, 336),
                                                                 workload="the 1-pair DUNE-S/14 336 workload")

    if rank == 0:
        pk, src = peaks()
        gemm_tf = prof["gemm_flop"] / (prof["gemm_ms"] * 1e-3) / 1e12 if prof["gemm_ms"] > 0 else 0.0
        attn_tf = prof["attn_flop"] / (prof["attn_ms"] * 1e-3) / 1e12 if prof["attn_ms"] > 0 else 0.0
        peak_tc = float(pk["bf16_tflops_sustained"])
        peak_burst = float(pk["bf16_tflops"])
        fc1 = ops.get("enc.fc1", {"ms": 0.0, "flop": 0.0, "launches": 1})
        fc1_tf = (fc1["flop"] / fc1["launches"]) / (fc1["ms"] / fc1["launches"] * 1e-3) / 1e12 if fc1["ms"] > 0 else 0.0
        fc1_rows = 2 * per * (IMAGE_HW[0] // d.patch) * (IMAGE_HW[1] // d.patch)
        fc1_alg_bytes = fc1_rows * d.enc_dim * 2 + d.enc_mlp * d.enc_dim * 2 + fc1_rows * d.enc_mlp * 2
        fpp = flops_per_pair(d, IMAGE_HW)
        if attention_iso is not None:
            for k in ("self", "cross"):
                attention_iso[k]["frac_of_burst"] = attention_iso[k]["tflops"] / peak_burst
                for other_dt in ("fp16", "bf16"):
                    if other_dt in attention_iso:
                        attention_iso[other_dt][k]["frac_of_burst"] = attention_iso[other_dt][k]["tflops"] / peak_burst
        line = {
            "metric": METRIC, "value": value, "unit": "pairs/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": total_ms / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": args.dtype, "data": "synthetic",
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
                         "traffic_source": "SCALED, not measured at this size: ncu dram__bytes_read.sum + "
                                           "dram__bytes_write.sum of one fc1 launch at 16 pairs (24576 rows), "
                                           "times the rows of this launch",
                         "algorithmic_bytes": fc1_alg_bytes},
            "gemm_family": {"kernel": "gemm_tc_kernel (all GEMM/conv launches of a step)", "achieved": gemm_tf,
                            "peak": peak_tc, "unit": "TFLOP/s", "frac": gemm_tf / peak_tc,
                            "ms_per_step": prof["gemm_ms"], "launches_per_step": int(prof["gemm_launches"])},
            "attention": {"achieved": attn_tf, "peak": peak_tc, "unit": "TFLOP/s", "frac": attn_tf / peak_tc,
                          "frac_of_burst": attn_tf / peak_burst,
                          "ms_per_step": prof["attn_ms"], "launches_per_step": int(prof["attn_launches"])},
            "attention_isolated": attention_iso,
            "matcher": matcher,
            "small_configs": small,
            "model_tflops": fpp * total_pairs * args.steps / (total_ms / 1000.0) / 1e12,
            "kernel_ms_per_step": {"gemm": prof["gemm_ms"], "attention": prof["attn_ms"], "other": prof["other_ms"]},
            # per operation of the model: [device ms per step, TFLOP/s (0 for non-contractions)]
            "ops": {k: [round(o["ms"], 3), round(o["flop"] / (o["ms"] * 1e-3) / 1e12, 1) if o["ms"] > 0 else 0.0]
                    for k, o in ops.items()},
            "other_dtype": other,
            "e2e": e2e_line,
            "latency": latency,
            "wall_ms_per_step": 1000.0 * wall / args.steps,
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clk,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
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
    ap.add_argument("--dtype", choices=("fp16", "bf16"), default="fp16", help="operand type of the headline line")
    ap.add_argument("--no-other-dtype", action="store_true", help="skip the pass in the other 16-bit type")
    ap.add_argument("--no-matcher", action="store_true",
                    help="skip the matcher, isolated-attention and small-configuration lines")
    args = ap.parse_args()
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
