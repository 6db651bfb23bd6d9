#!/usr/bin/env python3
"""Benchmark of the B200 FlashAttention-2 forward (one JSON line on rank 0).

Headline workload (default, --config cfg4): causal GQA forward, bf16,
B=4 S=8192 Hq=32 Hkv=8 D=128, rotate-half RoPE theta=5e5, seeded N(0,1)
inputs resident in HBM. A step is one `_flash_attn_metal.forward` call
(fp16 staging pass + attention kernel). With --gpus N (torchrun, one
process per GPU) the SAME problem is split across the ranks: its 32
(batch, KV-head) units go 32/N per rank through multi_gpu.unit_forward
(strong scaling, no collective on the data path); value = FLOPs of the
whole problem / max-over-ranks device time. The weak-scaling figure (every
rank its own full cfg4) stays on the line as `replicas`, and the few-heads
long-context problem cfg5b (8 query heads over one KV head, S = 65536) is
split over the ranks both ways -- zig-zag query rows with K/V replicated
(split_q) and key ranges merged by the row owners over NVLink (split_kv) --
each checked in-run against an fp32 evaluation on the rank's own GPU.

At N = 1 the line also carries every configuration's kernel / step / e2e
TFLOP/s (`configs`), the reference's own benchmark protocol on its
published shapes through the NumPy API (`readme_shapes`: median of 100
calls after 20 warm-up, test.py:183-200 on test.py:502-510), the cfg4
end-to-end figure through the NumPy (pageable) API (`e2e_numpy`), and the
reference's PyTorch CPU attention on the host cores (`cpu_baseline`).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config cfg4]
    python bench.py --impl reference ...   # the reference's CPU attention on the host cores

FLOPs per step = 4*B*Hq*S^2*D, halved for causal.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
# Rank 0's stdout carries exactly one JSON line: keep NCCL's banner off it.
os.environ.setdefault("NCCL_DEBUG", "WARN")
# The only collectives are one-element barriers: no NVLink multicast objects.
os.environ.setdefault("NCCL_NVLS_ENABLE", "0")

METRIC = "attn fwd TFLOP/s and % of B200 dense BF16 peak at 1/2/4/8 GPUs; ms/call"
DATASHEET_BF16_TFLOPS = 2250.0
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
L2_BYTES = 126 * 1024 * 1024

# name: (B, S, Hq, Hkv, D, dtype, causal, rope_theta, amplitude, description)
CONFIGS = {
    "cfg1": (1, 512, 8, 8, 64, "float32", True, None, 1.0, "causal MHA fp32 B1 S512 H8 D64 (README example)"),
    "cfg2": (4, 1024, 16, 16, 64, "float16", False, None, 1.0, "MHA fp16 B4 S1024 H16 D64 non-causal"),
    "cfg3": (8, 2048, 32, 32, 128, "float16", True, 10000.0, 1.0, "causal MHA fp16 B8 S2048 H32 D128 RoPE 1e4"),
    "cfg4": (4, 8192, 32, 8, 128, "bfloat16", True, 500000.0, 1.0,
             "causal GQA bf16 B4 S8192 Hq32 Hkv8 D128 RoPE 5e5"),
    "cfg5a": (1, 65536, 64, 8, 128, "bfloat16", True, 500000.0, 0.5,
              "long-context causal GQA bf16 B1 S65536 Hq64 Hkv8 D128 RoPE 5e5"),
    "cfg5b": (1, 65536, 8, 1, 128, "bfloat16", True, 500000.0, 0.5,
              "long-context causal MQA bf16 B1 S65536 Hq8 Hkv1 D128 RoPE 5e5 (split-KV across GPUs)"),
}
# Configs whose one problem is split across the ranks by query rows or key ranges (--split).
SPLIT_KV = {"cfg5b"}
# The reference's benchmark shapes (test.py:502-510; fp16, non-causal, H=8,
# k = v = q = 0.02 * N(0,1) with seed 42, scale 1/sqrt(D)) and its published
# Metal ms (README.md:22-30, Apple GPU, chip unstated) for context.
README_SHAPES = [((4, 256, 8, 64), 0.20), ((4, 512, 8, 64), 0.31), ((4, 1024, 8, 64), 0.48),
                 ((4, 2048, 8, 64), 1.05), ((4, 384, 8, 128), 0.39), ((4, 768, 8, 128), 0.65),
                 ((1, 1024, 8, 64), 0.19), ((2, 1024, 8, 64), 0.30), ((8, 1024, 8, 64), 0.85)]


def flops(B, S, Hq, D, causal):
    f = 4.0 * B * Hq * S * S * D
    return f / 2 if causal else f


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return {k: float(p[k]) for k in ("hbm_gbs", "bf16_tflops", "bf16_tflops_sustained")}, "measured"
    except (OSError, KeyError, ValueError):
        return dict(FALLBACK_PEAKS), "fallback"


def load_traffic(config_name):
    """DRAM bytes per attention launch from the committed ncu summary, if any."""
    path = os.path.join(ROOT, "profiles", "attn_fwd_traffic.json")
    try:
        with open(path) as f:
            return json.load(f).get(config_name)
    except (OSError, ValueError):
        return None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 50 ms while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str):
        self.gpu_id = gpu_id
        self.proc = None
        self.lines = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", self.gpu_id, f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        rows, reasons = [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), float(parts[3])))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not rows:
            return None
        # "Under load": samples drawing at least 60 % of the highest power seen
        # (the sampler also runs a little before and after the timed region).
        p_max = max(r[2] for r in rows)
        loaded = [r for r in rows if r[2] >= 0.6 * p_max] or rows
        return {"sm_mhz": statistics.median(r[0] for r in loaded), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": sorted(reasons), "samples": len(rows), "samples_under_load": len(loaded),
                "power_w_max": p_max}


def make_inputs(cfg, device, seed):
    import torch

    B, S, Hq, Hkv, D, dt, causal, theta, amp, _ = cfg
    tdt = {"float16": torch.float16, "bfloat16": torch.bfloat16, "float32": torch.float32}[dt]
    g = torch.Generator(device=device).manual_seed(seed)
    q = (torch.randn((B, S, Hq, D), generator=g, device=device) * amp).to(tdt)
    k = (torch.randn((B, S, Hkv, D), generator=g, device=device) * amp).to(tdt)
    v = (torch.randn((B, S, Hkv, D), generator=g, device=device) * amp).to(tdt)
    return q, k, v


def scale_of(name, D):
    return 0.125 if name == "cfg1" else 1.0 / math.sqrt(D)


# ------------------------------------------------------------------ CPU baseline
def cpu_threads():
    """All host cores, also under torchrun (which sets OMP_NUM_THREADS=1)."""
    import torch

    torch.set_num_threads(os.cpu_count() or 1)
    return torch.get_num_threads()


def cpu_sample(cfg, budget_s=12.0, max_heads=64):
    """The reference's PyTorch CPU attention (a restatement of test.py:39-93
    attention_ref with the same torch ops, pinned by the golden fixtures; plus
    rotate-half RoPE) on whole (batch, head) slices of the workload until
    `budget_s` of CPU time. Returns (TFLOP/s, threads, seconds, description)."""
    import torch

    from oracle.torch_cpu_reference import attention_ref_torch

    B, S, Hq, Hkv, D, dt, causal, theta, amp, _ = cfg
    threads = cpu_threads()
    g = torch.Generator().manual_seed(0)
    heads, t_total = 0, 0.0
    while heads < max_heads and (t_total < budget_s or heads == 0):
        q, k, v = (torch.randn((1, S, 1, D), generator=g) * amp for _ in range(3))
        t0 = time.perf_counter()
        attention_ref_torch(q, k, v, causal=causal, softmax_scale=1 / math.sqrt(D), rope_theta=theta)
        t_total += time.perf_counter() - t0
        heads += 1
    f = flops(1, S, heads, D, causal)
    return (f / t_total / 1e12, threads, t_total,
            f"{heads} (batch, head) slices of S={S} D={D} ({t_total:.1f} s), fp32, "
            f"{threads} torch threads of os.cpu_count()={os.cpu_count()}")


def run_reference(args, cfg, rank, world):
    """--impl reference: the reference's PyTorch CPU attention on the host
    cores, one (batch, head) slice of the workload per step."""
    if rank != 0:
        return 0
    B, S, Hq, Hkv, D, dt, causal, theta, amp, desc = cfg
    times = []
    threads = None
    per_step_flops = flops(1, S, 1, D, causal)
    for i in range(args.warmup + args.steps):
        _, threads, t, _ = cpu_sample(cfg, budget_s=0.0, max_heads=1)
        if i >= args.warmup:
            times.append(t)
    ms = statistics.mean(times) * 1e3
    value = per_step_flops / (ms / 1e3) / 1e12
    sample = (f"one (batch, head) slice S={S} D={D} per step: PyTorch CPU restatement of test.py:39-93 "
              f"attention_ref (+ rotate-half RoPE), {threads} threads of os.cpu_count()={os.cpu_count()}")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": args.config + ": " + desc, "sample_per_step": f"one (batch, head) slice S={S} D={D}"},
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------ timing helpers
def timed(fa, step, steps, stream, flush=None):
    """Per-step device times (ms, CUDA events on `stream`) and the attention
    kernel's summed time and launch count over the steps. With `flush`, L2 is
    flushed before every step, outside the events."""
    import torch

    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    torch.cuda.synchronize()
    fa.kernel_timing_enable()
    for a, b in evs:
        if flush is not None:
            flush()
        a.record(stream)
        step()
        b.record(stream)
    torch.cuda.synchronize()
    kern_ms, kern_n = fa.kernel_timing_read()
    return [a.elapsed_time(b) for a, b in evs], kern_ms, kern_n


def make_flush(device):
    import torch

    buf = torch.empty(2 * L2_BYTES // 4, dtype=torch.float32, device=device)
    return lambda: buf.fill_(1.0)


# ------------------------------------------------------------------ fp32 check (bench-local)
def fp32_rows(q, k, v, causal, scale, theta, rows, head_block=8):
    """fp32 evaluation of rows [r0, r1) of every head on the GPU (TF32 off):
    RoPE tables in float64, scores, top-left causal mask, softmax, P @ V.
    An in-run parity check of the multi-GPU paths, outside every timed region."""
    import torch

    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        r0, r1 = rows
        B, Sq, Hq, D = q.shape
        Hk = k.shape[2]
        g = Hq // Hk
        kend = min(k.shape[1], r1) if causal else k.shape[1]
        qf, kf, vf = q[:, r0:r1].float(), k[:, :kend].float(), v[:, :kend].float()
        if theta:
            i = torch.arange(D // 2, dtype=torch.float64, device=q.device)
            inv = torch.pow(torch.tensor(float(theta), dtype=torch.float64, device=q.device), -2.0 * i / D)

            def rot(x, p0):
                pos = torch.arange(p0, p0 + x.shape[1], dtype=torch.float64, device=q.device)
                ang = pos[:, None] * inv[None, :]
                c, s = torch.cos(ang).float()[None, :, None, :], torch.sin(ang).float()[None, :, None, :]
                a, b = x[..., :D // 2], x[..., D // 2:]
                return torch.cat([a * c - b * s, a * s + b * c], dim=-1)

            qf, kf = rot(qf, r0), rot(kf, 0)
        out = torch.empty((B, r1 - r0, Hq, D), dtype=torch.float32, device=q.device)
        cols = torch.arange(kend, device=q.device)
        rws = torch.arange(r0, r1, device=q.device)
        for b in range(B):
            for h in range(Hq):
                s = (qf[b, :, h] @ kf[b, :, h // g].t()) * scale
                if causal:
                    s = s.masked_fill(cols[None, :] > rws[:, None], float("-inf"))
                out[b, :, h] = torch.softmax(s, dim=-1) @ vf[b, :, h // g]
        return out
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


# ------------------------------------------------------------------ N = 1 extras
def measure_configs(fa, device, steps, warmup, e2e_steps, skip):
    """Kernel / step / e2e TFLOP/s of every configuration but the headline."""
    import torch

    out_all = {}
    stream = torch.cuda.current_stream(device)
    flush = make_flush(device)
    for name, cfg in CONFIGS.items():
        if name in skip:
            continue
        B, S, Hq, Hkv, D, dt, causal, theta, amp, desc = cfg
        q, k, v = make_inputs(cfg, device, seed=1234)
        scale = scale_of(name, D)
        kw = {"rope_theta": theta} if theta else {}
        out = torch.empty_like(q)
        big = sum(x.numel() * x.element_size() for x in (q, k, v, out)) > L2_BYTES

        def step():
            fa.forward(q, k, v, softmax_scale=scale, is_causal=causal, out=out, **kw)

        for _ in range(warmup):
            step()
        n = steps if S < 65536 else max(3, steps // 4)
        per, kern_ms, kern_n = timed(fa, step, n, stream, flush=None if big else flush)
        f = flops(B, S, Hq, D, causal)
        rec = {"workload": desc, "step_tflops": f * n / (sum(per) / 1e3) / 1e12,
               "step_ms_median": statistics.median(per),
               "kernel_tflops": (f / (kern_ms / kern_n / 1e3) / 1e12) if kern_n else None,
               "kernel_launches_per_step": kern_n / n,
               "l2": "inputs > L2" if big else "L2 flushed before every step (2 x 126 MB write)"}
        if e2e_steps > 0:
            qh, kh, vh = (x.cpu().pin_memory() for x in (q, k, v))
            oh = torch.empty(out.shape, dtype=out.dtype).pin_memory()

            def e2e():
                fa.forward(qh, kh, vh, softmax_scale=scale, is_causal=causal, out=oh, **kw)

            e2e()
            ne = e2e_steps if S < 65536 else 2
            t0 = time.perf_counter()
            for _ in range(ne):
                e2e()
            dt_s = (time.perf_counter() - t0) / ne
            rec["e2e_tflops"] = f / dt_s / 1e12
            rec["e2e_ms"] = dt_s * 1e3
            del qh, kh, vh, oh
        out_all[name] = rec
        del q, k, v, out
        torch.cuda.empty_cache()
    return out_all


def readme_inputs(B, S, H, D):
    """The reference benchmark's inputs (test.py:518-521)."""
    import numpy as np

    np.random.seed(42)
    q = np.random.randn(B, S, H, D).astype(np.float16) * 0.02
    return q, q.copy(), q.copy(), 1.0 / np.sqrt(D)


def readme_shapes(fa, runs=100, warmup=20):
    """The reference's benchmark protocol (test.py:183-200: median wall time
    of `runs` calls after `warmup`, host copies included) on its published
    shapes through the NumPy API."""
    import numpy as np

    res = []
    for (B, S, H, D), metal_ms in README_SHAPES:
        q, k, v, scale = readme_inputs(B, S, H, D)
        for _ in range(warmup):
            fa.forward(q, k, v, softmax_scale=scale, is_causal=False)
        times = []
        for _ in range(runs):
            t0 = time.perf_counter()
            fa.forward(q, k, v, softmax_scale=scale, is_causal=False)
            times.append((time.perf_counter() - t0) * 1e3)
        ms = float(np.median(times))
        res.append({"shape": f"{B}x{S}x{H}x{D}", "ms_median": ms, "tflops": flops(B, S, H, D, False) / ms / 1e9,
                    "reference_metal_ms_published": metal_ms})
    return res


def readme_shapes_cpu(res, cpu_runs=5):
    """The PyTorch CPU attention on the same shapes (test.py:236-252, fewer
    runs), added to readme_shapes' records. Runs after every GPU and
    host-copy measurement: torch's CPU threads keep spinning after their
    work and would slow the library's copy workers."""
    import numpy as np
    import torch

    from oracle.torch_cpu_reference import attention_ref_torch

    threads = cpu_threads()
    for rec, ((B, S, H, D), _) in zip(res, README_SHAPES):
        q, _, _, scale = readme_inputs(B, S, H, D)
        qt = torch.from_numpy(q)
        attention_ref_torch(qt, qt, qt, causal=False, softmax_scale=scale)
        cpu_t = []
        for _ in range(cpu_runs):
            t0 = time.perf_counter()
            attention_ref_torch(qt, qt, qt, causal=False, softmax_scale=scale)
            cpu_t.append((time.perf_counter() - t0) * 1e3)
        cpu_ms = float(np.median(cpu_t))
        rec.update({"torch_cpu_ms_median": cpu_ms, "torch_cpu_threads": threads,
                    "speedup_vs_torch_cpu": cpu_ms / rec["ms_median"]})
    return res


def e2e_numpy(fa, cfg, steps=3):
    """The headline workload through the NumPy API with pageable arrays, the
    way the reference's callers pass data (test.py:191-197)."""
    import ml_dtypes
    import numpy as np
    import torch

    B, S, Hq, Hkv, D, dt, causal, theta, amp, _ = cfg
    npdt = {"bfloat16": ml_dtypes.bfloat16, "float16": np.float16, "float32": np.float32}[dt]
    q, k, v = make_inputs(cfg, torch.device("cuda", torch.cuda.current_device()), seed=1234)
    qn, kn, vn = (x.float().cpu().numpy().astype(npdt) for x in (q, k, v))
    del q, k, v
    kw = {"rope_theta": theta} if theta else {}
    # Warm-up: the first calls fill the pinned-buffer pool (the staging of
    # the inputs, plus two results: each call's result is allocated while
    # the previous one is still alive).
    for _ in range(3):
        o = fa.forward(qn, kn, vn, softmax_scale=1 / math.sqrt(D), is_causal=causal, **kw)
    t0 = time.perf_counter()
    for _ in range(steps):
        o = fa.forward(qn, kn, vn, softmax_scale=1 / math.sqrt(D), is_causal=causal, **kw)
    s = (time.perf_counter() - t0) / steps
    return {"value": flops(B, S, Hq, D, causal) / s / 1e12, "unit": "TFLOP/s", "ms_per_step": s * 1e3,
            "h2d_bytes_per_step": int(qn.nbytes + kn.nbytes + vn.nbytes), "d2h_bytes_per_step": int(o.nbytes),
            "api": "_flash_attn_metal.forward on pageable NumPy arrays (ml_dtypes.bfloat16)"}


# ------------------------------------------------------------------ N > 1 extras
def cfg5b_splits(fa, device, rank, world, dist, steps, warmup):
    """cfg5b over all ranks, split by query rows (K/V replicated, no merge)
    and by key ranges (partials stored into the row owners' staging over
    NVLink, one-element barrier, owner merge); each timed (max over ranks)
    and each rank's rows checked against an fp32 evaluation on its GPU."""
    import torch

    from flash_attn_metal_cpp_b200.multi_gpu import QShardAttention, SplitKVAttention

    cfg = CONFIGS["cfg5b"]
    B, S, Hq, Hkv, D, dt, causal, theta, amp, _ = cfg
    q, k, v = make_inputs(cfg, device, seed=4321)  # same seed on every rank: one problem
    scale = 1 / math.sqrt(D)
    stream = torch.cuda.current_stream(device)
    f_job = flops(B, S, Hq, D, causal)
    res = {}

    def max_over_ranks(x):
        t = torch.tensor([x], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # split_q
    qs = QShardAttention(S, rank, world, device)
    out = torch.empty_like(q)
    for _ in range(warmup):
        qs.forward(q, k, v, scale, causal, out, rope_theta=theta)
    dist.barrier()
    per, _, _ = timed(fa, lambda: qs.forward(q, k, v, scale, causal, out, rope_theta=theta), steps, stream)
    ms = max_over_ranks(sum(per) / steps)
    out32 = torch.empty(q.shape, dtype=torch.float32, device=device)
    qs.forward(q, k, v, scale, causal, out32, rope_theta=theta)
    errs = []
    for lo, hi in qs.ranges:
        for r0 in (lo, max(lo, hi - 128)):
            ref = fp32_rows(q, k, v, causal, scale, theta, (r0, r0 + 128))
            errs.append((out32[:, r0:r0 + 128] - ref).abs())
    e = torch.cat([x.flatten() for x in errs])
    mx, mean = max_over_ranks(float(e.max())), max_over_ranks(float(e.mean()))
    res["split_q"] = {"tflops": f_job / (ms / 1e3) / 1e12, "ms_per_step": ms, "max_abs": mx, "mean_abs": mean,
                      "checked_rows_per_rank": len(errs) * 128, "parity": mx <= 2e-3 and mean <= 2e-4,
                      "ranges_rank0": qs.ranges if rank == 0 else None}
    del out, out32

    # split_kv
    att = SplitKVAttention(B, S, S, Hq, Hkv, D, causal)
    try:
        blo, bhi = att.plan.owner_block(rank)
        out = torch.empty((B, bhi - blo, Hq, D), dtype=q.dtype, device=device)
        for _ in range(warmup):
            att.forward(q, k, v, scale, out=out, rope_theta=theta)
        dist.barrier()
        per, kern_ms, kern_n = timed(fa, lambda: att.forward(q, k, v, scale, out=out, rope_theta=theta), steps,
                                     stream)
        ms = max_over_ranks(sum(per) / steps)
        o32 = att.forward(q, k, v, scale, rope_theta=theta, out_dtype=torch.float32)
        torch.cuda.synchronize()
        errs = []
        if bhi > blo:
            for r0 in sorted({blo, blo + (bhi - blo) // 2 // 128 * 128, max(blo, bhi - 128)}):
                r1 = min(bhi, r0 + 128)
                ref = fp32_rows(q, k, v, causal, scale, theta, (r0, r1))
                errs.append((o32[:, r0 - blo:r1 - blo] - ref).abs())
        if errs:
            e = torch.cat([x.flatten() for x in errs])
            emax, emean = float(e.max()), float(e.mean())
        else:
            emax = emean = 0.0
        mx, mean = max_over_ranks(emax), max_over_ranks(emean)
        res["split_kv"] = {"tflops": f_job / (ms / 1e3) / 1e12, "ms_per_step": ms, "max_abs": mx, "mean_abs": mean,
                           "checked_rows_per_rank": sum(x.shape[1] for x in errs),
                           "parity": mx <= 2e-3 and mean <= 2e-4,
                           "kernel_ms_rank": kern_ms / max(kern_n, 1),
                           "key_ranges": att.plan.kv_ranges, "owner_rows": att.plan.owner_rows}
    finally:
        att.close()
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=sorted(CONFIGS), default="cfg4")
    ap.add_argument("--e2e-steps", type=int, default=5)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true",
                    help="headline only (no per-config table, README shapes, NumPy e2e, replicas or cfg5b splits)")
    ap.add_argument("--batch", type=int, default=None, help="override the batch size (profiling runs)")
    ap.add_argument("--split", choices=["kv", "q"], default="q",
                    help="how --config cfg5b is split over ranks: zig-zag query rows with K/V replicated (q, the "
                         "faster: no merge) or key ranges with partials merged by the row owners (kv)")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    cfg = CONFIGS[args.config]
    if args.batch is not None:
        cfg = (args.batch,) + cfg[1:]

    if args.impl == "reference":
        return run_reference(args, cfg, rank, world)

    import torch

    import flash_attn_metal_cpp_b200  # noqa: F401  (registers _flash_attn_metal)
    import _flash_attn_metal as fa
    from flash_attn_metal_cpp_b200 import sharding
    from flash_attn_metal_cpp_b200.multi_gpu import unit_forward

    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
    assert fa.initialize(), "CUDA initialisation failed"

    B, S, Hq, Hkv, D, dt, causal, theta, amp, desc = cfg
    scale = scale_of(args.config, D)
    split_cfg = args.config in SPLIT_KV and world > 1  # cfg5b: rows or keys over the ranks
    split_kv = split_cfg and args.split == "kv"
    units = None if split_cfg else sharding.unit_ranges(B, Hkv, world, rank)
    if not split_cfg and units is None:
        raise SystemExit(f"{world} ranks do not split {B} x {Hkv} (batch, KV-head) units into rectangles")
    # Every rank generates the same problem (same seed) and works on its share.
    q, k, v = make_inputs(cfg, device, seed=1234)
    kw = {"rope_theta": theta} if theta else {}
    att = qs = None
    if split_kv:
        from flash_attn_metal_cpp_b200.multi_gpu import SplitKVAttention

        att = SplitKVAttention(B, S, S, Hq, Hkv, D, causal)
        blo, bhi = att.plan.owner_block(rank)
        out = torch.empty((B, bhi - blo, Hq, D), dtype=q.dtype, device=device)
        share = att.plan.pair_work(rank) / max(1, sum(att.plan.pair_work(r) for r in range(world)))

        def step():
            att.forward(q, k, v, scale, out=out, **kw)
    elif split_cfg:
        from flash_attn_metal_cpp_b200.multi_gpu import QShardAttention

        qs = QShardAttention(S, rank, world, device)
        out = torch.empty((B, S, Hq, D), dtype=q.dtype, device=device)
        rows_work = sum((hi * (hi + 1) - lo * (lo + 1)) // 2 if causal else (hi - lo) * S for lo, hi in qs.ranges)
        share = rows_work / ((S * (S + 1)) // 2 if causal else S * S)

        def step():
            qs.forward(q, k, v, scale, causal, out, **kw)
    else:
        (b0, b1), (h0, h1) = units
        g = Hq // Hkv
        share = (b1 - b0) * (h1 - h0) / (B * Hkv)
        out = torch.empty((b1 - b0, S, (h1 - h0) * g, D), dtype=q.dtype, device=device)

        def step():
            unit_forward(q, k, v, rank, world, softmax_scale=scale, is_causal=causal, out=out, **kw)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    fa.check_status()

    props = torch.cuda.get_device_properties(device)
    sampler = ClockSampler(f"GPU-{props.uuid}" if getattr(props, "uuid", None) else str(local_rank))
    stream = torch.cuda.current_stream(device)
    # One event per step boundary: the first and last bracket the timed
    # region, the ones between give per-step times (median / p10 / p90).
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
    ev0, ev1 = evs[0], evs[-1]
    sampler.start()
    time.sleep(0.3)
    n_launch0 = fa.launch_count()
    fa.kernel_timing_enable()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    ev0.record(stream)
    for i in range(args.steps):
        step()
        evs[i + 1].record(stream)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    kern_ms, kern_launches = fa.kernel_timing_read()
    gpu_launches = fa.launch_count() - n_launch0
    clocks = sampler.stop()
    fa.check_status()
    elapsed_ms = ev0.elapsed_time(ev1)
    step_ms = sorted(evs[i].elapsed_time(evs[i + 1]) for i in range(args.steps))

    def pct(p_):
        return step_ms[min(len(step_ms) - 1, int(round(p_ * (len(step_ms) - 1))))]
    t = torch.tensor([elapsed_ms], dtype=torch.float64, device=device)
    if dist:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    max_ms = float(t.item())

    f_job = flops(B, S, Hq, D, causal)  # one problem over all ranks
    value = f_job * args.steps / (max_ms / 1e3) / 1e12
    ms_per_step = max_ms / args.steps

    # End to end through the public API with pinned host buffers: every step
    # copies this rank's inputs host->device, runs, and copies its output
    # device->host.
    e2e = None
    if args.e2e_steps > 0:
        if split_kv:
            # The query rows and the key range this rank's share reads in, its owned rows out.
            qlo, _ = att.plan.q_ranges[rank]
            klo, khi = att.plan.kv_ranges[rank]
            qh = q[:, qlo:].cpu().pin_memory()
            kh, vh = (x[:, klo:khi].cpu().pin_memory() for x in (k, v))
            oh = torch.empty(out.shape, dtype=out.dtype).pin_memory()
            h2d_rank = sum(x.numel() * x.element_size() for x in (qh, kh, vh))

            def e2e_step():
                q[:, qlo:].copy_(qh, non_blocking=True)
                k[:, klo:khi].copy_(kh, non_blocking=True)
                v[:, klo:khi].copy_(vh, non_blocking=True)
                att.forward(q, k, v, scale, out=out, **kw)
                oh.copy_(out, non_blocking=True)
                torch.cuda.current_stream(device).synchronize()
            d2h_rank = out.numel() * out.element_size()
        elif split_cfg:
            # Query rows of the rank's two chunks in, keys up to its last row in, its rows out.
            kv_hi = max(hi for _, hi in qs.ranges) if causal else S
            qhs = [q[:, lo:hi].cpu().pin_memory() for lo, hi in qs.ranges]
            kh, vh = (x[:, :kv_hi].cpu().pin_memory() for x in (k, v))
            ohs = [torch.empty(x.shape, dtype=out.dtype).pin_memory() for x in qhs]
            h2d_rank = sum(x.numel() * x.element_size() for x in qhs + [kh, vh])

            def e2e_step():
                for (lo, hi), x in zip(qs.ranges, qhs):
                    q[:, lo:hi].copy_(x, non_blocking=True)
                k[:, :kv_hi].copy_(kh, non_blocking=True)
                v[:, :kv_hi].copy_(vh, non_blocking=True)
                qs.forward(q, k, v, scale, causal, out, **kw)
                for (lo, hi), x in zip(qs.ranges, ohs):
                    x.copy_(out[:, lo:hi], non_blocking=True)
                torch.cuda.current_stream(device).synchronize()
            d2h_rank = sum(x.numel() * x.element_size() for x in ohs)
        else:
            # This rank's (batch, KV-head) shard as contiguous pinned host
            # tensors through the host-pointer path (copy in, run, copy out).
            (b0, b1), (h0, h1) = units
            g = Hq // Hkv
            qh = q[b0:b1, :, h0 * g:h1 * g].contiguous().cpu().pin_memory()
            kh, vh = (x[b0:b1, :, h0:h1].contiguous().cpu().pin_memory() for x in (k, v))
            oh = torch.empty(out.shape, dtype=out.dtype).pin_memory()
            h2d_rank = sum(x.numel() * x.element_size() for x in (qh, kh, vh))

            def e2e_step():
                fa.forward(qh, kh, vh, softmax_scale=scale, is_causal=causal, out=oh, **kw)
            d2h_rank = oh.numel() * oh.element_size()

        e2e_step()
        if dist:
            dist.barrier()
        t0 = time.perf_counter()
        for _ in range(args.e2e_steps):
            e2e_step()
        e2e_s = torch.tensor([(time.perf_counter() - t0) / args.e2e_steps], dtype=torch.float64, device=device)
        if dist:
            dist.all_reduce(e2e_s, op=dist.ReduceOp.MAX)
        h2d = torch.tensor([h2d_rank, d2h_rank], dtype=torch.float64, device=device)
        if dist:
            dist.all_reduce(h2d)
        e2e = {"value": f_job / float(e2e_s.item()) / 1e12, "unit": "TFLOP/s",
               "ms_per_step": float(e2e_s.item()) * 1e3,
               "h2d_bytes_per_step": int(h2d[0].item()), "d2h_bytes_per_step": int(h2d[1].item()),
               "api": "_flash_attn_metal.forward on pinned host torch tensors" if not split_cfg else
                      "pinned host copies + the split driver"}

    peaks, peak_kind = load_peaks()
    # Algorithmic bytes of this rank's share: Q, K, V read once and O written once.
    alg_bytes = (sum(x.numel() * x.element_size() for x in (q, k, v)) + B * S * Hq * D * q.element_size()) * share
    kern_avg_ms = kern_ms / max(kern_launches, 1)
    if split_cfg and not split_kv:
        # Two concurrent launches per step: time the pair by the step itself.
        kern_avg_ms = elapsed_ms / args.steps
    kern_ranks = torch.zeros(world, dtype=torch.float64, device=device)
    kern_ranks[rank] = kern_avg_ms
    if dist:
        dist.all_reduce(kern_ranks)
    # FLOPs of this rank's launches (its share of the problem).
    achieved = f_job * share / (kern_avg_ms / 1e3) / 1e12 if kern_launches else None
    long_region = max_ms > 1000.0
    peak = peaks["bf16_tflops_sustained"] if long_region else peaks["bf16_tflops"]
    # DRAM bytes of one full-size attention launch (ncu launch list, committed
    # profile), scaled to this rank's share.
    traffic = load_traffic(args.config)
    if traffic is not None:
        traffic = traffic * share
    roofline = {
        "bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
        "frac": (achieved / peak) if achieved else None, "traffic": traffic,
        "kernel": "attn_fwd_sm100 (tcgen05)", "kernel_ms_avg": kern_avg_ms,
        "kernel_ms_per_rank": [round(float(x), 4) for x in kern_ranks.tolist()],
        "peak_source": f"{peak_kind} {'sustained' if long_region else 'burst'} bf16 GEMM",
        "frac_of_datasheet_2250": (achieved / DATASHEET_BF16_TFLOPS) if achieved else None,
    }
    del q, k, v
    torch.cuda.empty_cache()

    extras = {}
    if not args.no_extras and not split_cfg and args.batch is None:
        if world > 1:
            # Weak scaling for comparison: every rank its own full problem.
            qr, kr, vr = make_inputs(cfg, device, seed=1234 + rank)
            outr = torch.empty_like(qr)

            def rstep():
                fa.forward(qr, kr, vr, softmax_scale=scale, is_causal=causal, out=outr, **kw)

            for _ in range(args.warmup):
                rstep()
            dist.barrier()
            per, _, _ = timed(fa, rstep, args.steps, stream)
            t = torch.tensor([sum(per)], dtype=torch.float64, device=device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            extras["replicas"] = {"value": f_job * world * args.steps / (float(t.item()) / 1e3) / 1e12,
                                  "unit": "TFLOP/s", "ms_per_step": float(t.item()) / args.steps,
                                  "scaling": "weak", "global_batch": B * world,
                                  "note": "every rank its own full problem (batch shard x{})".format(world)}
            del qr, kr, vr, outr
            torch.cuda.empty_cache()
            extras["cfg5b"] = cfg5b_splits(fa, device, rank, world, dist, args.steps, args.warmup)
        else:
            extras["configs"] = measure_configs(fa, device, args.steps, args.warmup, args.e2e_steps,
                                                skip={args.config})
            extras["readme_shapes"] = readme_shapes(fa)
            extras["e2e_numpy"] = e2e_numpy(fa, cfg)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        # CPU work last: torch's CPU threads keep spinning after it.
        if "readme_shapes" in extras:
            readme_shapes_cpu(extras["readme_shapes"])
        tflops, threads, secs, sample = cpu_sample(cfg)
        cpu = {"value": tflops, "unit": "TFLOP/s", "cores": threads, "kind": "port",
               "sample": "PyTorch CPU restatement of test.py:39-93 attention_ref (+ rotate-half RoPE) on " + sample}

    if rank == 0:
        if split_kv:
            parallelism = f"split-KV x{world} (key ranges {att.plan.kv_ranges}, owner rows {att.plan.owner_rows})"
        elif split_cfg:
            parallelism = f"zig-zag query rows x{world} (K/V replicated, no merge)"
        else:
            parallelism = f"(batch, KV-head) units x{world}: {B * Hkv // world} of {B * Hkv} per rank"
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None, "dtype": {"float32": "f32", "float16": "fp16", "bfloat16": "bf16"}[dt],
            "data": "synthetic (seeded N(0,1); one problem shared by all ranks)",
            "config": {
                "workload": args.config + ": " + desc, "global_batch": B,
                "seq_len": S, "heads_q": Hq, "heads_kv": Hkv, "head_dim": D, "causal": causal,
                "rope_theta": theta, "softmax_scale": scale, "parallelism": parallelism,
                "flops_per_step": f_job, "flops_per_step_per_gpu": f_job * share,
                "l2": "inputs + output {:.0f} MB > 126 MB L2 (no flush)".format(
                    (alg_bytes / max(share, 1e-9)) / 1e6),
                "mma_operands": "fp16 for bf16 inputs (converted in the staging pass), fp32 accumulate",
            },
            "pct_of_peak": {"measured_" + ("sustained" if long_region else "burst"): value / world / peak,
                            "datasheet_2250": value / world / DATASHEET_BF16_TFLOPS},
            "roofline": roofline,
            "step_ms_rank0": {"median": pct(0.5), "p10": pct(0.1), "p90": pct(0.9), "n": len(step_ms)},
            # Memory-side sanity check: algorithmic bytes (this rank's Q, K, V
            # read once, O written once) over the step time.
            "hbm": {"algorithmic_bytes_per_step_per_gpu": alg_bytes,
                    "achieved_gbs": alg_bytes / (ms_per_step / 1e3) / 1e9,
                    "peak_gbs": peaks["hbm_gbs"],
                    "frac": alg_bytes / (ms_per_step / 1e3) / 1e9 / peaks["hbm_gbs"]},
            "cpu_baseline": cpu,
            "e2e": e2e,
            "gpu_launches": gpu_launches,
            "clocks": clocks,
        }
        line.update(extras)
        print(json.dumps(line), flush=True)
    if att is not None:
        att.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
