#!/usr/bin/env python3
"""Benchmark of the B200 FlashAttention-2 forward (one JSON line on rank 0).

Workload (default): causal GQA forward, bf16, B=4 S=8192 Hq=32 Hkv=8 D=128,
rotate-half RoPE theta=5e5, seeded N(0,1) inputs resident in HBM. A step is
one `_flash_attn_metal.forward` call (RoPE/convert pre-pass + attention
kernel). With --gpus N (torchrun, one process per GPU) every rank runs its
own batch shard of that size (weak scaling, no collective on the data path);
value = FLOPs of all ranks / max-over-ranks device time. cfg5b (8 query
heads over one KV head) instead splits ONE problem across the ranks (strong
scaling): by default each rank computes zig-zag query-row chunks against the
replicated K/V (no merge); with --split kv each rank computes one key range,
its kernel epilogue stores the partials into the row owners' staging over
NVLink, and after a one-element NCCL barrier the owners merge.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config cfg4]
    python bench.py --impl reference ...   # the oracle port on the host cores

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

METRIC = "attn fwd TFLOP/s and % of B200 dense BF16 peak at 1/2/4/8 GPUs; ms/call"
DATASHEET_BF16_TFLOPS = 2250.0
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}

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
# Configs whose one problem is split across the ranks (strong scaling, --split).
SPLIT_KV = {"cfg5b"}


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
    """nvidia-smi clocks / throttle reasons sampled every 200 ms while running."""

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


def cpu_sample(cfg, budget_s=12.0, max_heads=64):
    """Oracle port (NumPy, all BLAS threads) on whole (batch, head) slices of
    the workload until `budget_s` of CPU time; returns (TFLOP/s, cores, sample)."""
    import numpy as np

    from oracle import attention_oracle as orc

    B, S, Hq, Hkv, D, dt, causal, theta, amp, _ = cfg
    # All host cores, also under torchrun (which sets OMP_NUM_THREADS=1).
    try:
        from threadpoolctl import threadpool_info, threadpool_limits

        threadpool_limits(limits=os.cpu_count())
        cores = max((i.get("num_threads", 1) for i in threadpool_info()), default=os.cpu_count())
    except Exception:  # pragma: no cover
        cores = os.cpu_count()
    rng = np.random.default_rng(0)
    heads, t_total = 0, 0.0
    cs = sn = None
    if theta:
        cs, sn = orc.rope_tables(S, D, theta)
    while heads < max_heads and (t_total < budget_s or heads == 0):
        q = (rng.standard_normal((1, S, 1, D), dtype=np.float32) * amp)
        k = (rng.standard_normal((1, S, 1, D), dtype=np.float32) * amp)
        v = (rng.standard_normal((1, S, 1, D), dtype=np.float32) * amp)
        t0 = time.perf_counter()
        if theta:
            q, k = orc.rotate_half_rope(q, cs, sn), orc.rotate_half_rope(k, cs, sn)
        orc.attention_ref(q, k, v, causal=causal, softmax_scale=1 / math.sqrt(D), q_block=1024)
        t_total += time.perf_counter() - t0
        heads += 1
    f = flops(1, S, heads, D, causal)
    return f / t_total / 1e12, cores, t_total, f"{heads} (batch, head) slices of S={S} D={D} ({t_total:.1f} s)"


def run_reference(args, cfg, rank, world):
    if rank != 0:
        return 0
    B, S, Hq, Hkv, D, dt, causal, theta, amp, desc = cfg
    times = []
    cores = None
    per_step_flops = flops(1, S, 1, D, causal)
    for i in range(args.warmup + args.steps):
        tflops, cores, t, sample = cpu_sample(cfg, budget_s=0.0, max_heads=1)
        if i >= args.warmup:
            times.append(t)
    ms = statistics.mean(times) * 1e3
    value = per_step_flops / (ms / 1e3) / 1e12
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": args.config + ": " + desc, "sample_per_step": f"one (batch, head) slice S={S} D={D}"},
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": cores, "kind": "port",
                         "sample": f"one (batch, head) slice of S={S}, D={D} per step, NumPy port of test.py:39-93"},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=sorted(CONFIGS), default="cfg4")
    ap.add_argument("--e2e-steps", type=int, default=5)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--batch", type=int, default=None, help="override the batch size (profiling runs)")
    ap.add_argument("--split", choices=["kv", "q"], default="q",
                    help="how cfg5b is split over ranks: zig-zag query rows with K/V replicated (q, the faster: "
                         "no merge) or key ranges with partials merged by the row owners (kv)")
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

    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
    assert fa.initialize(), "CUDA initialisation failed"

    B, S, Hq, Hkv, D, dt, causal, theta, amp, desc = cfg
    scale = 1.0 / math.sqrt(D) if args.config != "cfg1" else 0.125
    shared = args.config in SPLIT_KV and world > 1  # one problem over all ranks
    split_kv = shared and args.split == "kv"
    # Ranks sharing one problem use the same seed.
    q, k, v = make_inputs(cfg, device, seed=1234 + (0 if args.config in SPLIT_KV else rank))
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
    elif shared:
        from flash_attn_metal_cpp_b200.multi_gpu import QShardAttention

        qs = QShardAttention(S, rank, world, device)
        out = torch.empty((B, S, Hq, D), dtype=q.dtype, device=device)
        rows_work = sum((hi * (hi + 1) - lo * (lo + 1)) // 2 if causal else (hi - lo) * S for lo, hi in qs.ranges)
        share = rows_work / ((S * (S + 1)) // 2 if causal else S * S)

        def step():
            qs.forward(q, k, v, scale, causal, out, **kw)
    else:
        out = torch.empty((B, S, Hq, D), dtype=q.dtype, device=device)
        share = 1.0

        def step():
            fa.forward(q, k, v, softmax_scale=scale, is_causal=causal, out=out, **kw)

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
    t = torch.tensor([elapsed_ms], device=device, dtype=torch.float64)
    if dist:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    max_ms = float(t.item())

    f_step = flops(B, S, Hq, D, causal)
    f_job = f_step if shared else f_step * world  # shared: one problem over all ranks
    value = f_job * args.steps / (max_ms / 1e3) / 1e12
    ms_per_step = max_ms / args.steps

    # End to end through the public API with pinned host buffers: every step
    # copies Q/K/V host->device, runs, and copies O device->host.
    e2e = None
    if args.e2e_steps > 0:
        if split_kv:
            # Each rank copies in the query rows and the key range its share
            # reads, and copies out the rows it owns.
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
        elif shared:
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
        else:
            qh, kh, vh = (x.cpu().pin_memory() for x in (q, k, v))
            oh = torch.empty(out.shape, dtype=out.dtype).pin_memory()
            h2d_rank = sum(x.numel() * x.element_size() for x in (q, k, v))

            def e2e_step():
                fa.forward(qh, kh, vh, softmax_scale=scale, is_causal=causal, out=oh, **kw)

        e2e_step()
        if dist:
            dist.barrier()
        t0 = time.perf_counter()
        for _ in range(args.e2e_steps):
            e2e_step()
        e2e_s = torch.tensor([(time.perf_counter() - t0) / args.e2e_steps], dtype=torch.float64, device=device)
        if dist:
            dist.all_reduce(e2e_s, op=dist.ReduceOp.MAX)
        d2h_rank = sum(x.numel() * x.element_size() for x in ohs) if (shared and not split_kv) else \
            out.numel() * out.element_size()
        h2d = torch.tensor([h2d_rank, d2h_rank], dtype=torch.float64, device=device)
        if dist:
            dist.all_reduce(h2d)
        e2e = {"value": f_job / float(e2e_s.item()) / 1e12, "unit": "TFLOP/s",
               "ms_per_step": float(e2e_s.item()) * 1e3,
               "h2d_bytes_per_step": int(h2d[0].item()), "d2h_bytes_per_step": int(h2d[1].item())}

    peaks, peak_kind = load_peaks()
    alg_bytes = sum(x.numel() * x.element_size() for x in (q, k, v, out)) * (share if shared else 1.0)
    kern_avg_ms = kern_ms / max(kern_launches, 1)
    if shared and not split_kv:
        # Two concurrent launches per step: time the pair by the step itself.
        kern_avg_ms = elapsed_ms / args.steps
    kern_ranks = torch.zeros(world, dtype=torch.float64, device=device)
    kern_ranks[rank] = kern_avg_ms
    if dist:
        dist.all_reduce(kern_ranks)
    # FLOPs of this rank's launches (its share of the problem under split-KV).
    achieved = f_step * share / (kern_avg_ms / 1e3) / 1e12 if kern_launches else None
    long_region = max_ms > 1000.0
    peak = peaks["bf16_tflops_sustained"] if long_region else peaks["bf16_tflops"]
    traffic = load_traffic(args.config)
    roofline = {
        "bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
        "frac": (achieved / peak) if achieved else None, "traffic": traffic,
        "kernel": "attn_fwd_sm100 (tcgen05)", "kernel_ms_avg": kern_avg_ms,
        "kernel_ms_per_rank": [round(float(x), 4) for x in kern_ranks.tolist()],
        "peak_source": f"{peak_kind} {'sustained' if long_region else 'burst'} bf16 GEMM",
        "frac_of_datasheet_2250": (achieved / DATASHEET_BF16_TFLOPS) if achieved else None,
    }

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        tflops, cores, secs, sample = cpu_sample(cfg)
        cpu = {"value": tflops, "unit": "TFLOP/s", "cores": cores, "kind": "port",
               "sample": "NumPy port of test.py:39-93 attention_ref (+ rotate-half RoPE) on " + sample}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
            "scaling": "strong" if args.config in SPLIT_KV else "weak",
            "vs_baseline": None, "dtype": {"float32": "f32", "float16": "fp16", "bfloat16": "bf16"}[dt],
            "data": "synthetic (seeded N(0,1); one problem shared by all ranks)" if args.config in SPLIT_KV
                    else "synthetic (seeded N(0,1) per rank)",
            "config": {
                "workload": args.config + ": " + desc, "batch_per_gpu": None if shared else B,
                "global_batch": B if args.config in SPLIT_KV else B * world,
                "seq_len": S, "heads_q": Hq, "heads_kv": Hkv, "head_dim": D, "causal": causal,
                "rope_theta": theta, "softmax_scale": scale,
                "parallelism": (f"split-KV x{world} (key ranges {att.plan.kv_ranges}, owner rows "
                                f"{att.plan.owner_rows})") if split_kv else
                               (f"zig-zag query rows x{world} (K/V replicated, no merge)" if shared
                                else f"batch shard x{world}"),
                "flops_per_step_per_gpu": f_step * share if shared else f_step,
                "l2": "inputs + output {:.0f} MB > 126 MB L2 (no flush)".format(
                    sum(x.numel() * x.element_size() for x in (q, k, v, out)) / 1e6),
                "mma_operands": "fp16 for bf16 inputs (converted in the RoPE pre-pass), fp32 accumulate",
            },
            "pct_of_peak": {"measured_" + ("sustained" if long_region else "burst"): value / world / peak,
                            "datasheet_2250": value / world / DATASHEET_BF16_TFLOPS},
            "roofline": roofline,
            "step_ms_rank0": {"median": pct(0.5), "p10": pct(0.1), "p90": pct(0.9), "n": len(step_ms)},
            # Memory-side sanity check: algorithmic bytes (Q, K, V read once, O
            # written once, as the caller holds them) over the step time.
            "hbm": {"algorithmic_bytes_per_step_per_gpu": alg_bytes,
                    "achieved_gbs": alg_bytes / (ms_per_step / 1e3) / 1e9,
                    "peak_gbs": peaks["hbm_gbs"],
                    "frac": alg_bytes / (ms_per_step / 1e3) / 1e9 / peaks["hbm_gbs"]},
            "cpu_baseline": cpu,
            "e2e": e2e,
            "gpu_launches": gpu_launches,
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    if att is not None:
        att.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
