#!/usr/bin/env python
"""Attention-forward benchmark (bf16, head dim 128, non-causal) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c2] [--impl ours|reference]

One step = one forward over the configuration's inputs, already resident in
HBM. Each timed launch is bracketed by CUDA events on the launching stream;
L2 (126 MB) is flushed by a 256 MiB write between timed steps, outside the
events. value = algorithmic FLOPs (4*B*H*Sq*Sk*128) of all ranks / the
slowest rank's mean step time. With N > 1 ranks (torchrun, one per GPU):
configurations with several heads are sharded over heads (no exchange in the
data path; NCCL only gathers O afterwards when --validate is given); single
(batch, head) configurations run one replica per GPU.

`--impl reference` times the reference's own kernel (llm_fa.cu built from its
sources into oracle/_ref/) through its own `llm_fa_forward` on rank 0, one 2-D
launch per (batch, head), kernel durations from CUPTI (the reference launcher
allocates O and synchronises the device inside every call, so events on the
stream cannot bracket its kernel alone); when that module is absent it times
the reference's CPU oracle path (fp32 SDPA, validate.py:19-27) instead.
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

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "attn fwd TFLOP/s bf16 hd128 & % of tensor peak; µs vs llm_fa.cu/FA4 same box"
UNIT = "TFLOP/s"
# Reference's published TFLOP/s for the same shapes (ncu, SM clock locked
# at ~1.07 GHz, computed from the published microseconds of llm_fa.cu).
PUBLISHED_REF_TFLOPS = {"c2": 362.5, "c3": 810.6}
# DRAM bytes per launch (dram__bytes_read.sum + dram__bytes_write.sum) from the ncu capture
# summarised in profiles/; None until measured for that configuration.
PROFILED_TRAFFIC_BYTES: dict[str, float | None] = {
    "c2": 12.66e6,   # profiles/llm_fa_kernel_c2_ncu.md
    "c3": 142.6e6,   # profiles/llm_fa_kernel_c3_ncu.md
}
L2_FLUSH_BYTES = 256 << 20


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="c2", help="c1..c5 (BASELINE.json configs)")
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--validate", action="store_true", help="NCCL-gather O to rank 0 afterwards")
    ap.add_argument("--cpu-seconds", type=float, default=10.0, help="CPU baseline sample budget")
    ap.add_argument("--sweep", action="store_true",
                    help="time this kernel and the reference kernel on the reference's eight "
                         "published single-head shapes (one JSON line per shape)")
    return ap.parse_args()


# ------------------------------------------------------------------ environment
def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return json.loads(p.read_text())
        except Exception:
            pass
    return {}


class ClockSampler:
    """nvidia-smi samples (200 ms) of one GPU while the timed region runs.

    nvidia-smi writes its samples to a file (`-f`), read after the timed region: a
    Python thread reading a pipe would take the interpreter lock during the timed
    steps and delay their launches."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []
        self.path = None

    def start(self):
        import tempfile
        fd, self.path = tempfile.mkstemp(prefix="llmfa_clocks_", suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200", "-f", self.path],
                stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
        except (OSError, ValueError):
            self.proc = None

    def stop(self) -> dict | None:
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        try:
            with open(self.path) as f:
                self.lines = [ln.strip() for ln in f]
            os.unlink(self.path)
        except OSError:
            self.lines = []
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[0]))
                mx.append(float(parts[1]))
            except ValueError:
                continue
            for nm, val in zip(names, parts[4:8]):
                if val.lower() == "active":
                    reasons.add(nm)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------------ workload
def local_shard(cfg, world: int, rank: int):
    """Which part of the workload this rank runs: ('heads', h0, h1), ('batch', b0, b1) or
    ('replica',)."""
    if world == 1:
        return ("all",)
    if cfg.heads % world == 0:
        hs = cfg.heads // world
        return ("heads", rank * hs, (rank + 1) * hs)
    if cfg.batch % world == 0:
        bs = cfg.batch // world
        return ("batch", rank * bs, (rank + 1) * bs)
    return ("replica",)


def slice_inputs(q, k, v, shard):
    if shard[0] == "heads":
        return tuple(t[:, :, shard[1]:shard[2]].contiguous() for t in (q, k, v))
    if shard[0] == "batch":
        return tuple(t[shard[1]:shard[2]].contiguous() for t in (q, k, v))
    return q, k, v


def cpu_baseline(cfg, budget_s: float) -> dict:
    """The reference's oracle path (fp32 SDPA, validate.py:19-27) on host cores, on a
    seeded subset of query rows of one head (rows are independent)."""
    import torch

    from llm_fa_b200.workloads import make_inputs, sample_rows
    from oracle.sdpa_oracle import sdpa_fp32

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(cfg.seed)
    # one (batch, head) slice of the workload's shape, same distribution
    small = type(cfg)(cfg.name, 1, 1, cfg.seq_q, cfg.seq_k, cfg.seed, cfg.stress_rows)
    q, k, v = make_inputs(small) if cfg.seq_q * cfg.seq_k <= (1 << 34) else (
        torch.randn(1, cfg.seq_q, 1, 128, generator=g).bfloat16(),
        torch.randn(1, cfg.seq_k, 1, 128, generator=g).bfloat16(),
        torch.randn(1, cfg.seq_k, 1, 128, generator=g).bfloat16())
    rows = sample_rows(small, 64)
    sdpa_fp32(q, k, v, rows=rows)  # warm-up
    t0 = time.perf_counter()
    sdpa_fp32(q, k, v, rows=rows)
    t_one = max(time.perf_counter() - t0, 1e-4)
    n = int(min(cfg.seq_q, max(64, 64 * budget_s / 3.0 / t_one)))
    rows = sample_rows(small, n)
    reps, total = 0, 0.0
    while total < budget_s * 0.66 or reps < 1:
        t0 = time.perf_counter()
        sdpa_fp32(q, k, v, rows=rows)
        total += time.perf_counter() - t0
        reps += 1
        if reps >= 3:
            break
    t = total / reps
    flops = 4.0 * len(rows) * cfg.seq_k * 128
    return {"value": flops / t / 1e12, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"fp32 SDPA (torch CPU) on {len(rows)} seeded query rows x {cfg.seq_k} keys "
                      f"of one head, {reps} reps, {t:.2f} s/rep; TFLOP/s of that sample"}


# ------------------------------------------------------------------ our arm
def run_ours(args, cfg, world, rank, local):
    import torch
    import torch.distributed as dist

    from llm_fa_b200 import attention_forward, device_status, launch_plan
    from llm_fa_b200.workloads import make_inputs

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    shard = local_shard(cfg, world, rank)
    q_h, k_h, v_h = slice_inputs(*make_inputs(cfg), shard)
    B, Sq, H, _ = q_h.shape
    Sk = k_h.shape[1]
    flops_local = 4 * B * H * Sq * Sk * 128
    q, k, v = q_h.to(dev), k_h.to(dev), v_h.to(dev)
    plan = launch_plan(B, H, Sq, Sk)  # kernels per forward: attention (+ split-KV combine)
    o = torch.empty_like(q)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)

    def step():
        attention_forward(q, k, v, out=o)

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize(dev)
    st = device_status(dev)
    if st != 0:
        raise RuntimeError(f"device status {st:#x} after warm-up")
    if world > 1:
        dist.barrier()
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    # The GPU idled during the sleep and lowers its clocks meanwhile (the first step
    # after it measured ~2x slower): the warm-up steps run again right before timing.
    for _ in range(max(args.warmup, 3)):
        flush.zero_()
        step()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    # Each step's 256 MiB flush runs ~70 µs on the GPU, longer than the host needs to
    # queue the step's events and launches, so no event interval contains host time.
    for i in range(args.steps):
        flush.zero_()
        starts[i].record(stream)
        step()
        ends[i].record(stream)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    clocks = sampler.stop()
    times_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    mean_ms = statistics.fmean(times_ms)
    st = device_status(dev)
    if st != 0:
        raise RuntimeError(f"device status {st:#x} after timed steps")

    # end to end through the public API for host-resident data
    # (llm_fa_b200.host.HostAttention): every step copies its Q, K, V in from pinned host
    # memory and its O back; the copies of neighbouring steps overlap the compute.
    e2e = None
    if not args.no_e2e:
        from llm_fa_b200.host import HostAttention
        qp, kp, vp = (t.contiguous().pin_memory() for t in (q_h, k_h, v_h))
        op = torch.empty(qp.shape, dtype=qp.dtype).pin_memory()
        ha = HostAttention(dev, depth=2)
        for _ in range(max(args.warmup, 3)):
            ha.submit(qp, kp, vp, op)
        ha.synchronize()
        if world > 1:
            dist.barrier()
        e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e_start.record(ha.s_in)
        for i in range(args.steps):
            ha.submit(qp, kp, vp, op)
        e_end.record(ha.s_out)
        ha.synchronize()
        torch.cuda.synchronize(dev)
        e2e_ms = e_start.elapsed_time(e_end) / args.steps
        e2e = {"ms": e2e_ms, "h2d": sum(t.numel() * t.element_size() for t in (q_h, k_h, v_h)),
               "d2h": o.numel() * o.element_size()}

    # max over ranks
    if world > 1:
        t = torch.tensor([mean_ms, e2e["ms"] if e2e else 0.0], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        mean_ms_max, e2e_ms_max = float(t[0]), float(t[1])
        tot = torch.tensor([float(flops_local)], dtype=torch.float64, device=dev)
        dist.all_reduce(tot)
        flops_total = float(tot[0])
        if args.validate:
            gathered = [torch.empty_like(o) for _ in range(world)]
            dist.all_gather(gathered, o)
            if rank == 0:
                ok = all(torch.isfinite(g.float()).all().item() for g in gathered)
                print(f"# gathered O from {world} ranks over NCCL: finite={ok}", file=sys.stderr)
    else:
        mean_ms_max = mean_ms
        e2e_ms_max = e2e["ms"] if e2e else 0.0
        flops_total = float(flops_local)

    if rank != 0:
        return None
    peaks = measured_peaks()
    peak = peaks.get("bf16_tflops")
    peak_src = "measured burst (MEASURED_PEAKS.json bf16_tflops)" if peak else "fallback 1590"
    peak = float(peak) if peak else 1590.0
    achieved = flops_local / (mean_ms / 1e3) / 1e12  # this rank's kernel, per launch
    value = flops_total / (mean_ms_max / 1e3) / 1e12
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(mean_ms_max, 5),
        # this rank's spread of the step times behind the mean
        "ms_per_step_median": round(statistics.median(times_ms), 5),
        "ms_per_step_min": round(min(times_ms), 5),
        "higher_is_better": True,
        "scaling": "strong" if shard[0] in ("heads", "batch") else "weak",
        "vs_baseline": (round(value / world / PUBLISHED_REF_TFLOPS[cfg.name], 3)
                        if cfg.name in PUBLISHED_REF_TFLOPS else None),
        "dtype": "bf16", "data": "synthetic (seeded N(0,1) bf16 inputs, BASELINE.json shapes)",
        "config": {"workload": f"{cfg.name}: {cfg.describe()} non-causal, scale 1/sqrt(128)",
                   "global_batch": cfg.batch, "heads": cfg.heads, "seq_q": cfg.seq_q,
                   "seq_k": cfg.seq_k, "head_dim": 128,
                   "parallelism": {"all": "single GPU", "heads": f"heads sharded over {world} GPUs",
                                   "batch": f"batch sharded over {world} GPUs",
                                   "replica": f"{world} independent replicas"}[shard[0]],
                   "l2": "flushed between timed steps (256 MiB write, outside the events)"},
        "roofline": {"bound": "tensor", "achieved": round(achieved, 2), "peak": peak,
                     "unit": "TFLOP/s", "frac": round(achieved / peak, 4),
                     "peak_source": peak_src,
                     "traffic": PROFILED_TRAFFIC_BYTES.get(cfg.name),
                     "algorithmic_bytes": cfg.io_bytes},
        "gpu_launches": args.steps * plan["kernels"],
        "launch_plan": plan,
        "clocks": clocks,
    }
    if e2e is not None:
        line["e2e"] = {"value": round(flops_total / (e2e_ms_max / 1e3) / 1e12, 2), "unit": UNIT,
                       "h2d_bytes_per_step": e2e["h2d"], "d2h_bytes_per_step": e2e["d2h"],
                       "ms_per_step": round(e2e_ms_max, 4),
                       "pipeline_depth": 2,
                       "path": ("llm_fa_b200.host.HostAttention: pinned host Q/K/V in, O out, "
                                "every step; copies of neighbouring steps overlap compute; "
                                "device-timed over all steps / steps")}
        line["gpu_launches"] += args.steps * plan["kernels"]
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(cfg, args.cpu_seconds)
    return line


# ------------------------------------------------------------------ reference arm
def run_reference(args, cfg, world, rank, local):
    if rank != 0:
        return None
    line = {"metric": METRIC, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "higher_is_better": True, "impl": "reference",
            "dtype": "bf16", "data": "synthetic (seeded N(0,1) bf16 inputs, BASELINE.json shapes)",
            "vs_baseline": None}
    import torch
    mod = None
    try:
        from oracle.build_ref import load_module
        if torch.cuda.is_available():
            mod = load_module()
    except Exception as exc:  # fall back to the CPU oracle path
        print(f"# reference kernel unavailable ({exc}); timing the CPU oracle path",
              file=sys.stderr)
    cpu = cpu_baseline(cfg, args.cpu_seconds)
    if mod is None:
        line.update({"value": round(cpu["value"], 6), "scaling": "weak",
                     "ms_per_step": None, "cpu_baseline": cpu,
                     "config": {"workload": f"{cfg.name}: {cfg.describe()}",
                                "parallelism": "CPU, all host threads"},
                     "e2e": {"value": round(cpu["value"], 6), "unit": UNIT,
                             "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}})
        return line
    from torch.profiler import ProfilerActivity, profile

    from llm_fa_b200.workloads import make_inputs
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    q, k, v = make_inputs(cfg)
    # the reference takes 2-D (q,128)/(sk,128) contiguous tensors: one launch per (b, h)
    heads = [(b, h) for b in range(cfg.batch) for h in range(cfg.heads)]
    per_head = [(q[b, :, h].contiguous().to(dev), k[b, :, h].contiguous().to(dev),
                 v[b, :, h].contiguous().to(dev)) for b, h in heads]
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    for _ in range(max(args.warmup, 3)):
        for Q, K, V in per_head:
            mod.llm_fa_forward(Q, K, V)
    torch.cuda.synchronize()
    n_warm = max(args.warmup, 3)
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        # warm-up launches again inside the profiled region (the GPU may have lowered
        # its clocks while the profiler started); only the last steps' launches count
        for _ in range(n_warm + args.steps):
            flush.zero_()
            for Q, K, V in per_head:
                mod.llm_fa_forward(Q, K, V)
        torch.cuda.synchronize()
    kern = sorted((e for e in prof.events()
                   if "llm_fa_kernel" in e.name
                   and e.device_type == torch.autograd.DeviceType.CUDA),
                  key=lambda e: e.time_range.start)
    durs = [e.device_time_total for e in kern][n_warm * len(per_head):]
    total_us = sum(durs)
    step_ms = total_us / 1e3 / args.steps
    value = cfg.flops / (step_ms / 1e3) / 1e12
    line.update({
        "value": round(value, 2), "ms_per_step": round(step_ms, 5), "scaling": "weak",
        "config": {"workload": f"{cfg.name}: {cfg.describe()} non-causal",
                   "parallelism": "single GPU, one 2-D launch per (batch, head)",
                   "l2": "flushed between timed steps (256 MiB write)",
                   "timing": f"CUPTI kernel durations of {len(durs)} llm_fa_kernel launches"},
        "kernel_us_per_launch": round(total_us / max(len(durs), 1), 2),
        "gpu_launches": len(durs),
        # this run: the reference's own implementation of the path (its llm_fa.cu kernel,
        # compiled from the reference sources; it has no CPU implementation of the path)
        "cpu_baseline": {"value": round(value, 2), "unit": UNIT, "cores": 1, "kind": "reference",
                         "sample": (f"reference llm_fa_kernel (oracle/_ref), {args.steps} steps of "
                                    f"{len(heads)} launches, whole workload; launched from one "
                                    "host thread")},
        "cpu_oracle": cpu,  # the reference's CPU oracle path (fp32 SDPA), for context
        "e2e": {"value": round(value, 2), "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    })
    return line


# The reference's published single-head shapes (q, sk), README.md:58-65 of the reference.
SWEEP_SHAPES = [(q, sk) for q in (16384, 32768) for sk in (16384, 32768, 65536, 131072)]


def run_sweep(args) -> None:
    """This kernel and the reference's llm_fa.cu kernel (oracle/_ref) on the same GPU, on
    the reference's published shapes: CUDA events around each call, a 256 MiB L2 flush
    before every call, median of --steps calls after --warmup; also the largest
    difference between the two outputs."""
    import statistics

    import torch

    from llm_fa_b200 import attention_forward, device_status
    from oracle.build_ref import load_module
    mod = load_module()
    dev = torch.device("cuda", 0)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    gen = torch.Generator(device="cpu").manual_seed(0)

    def median_us(fn):
        ts = []
        for i in range(args.warmup + args.steps):
            torch.cuda._sleep(200000)  # the host queues the call before the GPU reaches it
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            torch.cuda.synchronize()
            if i >= args.warmup:
                ts.append(e0.elapsed_time(e1) * 1e3)
        return statistics.median(ts)

    for q_len, sk in SWEEP_SHAPES:
        Q, K, V = (torch.randn(n, 128, generator=gen).bfloat16().to(dev)
                   for n in (q_len, sk, sk))
        O = torch.empty_like(Q)
        t_ours = median_us(lambda: attention_forward(Q, K, V, out=O))
        t_ref = median_us(lambda: mod.llm_fa_forward(Q, K, V))
        diff = (O.float() - mod.llm_fa_forward(Q, K, V)[0].float()).abs().max().item()
        flops = 4 * q_len * sk * 128
        print(json.dumps({"q": q_len, "sk": sk, "ours_us": round(t_ours, 1),
                          "reference_us": round(t_ref, 1),
                          "speedup": round(t_ref / t_ours, 3),
                          "ours_tflops": round(flops / t_ours / 1e6, 1),
                          "reference_tflops": round(flops / t_ref / 1e6, 1),
                          "max_abs_diff_vs_reference": diff}), flush=True)
    if device_status() != 0:
        raise RuntimeError(f"device status {device_status()}")


def main():
    args = parse_args()
    if args.sweep:
        run_sweep(args)
        return
    world, rank, local = dist_env()
    if world != args.gpus:
        print(f"# note: --gpus {args.gpus} but WORLD_SIZE={world}; using WORLD_SIZE",
              file=sys.stderr)
    from llm_fa_b200.workloads import CONFIGS
    cfg = CONFIGS[args.config]
    if args.impl == "reference":
        line = run_reference(args, cfg, world, rank, local)
        if line is not None:
            print(json.dumps(line), flush=True)
        return
    import torch.distributed as dist
    if world > 1:
        import torch
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    try:
        line = run_ours(args, cfg, world, rank, local)
    finally:
        if world > 1:
            dist.destroy_process_group()
    if line is not None:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
