#!/usr/bin/env python
"""Attention-forward benchmark (bf16, head dim 128, non-causal) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c3] [--impl ours|reference]

One step = one forward over the configuration's inputs, already resident in
HBM. Each timed launch is bracketed by CUDA events on the launching stream;
L2 (126 MB) is flushed by a 256 MiB write between timed steps, outside the
events. value = algorithmic FLOPs (4*B*H*Sq*Sk*128) of all ranks / the
slowest rank's mean step time.

With N > 1 ranks (torchrun, one per GPU, NCCL) every rank runs an
exchange-free shard of the configuration: its heads when the head count
divides by N, else its batch entries, else a contiguous block of query rows
(rows of one head are independent; every rank holds all of K and V), else a
replica. The data path has no collective; NCCL only takes the max of the
ranks' times and, with --validate, gathers O afterwards.

`--impl reference` times the reference's own kernel (llm_fa.cu built from its
sources into oracle/_ref/) through its own `llm_fa_forward`, one 2-D launch per
(batch, head), on every rank with the same shard as this arm; kernel durations
come from CUPTI (the reference launcher allocates O and synchronises the
device inside every call, so stream events cannot bracket its kernel alone).
Its `e2e` takes the same host-data path as this arm's: pinned Q/K/V copied in,
the call, O copied back, every step. When that module is absent it times the
reference's CPU oracle path (fp32 SDPA, validate.py:19-27) instead.

On one GPU this arm's line also carries `same_box_library`: flashinfer's CUTLASS
Blackwell FMHA (baseline/library_fmha.py, prebuilt offline) on the same inputs,
timed the same way after this arm (FA4 itself is not installed in this image),
or why it is unavailable.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import time
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

from llm_fa_b200.gpuclocks import ClockSampler  # noqa: E402

METRIC = "attn fwd TFLOP/s bf16 hd128 & % of tensor peak; µs vs llm_fa.cu/FA4 same box"
UNIT = "TFLOP/s"
DATA = "synthetic (seeded N(0,1) bf16 inputs at the configuration's shapes, drawn on the CPU)"
# The reference's published TFLOP/s for two of the configurations, computed from its
# published kernel microseconds (llm_fa.cu at 16384^2 and 32768x131072), which were measured
# under ncu with the SM clock locked near 1.07 GHz: not comparable with CUDA-event timings
# at the default clock, so they are reported beside the line and vs_baseline stays null.
PUBLISHED_REF_TFLOPS = {"c2": 362.5, "c3": 810.6}
# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one launch of the attention
# kernel at this configuration, from an ncu capture of the current kernel: a profile-time
# figure (ncu replays each launch with cold caches, and O's writes can stay in L2 when the
# kernel ends), not a measurement of the timed steps.
PROFILED_TRAFFIC_BYTES: dict[str, float | None] = {
    "c2": 12.66e6,
    "c3": 160.3e6,
    "c4": 1055.4e6,
}
L2_FLUSH_BYTES = 256 << 20


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="c3", help="c1..c5 (llm_fa_b200.workloads.CONFIGS)")
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--validate", action="store_true", help="NCCL-gather O to rank 0 afterwards")
    ap.add_argument("--cpu-seconds", type=float, default=10.0, help="CPU baseline sample budget")
    ap.add_argument("--heads", type=int, default=None,
                    help="run only the first N heads of the configuration (a smaller case of the "
                         "same kernel, for profiling; the line's config says so)")
    ap.add_argument("--sweep", action="store_true",
                    help="time this kernel and the reference kernel on the reference's published "
                         "single-head shapes and on multi-wave ones (one JSON line per shape)")
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


# ------------------------------------------------------------------ workload
def local_shard(cfg, world: int, rank: int):
    """This rank's exchange-free part of the workload: ('all',), ('heads', h0, h1),
    ('batch', b0, b1), ('rows', s0, s1) (query rows; K and V whole) or ('replica',)."""
    if world == 1:
        return ("all",)
    if cfg.heads % world == 0:
        hs = cfg.heads // world
        return ("heads", rank * hs, (rank + 1) * hs)
    if cfg.batch % world == 0:
        bs = cfg.batch // world
        return ("batch", rank * bs, (rank + 1) * bs)
    if cfg.seq_q % (512 * world) == 0:  # whole 512-row query blocks per rank
        rs = cfg.seq_q // world
        return ("rows", rank * rs, (rank + 1) * rs)
    return ("replica",)


def slice_inputs(q, k, v, shard):
    if shard[0] == "heads":
        return tuple(t[:, :, shard[1]:shard[2]].contiguous() for t in (q, k, v))
    if shard[0] == "batch":
        return tuple(t[shard[1]:shard[2]].contiguous() for t in (q, k, v))
    if shard[0] == "rows":
        return q[:, shard[1]:shard[2]].contiguous(), k, v
    return q, k, v


def parallelism(shard, world: int) -> str:
    return {"all": "single GPU", "heads": f"heads sharded over {world} GPUs",
            "batch": f"batch sharded over {world} GPUs",
            "rows": f"query rows sharded over {world} GPUs (K/V on every GPU)",
            "replica": f"{world} independent replicas"}[shard[0]]


def config_dict(cfg, shard, world: int) -> dict:
    """The `config` object of both arms' lines (identical for the same run)."""
    return {"workload": f"{cfg.name}: {cfg.describe()} non-causal, scale 1/sqrt(128)",
            "global_batch": cfg.batch, "heads": cfg.heads, "seq_q": cfg.seq_q,
            "seq_k": cfg.seq_k, "head_dim": 128, "parallelism": parallelism(shard, world),
            "l2": "flushed between timed steps (256 MiB write, outside the timed kernels)"}


def cpu_baseline(cfg, budget_s: float) -> dict:
    """The reference's oracle path (fp32 SDPA, validate.py:19-27) on all host cores, on a
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
            "sample": f"fp32 SDPA (torch CPU, the reference's oracle path) on {len(rows)} seeded "
                      f"query rows x {cfg.seq_k} keys of one head, {reps} reps, {t:.2f} s/rep; "
                      "TFLOP/s of that sample"}


def copy_bandwidth(host_in, host_out, dev) -> dict:
    """Pinned-memory copy rates of this box for the step's own buffers: all inputs
    host-to-device, then the output device-to-host, each alone on one stream (best of 3,
    CUDA events). These bound a host-data step from below."""
    import torch
    dev_in = [torch.empty(t.shape, dtype=t.dtype, device=dev) for t in host_in]
    dev_out = torch.empty(host_out.shape, dtype=host_out.dtype, device=dev)
    n_in = sum(t.numel() * t.element_size() for t in host_in)
    n_out = host_out.numel() * host_out.element_size()
    best_in, best_out = float("inf"), float("inf")
    for _ in range(3):
        e = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        e[0].record()
        for d, h in zip(dev_in, host_in):
            d.copy_(h, non_blocking=True)
        e[1].record()
        host_out.copy_(dev_out, non_blocking=True)
        e[2].record()
        torch.cuda.synchronize(dev)
        best_in = min(best_in, e[0].elapsed_time(e[1]))
        best_out = min(best_out, e[1].elapsed_time(e[2]))
    return {"h2d_gbs": round(n_in / best_in / 1e6, 2), "d2h_gbs": round(n_out / best_out / 1e6, 2),
            "h2d_ms": best_in, "d2h_ms": best_out}


def max_over_ranks(values: list[float], dev) -> list[float]:
    import torch
    import torch.distributed as dist
    t = torch.tensor(values, dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(x) for x in t]


def gather_floats(value: float, dev) -> list[float]:
    import torch
    import torch.distributed as dist
    t = torch.tensor([value], dtype=torch.float64, device=dev)
    parts = [torch.empty_like(t) for _ in range(dist.get_world_size())]
    dist.all_gather(parts, t)
    return [float(p[0]) for p in parts]


def time_library(q, k, v, ours_out, flops: int, args, flush, ours_ms: float) -> dict:
    """flashinfer's CUTLASS Blackwell FMHA (baseline/library_fmha.py) on the same inputs and
    GPU, timed like this arm (warm-up, L2 flush before every call, CUDA events): a
    same-box library comparison beside the line, not part of `value`."""
    import torch
    try:
        from baseline.library_fmha import LibraryFMHA
        fmha = LibraryFMHA(q, k, v, 1.0 / 128 ** 0.5)
    except Exception as e:  # not built, or flashinfer missing: say so
        return {"unavailable": f"{type(e).__name__}: {e}"[:240]}
    for _ in range(max(args.warmup, 3)):
        flush.zero_()
        fmha()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    for i in range(args.steps):
        flush.zero_()
        starts[i].record()
        fmha()
        ends[i].record()
    torch.cuda.synchronize()
    ms = statistics.fmean(s.elapsed_time(e) for s, e in zip(starts, ends))
    diff = (fmha.out.float() - ours_out.float()).abs().max().item()
    return {"impl": fmha.version, "value": round(flops / (ms / 1e3) / 1e12, 2), "unit": UNIT,
            "ms_per_step": round(ms, 5), "speedup_of_this_arm": round(ms / ours_ms, 3),
            "max_abs_diff_vs_this_arm": diff,
            "note": "FA4 (flash_attn.cute) is not installed in this image; this is the "
                    "tcgen05 attention kernel that is, timed after this arm"}


def clocks_from_samplers(*clocks):
    got = [c for c in clocks if c]
    return got[0] if got else None


# ------------------------------------------------------------------ our arm
def run_ours(args, cfg, world, rank, local):
    import torch
    import torch.distributed as dist

    from llm_fa_b200 import attention_forward, build_info, device_status, launch_plan
    from llm_fa_b200.workloads import make_inputs

    info = build_info()
    if info["ablation"] != 0:
        raise RuntimeError(f"library built with ablation switch {info['ablation_name']!r}: "
                           "its output is not attention; it is not timed as the product")
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
        bw = copy_bandwidth([qp, kp, vp], op, dev)
        ha = HostAttention(dev, depth=2)
        for _ in range(max(args.warmup, 3)):
            ha.submit(qp, kp, vp, op)
        ha.synchronize()
        if world > 1:
            dist.barrier()
        e2e_sampler = ClockSampler(local)
        e2e_sampler.start()
        e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e_start.record(ha.s_in)
        for i in range(args.steps):
            ha.submit(qp, kp, vp, op)
        e_end.record(ha.s_out)
        ha.synchronize()
        torch.cuda.synchronize(dev)
        e2e_ms = e_start.elapsed_time(e_end) / args.steps
        e2e = {"ms": e2e_ms, "h2d": sum(t.numel() * t.element_size() for t in (q_h, k_h, v_h)),
               "d2h": o.numel() * o.element_size(), "bw": bw, "clocks": e2e_sampler.stop()}

    # max over ranks
    if world > 1:
        mean_ms_max, e2e_ms_max = max_over_ranks([mean_ms, e2e["ms"] if e2e else 0.0], dev)
        per_rank_ms = gather_floats(mean_ms, dev)
        flops_total = float(flops_local) * world if shard[0] != "all" else float(flops_local)
        if args.validate:
            gathered = [torch.empty_like(o) for _ in range(world)]
            dist.all_gather(gathered, o)
            if rank == 0:
                ok = all(torch.isfinite(g.float()).all().item() for g in gathered)
                print(f"# gathered O from {world} ranks over NCCL: finite={ok}", file=sys.stderr)
    else:
        mean_ms_max = mean_ms
        e2e_ms_max = e2e["ms"] if e2e else 0.0
        per_rank_ms = [mean_ms]
        flops_total = float(flops_local)

    if rank != 0:
        return None
    peaks = measured_peaks()
    peak = peaks.get("bf16_tflops")
    peak_src = "measured burst (MEASURED_PEAKS.json bf16_tflops)" if peak else "fallback 1590"
    peak = float(peak) if peak else 1590.0
    peak_sus = float(peaks.get("bf16_tflops_sustained") or 1400.0)
    achieved = flops_local / (mean_ms / 1e3) / 1e12  # this rank's kernels, per forward
    value = flops_total / (mean_ms_max / 1e3) / 1e12
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(mean_ms_max, 5),
        # this rank's spread of the step times behind the mean
        "ms_per_step_median": round(statistics.median(times_ms), 5),
        "ms_per_step_min": round(min(times_ms), 5),
        "higher_is_better": True,
        "scaling": "strong" if shard[0] in ("heads", "batch", "rows") else "weak",
        "vs_baseline": None,
        "dtype": "bf16", "data": DATA,
        "config": config_dict(cfg, shard, world),
        "roofline": {"bound": "tensor", "achieved": round(achieved, 2), "peak": peak,
                     "unit": "TFLOP/s", "frac": round(achieved / peak, 4),
                     "peak_source": peak_src,
                     "peak_sustained": peak_sus,
                     "frac_of_sustained": round(achieved / peak_sus, 4),
                     "traffic": PROFILED_TRAFFIC_BYTES.get(cfg.name) if shard[0] == "all" else None,
                     "traffic_source": ("ncu dram__bytes_read.sum + dram__bytes_write.sum of one "
                                        "attention-kernel launch at this configuration (profile "
                                        "time, cold caches; O writes may stay in L2)"),
                     "algorithmic_bytes": 2 * 128 * B * H * (2 * Sq + 2 * Sk)},
        "gpu_launches": args.steps * plan["kernels"],
        "launch_plan": plan,
        "clocks": clocks,
    }
    if world > 1:
        line["per_rank_ms"] = [round(x, 5) for x in per_rank_ms]
    if cfg.name in PUBLISHED_REF_TFLOPS:
        line["published_reference"] = {
            "value": PUBLISHED_REF_TFLOPS[cfg.name], "unit": UNIT,
            "conditions": "reference's published llm_fa.cu time: ncu, SM clock locked near "
                          "1.07 GHz; not comparable with this line (CUDA events, default "
                          "clocks); the same-box reference arm is the comparison"}
    if e2e is not None:
        e2e_value = flops_total / (e2e_ms_max / 1e3) / 1e12
        bound_ms = max(e2e["bw"]["h2d_ms"], e2e["bw"]["d2h_ms"], mean_ms)
        line["e2e"] = {"value": round(e2e_value, 2), "unit": UNIT,
                       "h2d_bytes_per_step": e2e["h2d"], "d2h_bytes_per_step": e2e["d2h"],
                       "ms_per_step": round(e2e_ms_max, 4),
                       "pipeline_depth": 2,
                       "path": ("llm_fa_b200.host.HostAttention: pinned host Q/K/V in, O out, "
                                "every step; copies of neighbouring steps overlap compute; "
                                "device-timed over all steps / steps"),
                       # the step can go no faster than its slowest stage: all inputs in at the
                       # box's pinned copy rate, the output out, or the kernels
                       "copy_roofline": {"h2d_gbs": e2e["bw"]["h2d_gbs"],
                                         "d2h_gbs": e2e["bw"]["d2h_gbs"],
                                         "bound_ms": round(bound_ms, 4),
                                         "frac": round(bound_ms / e2e_ms_max, 4)},
                       # copies and kernels back to back, with no idle gap: the clocks the
                       # kernels ran at (under the power cap they can sit below the timed
                       # steps' clocks, which `bound_ms` assumes)
                       "clocks": e2e["clocks"]}
        line["gpu_launches"] += args.steps * plan["kernels"]
    if world == 1:
        line["same_box_library"] = time_library(q, k, v, o, flops_local, args, flush, mean_ms)
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(cfg, args.cpu_seconds)
    return line


# ------------------------------------------------------------------ reference arm
def run_reference(args, cfg, world, rank, local):
    import torch
    line = {"metric": METRIC, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "higher_is_better": True, "impl": "reference",
            "dtype": "bf16", "data": DATA, "vs_baseline": None}
    mod = None
    try:
        from oracle.build_ref import load_module
        if torch.cuda.is_available():
            mod = load_module()
    except Exception as exc:  # fall back to the CPU oracle path
        print(f"# reference kernel unavailable ({exc}); timing the CPU oracle path",
              file=sys.stderr)
    if mod is None:
        if rank != 0:
            return None
        cpu = cpu_baseline(cfg, args.cpu_seconds)
        line.update({"value": round(cpu["value"], 6), "scaling": "weak",
                     "ms_per_step": None, "cpu_baseline": cpu,
                     "config": dict(config_dict(cfg, ("all",), 1),
                                    parallelism="CPU, all host threads"),
                     "e2e": {"value": round(cpu["value"], 6), "unit": UNIT,
                             "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}})
        return line
    from torch.profiler import ProfilerActivity, profile

    from llm_fa_b200.workloads import make_inputs
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    shard = local_shard(cfg, world, rank)
    q, k, v = slice_inputs(*make_inputs(cfg), shard)
    B, Sq, H, _ = q.shape
    Sk = k.shape[1]
    flops_local = 4 * B * H * Sq * Sk * 128
    # the reference takes 2-D (q,128)/(sk,128) contiguous tensors: one launch per (b, h)
    heads = [(b, h) for b in range(B) for h in range(H)]
    per_head_host = [(q[b, :, h].contiguous(), k[b, :, h].contiguous(), v[b, :, h].contiguous())
                     for b, h in heads]
    per_head = [tuple(t.to(dev) for t in x) for x in per_head_host]
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    for _ in range(max(args.warmup, 3)):
        for Q, K, V in per_head:
            mod.llm_fa_forward(Q, K, V)
    torch.cuda.synchronize()
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    n_warm = max(args.warmup, 3)
    sampler = ClockSampler(local)
    sampler.start()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        # warm-up launches again inside the profiled region (the GPU may have lowered
        # its clocks while the profiler started); only the last steps' launches count
        for _ in range(n_warm + args.steps):
            flush.zero_()
            for Q, K, V in per_head:
                mod.llm_fa_forward(Q, K, V)
        torch.cuda.synchronize()
    clocks = sampler.stop()
    kern = sorted((e for e in prof.events()
                   if "llm_fa_kernel" in e.name
                   and e.device_type == torch.autograd.DeviceType.CUDA),
                  key=lambda e: e.time_range.start)
    durs = [e.device_time_total for e in kern][n_warm * len(per_head):]
    step_ms = sum(durs) / 1e3 / args.steps

    # end to end, the host-data path a caller of the reference takes: per step, copy each
    # head's Q, K, V in from pinned host memory, call llm_fa_forward (it allocates O and
    # synchronises the device), copy O back to pinned host memory; CUDA events on the
    # stream all of it runs on (the legacy default stream)
    e2e = None
    if not args.no_e2e:
        pinned = [tuple(t.pin_memory() for t in x) for x in per_head_host]
        o_pinned = [torch.empty(x[0].shape, dtype=torch.bfloat16).pin_memory() for x in pinned]
        dev_in = [tuple(torch.empty_like(t, device=dev) for t in x) for x in pinned]

        def host_step():
            for (qh, kh, vh), (qd, kd, vd), oh in zip(pinned, dev_in, o_pinned):
                qd.copy_(qh, non_blocking=True)
                kd.copy_(kh, non_blocking=True)
                vd.copy_(vh, non_blocking=True)
                oh.copy_(mod.llm_fa_forward(qd, kd, vd)[0], non_blocking=True)

        for _ in range(max(args.warmup, 3)):
            host_step()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            host_step()
        e1.record()
        torch.cuda.synchronize()
        e2e = {"ms": e0.elapsed_time(e1) / args.steps,
               "h2d": sum(t.numel() * t.element_size() for x in pinned for t in x),
               "d2h": sum(t.numel() * t.element_size() for t in o_pinned)}

    if world > 1:
        step_ms_max, e2e_ms_max = max_over_ranks([step_ms, e2e["ms"] if e2e else 0.0], dev)
        per_rank_ms = gather_floats(step_ms, dev)
        flops_total = float(flops_local) * world
    else:
        step_ms_max, e2e_ms_max, per_rank_ms = step_ms, (e2e["ms"] if e2e else 0.0), [step_ms]
        flops_total = float(flops_local)
    if rank != 0:
        return None
    value = flops_total / (step_ms_max / 1e3) / 1e12
    line.update({
        "value": round(value, 2), "ms_per_step": round(step_ms_max, 5),
        "scaling": "strong" if shard[0] in ("heads", "batch", "rows") else "weak",
        "config": config_dict(cfg, shard, world),
        "reference_kernel": {
            "value": round(value, 2), "unit": UNIT,
            "kernel_us_per_launch": round(sum(durs) / max(len(durs), 1), 2),
            "launches_per_step": len(heads),
            "timing": (f"CUPTI kernel durations of {len(durs)} llm_fa_kernel launches "
                       "(oracle/_ref: the reference's llm_fa.cu built from its sources), one 2-D "
                       "launch per (batch, head)")},
        "gpu_launches": len(durs),
        "clocks": clocks,
    })
    if world > 1:
        line["per_rank_ms"] = [round(x, 5) for x in per_rank_ms]
    if e2e is not None:
        line["e2e"] = {"value": round(flops_total / (e2e_ms_max / 1e3) / 1e12, 2), "unit": UNIT,
                       "h2d_bytes_per_step": e2e["h2d"], "d2h_bytes_per_step": e2e["d2h"],
                       "ms_per_step": round(e2e_ms_max, 4),
                       "path": ("reference llm_fa_forward per (batch, head): pinned host Q/K/V "
                                "copied in, the call (allocates O, synchronises the device), O "
                                "copied out, every step; CUDA events around all steps")}
    if not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(cfg, args.cpu_seconds)
    return line


# The reference's published single-head shapes (q, sk) (its README's latency table), and
# multi-wave ones (q > 32768: the reference launches more 512-row clusters than fit at once).
SWEEP_SHAPES = [(q, sk) for q in (16384, 32768) for sk in (16384, 32768, 65536, 131072)] + [
    (65536, 16384), (65536, 131072), (131072, 32768)] + [
    # 60 and 74 query blocks: the reference's grid at 120 and 148 SMs
    (30720, 131072), (37888, 131072)]


def run_sweep(args) -> None:
    """This kernel and the reference's llm_fa.cu kernel (oracle/_ref) on the same GPU, on
    the sweep shapes: CUDA events around each call, a 256 MiB L2 flush before every call,
    median of --steps calls after --warmup; also the largest difference between the two
    outputs. This kernel is also timed on the reference's grid (one cluster per 512-row
    block, no KV split), which compares the two kernels' per-tile rates at equal
    occupancy. Where baseline/library_fmha.py's prebuilt library kernel exists, it is
    timed the same way beside them."""
    import torch

    from llm_fa_b200 import _lib, attention_forward, device_status
    from llm_fa_b200.attention import forward_with
    from oracle.build_ref import load_module
    mod = load_module()
    lib = _lib.lib()
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
        # the same kernel on the reference's grid (one cluster per 512-row block, no KV
        # split), so that the two kernels' per-tile rates compare at equal occupancy
        t_grid = median_us(lambda: forward_with(lib, Q, K, V, out=O, split_kv=False))
        t_ref = median_us(lambda: mod.llm_fa_forward(Q, K, V))
        diff = (O.float() - mod.llm_fa_forward(Q, K, V)[0].float()).abs().max().item()
        flops = 4 * q_len * sk * 128
        row = {"q": q_len, "sk": sk, "ours_us": round(t_ours, 1),
               "reference_us": round(t_ref, 1),
               "speedup": round(t_ref / t_ours, 3),
               "ours_tflops": round(flops / t_ours / 1e6, 1),
               "reference_tflops": round(flops / t_ref / 1e6, 1),
               "max_abs_diff_vs_reference": diff,
               "ours_on_reference_grid_us": round(t_grid, 1),
               "speedup_on_reference_grid": round(t_ref / t_grid, 3)}
        # the same-box library kernel (baseline/library_fmha.py), when built
        try:
            from baseline.library_fmha import LibraryFMHA
            fmha = LibraryFMHA(*(t.view(1, -1, 1, 128) for t in (Q, K, V)), 1.0 / 128 ** 0.5)
        except Exception as e:
            row["library"] = {"unavailable": f"{type(e).__name__}: {e}"[:160]}
        else:
            t_lib = median_us(fmha)
            row["library"] = {"impl": fmha.version, "us": round(t_lib, 1),
                              "tflops": round(flops / t_lib / 1e6, 1),
                              "speedup_of_this_kernel": round(t_lib / t_ours, 3),
                              "max_abs_diff_vs_this_kernel":
                                  (fmha.out.view(q_len, 128).float() - O.float()).abs().max().item()}
            del fmha
        print(json.dumps(row), flush=True)
        del Q, K, V, O
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
    import dataclasses

    from llm_fa_b200.workloads import CONFIGS
    cfg = CONFIGS[args.config]
    if args.heads is not None:
        if not 1 <= args.heads <= cfg.heads:
            raise SystemExit(f"--heads must be in 1..{cfg.heads}")
        cfg = dataclasses.replace(cfg, heads=args.heads)
    import torch.distributed as dist
    if world > 1:
        import torch
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    try:
        run = run_reference if args.impl == "reference" else run_ours
        line = run(args, cfg, world, rank, local)
    finally:
        if world > 1:
            dist.destroy_process_group()
    if line is not None:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
