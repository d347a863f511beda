"""Ablation ladder: where one forward's time goes, one softmax phase at a time.

    python -m llm_fa_b200.ladder [--config c3] [--rounds 5] [--steps 5] [--warmup 3]

The reference attributes its kernel's time by timing separate ladder kernels
beside it (scaffolding.cu: TMA + MMA + barrier floor, faux.cu: no softmax math;
its README's latency table). Here the rungs are compile-time switches of the
one kernel source (LLMFA_ABLATE, see fa_fwd_kernel.cuh), each built into its
own library file by llm_fa_b200.build.build_variant and loaded beside the
product library:

    floor   softmax and correction warps only pass the barrier hand-offs
    faux    P = bf16(S): no row max, scale, exponentials, row sums or rescale
    noexp   the full softmax with exp2(x) replaced by x
    full    the product

Every rung runs the same launch plan on the same inputs, timed as bench.py
times the product: each call bracketed by CUDA events after a 256 MiB L2
flush, all calls of a block queued before one synchronisation. Rungs take
turns block by block, each block after a short idle pause and its own
warm-up calls (so that no rung inherits another's power state), and the
median per rung is reported (ms,
TFLOP/s and the time the rung adds over the previous one), with the SM clocks
sampled over the whole run. The rungs' outputs are not attention: this is a
measurement tool, never a product path (bench.py refuses a library built with
an ablation switch).
"""
from __future__ import annotations

import argparse
import json
import statistics
import time

import torch

from . import _lib
from .attention import forward_with
from .build import build_variant
from .gpuclocks import ClockSampler

RUNGS = ["floor", "faux", "noexp", "full"]
EXPECTED = {"floor": 1, "faux": 2, "noexp": 3, "full": 0}


def load_rungs() -> dict:
    handles = {}
    for name in RUNGS:
        h = _lib.lib() if name == "full" else _lib.load(build_variant(name))
        cfg = _lib.build_config(h)
        if cfg["ablation"] != EXPECTED[name] or cfg["trace"]:
            raise RuntimeError(f"rung {name}: library reports {cfg}")
        handles[name] = h
    return handles


def main() -> None:
    from .workloads import CONFIGS, make_inputs

    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--config", default="c3")
    ap.add_argument("--rounds", type=int, default=5)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    a = ap.parse_args()
    cfg = CONFIGS[a.config]
    handles = load_rungs()
    dev = torch.device("cuda", 0)
    q, k, v = (t.to(dev) for t in make_inputs(cfg))
    o = torch.empty_like(q)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

    def timed(h) -> list[float]:
        time.sleep(0.1)
        for _ in range(a.warmup):
            flush.zero_()
            forward_with(h, q, k, v, out=o)
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(a.steps)]
        for e0, e1 in ev:
            flush.zero_()  # ~70 us on the GPU: covers the host's launch of the next call
            e0.record()
            forward_with(h, q, k, v, out=o)
            e1.record()
        torch.cuda.synchronize()
        return [e0.elapsed_time(e1) for e0, e1 in ev]

    times = {name: [] for name in RUNGS}
    sampler = ClockSampler(dev.index)
    sampler.start()
    for _ in range(a.rounds):
        for name in RUNGS:
            times[name] += timed(handles[name])
    clocks = sampler.stop()
    for name, h in handles.items():
        st = ctypes_status(h)
        if st != 0:
            raise RuntimeError(f"rung {name}: device status {st:#x}")
    print(json.dumps({"config": cfg.name, "clocks": clocks}), flush=True)
    prev = None
    for name in RUNGS:
        ms = statistics.median(times[name])
        print(json.dumps({"config": cfg.name, "rung": name, "ms": round(ms, 4),
                          "tflops": round(cfg.flops / ms / 1e9, 1),
                          "adds_ms": None if prev is None else round(ms - prev, 4),
                          "samples": len(times[name])}), flush=True)
        prev = ms


def ctypes_status(h) -> int:
    import ctypes
    out = ctypes.c_int(0)
    _lib.check(h.llmfa_device_status(ctypes.byref(out), ctypes.c_void_p(
        torch.cuda.current_stream().cuda_stream)), "llmfa_device_status")
    return out.value


if __name__ == "__main__":
    main()
