"""Read and summarise the kernel's event trace (library built with LLMFA_TRACE=1).

Counterpart of the reference's profiler ring (profiler.cuh:44-151) and its
Perfetto dumper (trace_dump.py:98-325): instead of a per-warp ring flushed
with atomics, the traced build records fixed hand-off events of Q tile 0 for
a window of KV iterations of cluster 0 (see TraceEvent in fa_fwd_kernel.cuh).
Output is a Chrome trace-event JSON (chrome://tracing, Perfetto UI) and a
table of per-hop latencies; no third-party tracing package is needed.
"""
from __future__ import annotations

import ctypes
import json

import numpy as np

from . import _lib

EVENTS = ["s_ready", "ld_done", "stat", "p_half", "p_full", "mma_p_half", "mma_p_full",
          "mma_qk_next", "corr_stat", "corr_arrive"]
TRACE_FIRST = 32
TRACE_ITERS = 16
RECORD = np.dtype([("globaltimer_ns", "<u8"), ("clock", "<i8")])


def read_trace() -> np.ndarray:
    """Structured array [cta rank 2][event][iteration] of (globaltimer_ns, clock)."""
    n = 2 * len(EVENTS) * TRACE_ITERS
    buf = np.zeros(n, dtype=RECORD)
    written = ctypes.c_uint64(0)
    rc = _lib.lib().llmfa_trace_read(ctypes.c_void_p(buf.ctypes.data), buf.nbytes,
                                     ctypes.byref(written))
    _lib.check(rc, "llmfa_trace_read (library built without LLMFA_TRACE=1?)")
    return buf.reshape(2, len(EVENTS), TRACE_ITERS)


def hop_latencies(tr: np.ndarray, clock_ghz: float) -> dict[str, float]:
    """Median latency (ns) of each hand-off of the tile-0 pipeline."""
    E = {e: i for i, e in enumerate(EVENTS)}

    def clk(rank, ev):
        return tr[rank, E[ev]]["clock"].astype(np.float64) / clock_ghz

    def gt(rank, ev):
        return tr[rank, E[ev]]["globaltimer_ns"].astype(np.float64)

    out = {}
    for r in (0, 1):
        out[f"cta{r}: S visible -> scores in registers"] = np.median(clk(r, "ld_done") - clk(r, "s_ready"))
        out[f"cta{r}: scores -> rescale factor published"] = np.median(clk(r, "stat") - clk(r, "ld_done"))
        out[f"cta{r}: rescale published -> P half"] = np.median(clk(r, "p_half") - clk(r, "stat"))
        out[f"cta{r}: P half -> P full"] = np.median(clk(r, "p_full") - clk(r, "p_half"))
        out[f"cta{r}: period (S visible to S visible)"] = np.median(np.diff(clk(r, "s_ready")))
        out[f"cta{r}: correction sees rescale factor after it is published"] = np.median(
            clk(r, "corr_stat") - clk(r, "stat"))
    out["cta0: P half (own softmax) -> MMA sees P half"] = np.median(clk(0, "mma_p_half") - clk(0, "p_half"))
    out["cta0: P full (own softmax) -> MMA sees P full"] = np.median(clk(0, "mma_p_full") - clk(0, "p_full"))
    out["cta1->cta0 (globaltimer): P full -> MMA sees P full"] = np.median(gt(0, "mma_p_full") - gt(1, "p_full"))
    out["cta0: MMA sees P full -> QK(j+1) issued"] = np.median(clk(0, "mma_qk_next") - clk(0, "mma_p_full"))
    out["cta0: QK(j+1) issued -> softmax sees S(j+1)"] = np.median(clk(0, "s_ready")[1:] - clk(0, "mma_qk_next")[:-1])
    return {k: float(v) for k, v in out.items()}


def to_chrome_json(tr: np.ndarray, path: str, clock_ghz: float) -> None:
    """Instant events per role (pid = CTA rank, tid = role), times in microseconds."""
    roles = {"s_ready": "softmax", "ld_done": "softmax", "stat": "softmax", "p_half": "softmax",
             "p_full": "softmax", "mma_p_half": "mma", "mma_p_full": "mma", "mma_qk_next": "mma",
             "corr_stat": "correction", "corr_arrive": "correction"}
    t0 = min(int(tr[r, e]["globaltimer_ns"][i]) for r in range(2) for e in range(len(EVENTS))
             for i in range(TRACE_ITERS) if tr[r, e]["globaltimer_ns"][i] > 0)
    events = []
    for r in range(2):
        base_clk = tr[r, 0]["clock"][0]
        base_gt = tr[r, 0]["globaltimer_ns"][0]
        for e, name in enumerate(EVENTS):
            for i in range(TRACE_ITERS):
                if tr[r, e]["globaltimer_ns"][i] == 0:
                    continue
                # clock64 for precise intra-CTA spacing, anchored on the CTA's globaltimer
                t_ns = (base_gt - t0) + (tr[r, e]["clock"][i] - base_clk) / clock_ghz
                events.append({"name": name, "ph": "i", "s": "t", "pid": f"cta{r}",
                               "tid": roles[name], "ts": t_ns / 1e3,
                               "args": {"iteration": TRACE_FIRST + i}})
    with open(path, "w") as f:
        json.dump({"traceEvents": events, "displayTimeUnit": "ns"}, f)
