"""Read and summarise the kernel's event trace (library built with LLMFA_TRACE=1).

Counterpart of the reference's profiler ring (profiler.cuh:44-151) and its
Perfetto dumper (trace_dump.py:98-325): instead of a per-warp ring flushed
with atomics, the traced build records fixed hand-off events of both Q tiles
for a window of KV iterations of cluster 0 (see TraceEvent in fa_fwd_kernel.cuh).
Output is a Chrome trace-event JSON (chrome://tracing, Perfetto UI) and a
table of per-hop latencies; no third-party tracing package is needed.
"""
from __future__ import annotations

import ctypes
import json

import numpy as np

from . import _lib

EVENTS = ["s_ready", "ld_done", "stat", "p_half", "p_full", "mma_p_half", "mma_p_full",
          "mma_qk_next", "corr_stat", "corr_arrive", "mma_kv_ready", "prod_load", "kv_landed",
          "mma_loop_top", "corr_p_full"]
ROLES = {"s_ready": "softmax", "ld_done": "softmax", "stat": "softmax", "p_half": "softmax",
         "p_full": "softmax", "mma_p_half": "mma", "mma_p_full": "mma", "mma_qk_next": "mma",
         "corr_stat": "correction", "corr_arrive": "correction", "mma_kv_ready": "mma",
         "prod_load": "producer", "kv_landed": "producer", "mma_loop_top": "mma",
         "corr_p_full": "correction"}
TRACE_FIRST = 32
TRACE_ITERS = 16
RECORD = np.dtype([("globaltimer_ns", "<u8"), ("clock", "<i8")])


def read_trace() -> np.ndarray:
    """Structured array [cta rank 2][Q tile 2][event][iteration] of (globaltimer_ns, clock)."""
    n = 2 * 2 * len(EVENTS) * TRACE_ITERS
    buf = np.zeros(n, dtype=RECORD)
    written = ctypes.c_uint64(0)
    rc = _lib.lib().llmfa_trace_read(ctypes.c_void_p(buf.ctypes.data), buf.nbytes,
                                     ctypes.byref(written))
    _lib.check(rc, "llmfa_trace_read (library built without LLMFA_TRACE=1?)")
    return buf.reshape(2, 2, len(EVENTS), TRACE_ITERS)


SEG_CLUSTERS = 160
SEG_SEGMENTS = 32


def read_segments() -> np.ndarray:
    """Segment timeline of every cluster, uint64 [cluster][segment][4]:
    %globaltimer of the first QK, of the epilogue seeing O complete, of the
    epilogue done, then u * 65536 + len (all zero for segments not run)."""
    n_ev = 2 * 2 * len(EVENTS) * TRACE_ITERS * RECORD.itemsize
    n_seg = SEG_CLUSTERS * SEG_SEGMENTS * 4 * 8
    buf = np.zeros(n_ev + n_seg, dtype=np.uint8)
    written = ctypes.c_uint64(0)
    rc = _lib.lib().llmfa_trace_read(ctypes.c_void_p(buf.ctypes.data), buf.nbytes,
                                     ctypes.byref(written))
    _lib.check(rc, "llmfa_trace_read (library built without LLMFA_TRACE=1?)")
    if written.value < n_ev + n_seg:
        raise RuntimeError("library trace has no segment timeline")
    return buf[n_ev:].view(np.uint64).reshape(SEG_CLUSTERS, SEG_SEGMENTS, 4)


def clock_ghz(tr: np.ndarray) -> float:
    """SM clock estimated from the trace: slope of %clock64 against %globaltimer."""
    g = tr["globaltimer_ns"].astype(np.float64)
    c = tr["clock"].astype(np.float64)
    out = []
    for r in (0, 1):  # clock64 offsets differ per SM
        m = g[r] > 0
        if m.sum() > 2:
            gx, cx = g[r][m], c[r][m]
            out.append(np.polyfit(gx - gx.mean(), cx - cx.mean(), 1)[0])
    return float(np.mean(out)) if out else float("nan")


def hop_latencies(tr: np.ndarray, clock_ghz: float) -> dict[str, float]:
    """Median latency (ns) of each hand-off of the pipeline, per CTA and Q tile.

    Intra-CTA hops use %clock64 divided by `clock_ghz`; the cross-CTA hop (the
    peer's P reaching the leader's MMA warp) uses %globaltimer, whose
    resolution on B200 is 32 ns.
    """
    E = {e: i for i, e in enumerate(EVENTS)}

    def clk(rank, tile, ev):
        return tr[rank, tile, E[ev]]["clock"].astype(np.float64) / clock_ghz

    def gt(rank, tile, ev):
        return tr[rank, tile, E[ev]]["globaltimer_ns"].astype(np.float64)

    out = {}
    for r in (0, 1):
        for t in (0, 1):
            k = f"cta{r} tile{t}: "
            out[k + "S visible -> scores in registers"] = np.median(clk(r, t, "ld_done") - clk(r, t, "s_ready"))
            out[k + "scores -> rescale factor published"] = np.median(clk(r, t, "stat") - clk(r, t, "ld_done"))
            out[k + "rescale published -> P half"] = np.median(clk(r, t, "p_half") - clk(r, t, "stat"))
            out[k + "P half -> P full"] = np.median(clk(r, t, "p_full") - clk(r, t, "p_half"))
            out[k + "softmax (S visible -> P full)"] = np.median(clk(r, t, "p_full") - clk(r, t, "s_ready"))
            out[k + "period (S visible to S visible)"] = np.median(np.diff(clk(r, t, "s_ready")))
            out[k + "correction sees rescale factor after it is published"] = np.median(
                clk(r, t, "corr_stat") - clk(r, t, "stat"))
            out[k + "correction P full - softmax P full (> 0: correction is later)"] = np.median(
                clk(r, t, "corr_p_full") - clk(r, t, "p_full"))
    for t in (0, 1):
        k = f"tile{t}: "
        out[k + "cta0 P half -> MMA sees P half"] = np.median(clk(0, t, "mma_p_half") - clk(0, t, "p_half"))
        out[k + "cta0 P full -> MMA sees P full"] = np.median(clk(0, t, "mma_p_full") - clk(0, t, "p_full"))
        out[k + "cta1 P full -> MMA sees P full (globaltimer)"] = np.median(
            gt(0, t, "mma_p_full") - gt(1, t, "p_full"))
        out[k + "MMA sees P full -> QK(j+1) issued"] = np.median(clk(0, t, "mma_qk_next") - clk(0, t, "mma_p_full"))
        out[k + "QK(j+1) issued -> softmax sees S(j+1)"] = np.median(
            clk(0, t, "s_ready")[1:] - clk(0, t, "mma_qk_next")[:-1])
        out[k + "K/V load issued -> landed"] = np.median(clk(0, t, "kv_landed") - clk(0, t, "prod_load"))
    out["tile1 S visible - tile0 S visible (same j)"] = np.median(clk(0, 1, "s_ready") - clk(0, 0, "s_ready"))
    return {k: float(v) for k, v in out.items()}


def timeline(tr: np.ndarray, clock_ghz: float, rank: int = 0, first: int = 4, count: int = 2):
    """(ns since S_0 visible at window iteration `first`, label) for CTA `rank`, sorted."""
    base = tr[rank, 0, 0]["clock"][first]
    rows = []
    for i in range(first, min(first + count, TRACE_ITERS)):
        for t in (0, 1):
            for e, name in enumerate(EVENTS):
                c = tr[rank, t, e]["clock"][i]
                if tr[rank, t, e]["globaltimer_ns"][i]:
                    rows.append(((c - base) / clock_ghz, f"it{TRACE_FIRST + i} tile{t} {name}"))
    return sorted(rows)


def to_chrome_json(tr: np.ndarray, path: str, clock_ghz: float) -> None:
    """Instant events per role and tile (pid = CTA rank, tid = role/tile), times in microseconds."""
    valid = tr["globaltimer_ns"] > 0
    t0 = int(tr["globaltimer_ns"][valid].min())
    events = []
    for r in range(2):
        anchor = tr[r, 0, 0][0]
        base_clk, base_gt = int(anchor["clock"]), int(anchor["globaltimer_ns"])
        for t in range(2):
            for e, name in enumerate(EVENTS):
                for i in range(TRACE_ITERS):
                    if tr[r, t, e]["globaltimer_ns"][i] == 0:
                        continue
                    # clock64 for precise intra-CTA spacing, anchored on the CTA's globaltimer
                    t_ns = (base_gt - t0) + (int(tr[r, t, e]["clock"][i]) - base_clk) / clock_ghz
                    events.append({"name": name, "ph": "i", "s": "t", "pid": f"cta{r}",
                                   "tid": f"{ROLES[name]} tile{t}", "ts": t_ns / 1e3,
                                   "args": {"iteration": TRACE_FIRST + i}})
    with open(path, "w") as f:
        json.dump({"traceEvents": events, "displayTimeUnit": "ns"}, f)
