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


SEG_CLUSTERS = 160
SEG_SEGMENTS = 32
WAIT_SLOTS = 16
# Bounded-wait sites of the attention kernel (WaitSite in fa_fwd_kernel.cuh): id -> (role,
# what the waiting warp waits for). Slot 0 of the statistics holds the CTAs' run time.
WAIT_SITES = {
    1: ("producer", "Q tile slot free (last QK of the previous unit done)"),
    2: ("producer", "K/V stage free (MMAs that read it done)"),
    3: ("mma", "Q tile landed"),
    4: ("mma", "K/V stage landed"),
    5: ("mma", "P published (half or full) by softmax + correction warps"),
    6: ("softmax", "S = QK^T in TMEM"),
    7: ("correction", "rescale factor published by the softmax warp"),
    8: ("correction", "end-of-segment row sum published"),
    9: ("correction", "O complete in TMEM (last PV of the segment)"),
    10: ("correction", "O staging buffer free / filled (TMA store)"),
    11: ("mma", "teardown drain of the last MMAs"),
}
# warps of one CTA that wait at each role's sites (lane 0 of each is counted)
ROLE_WARPS = {"producer": 1, "mma": 1, "softmax": 8, "correction": 4}

_EV_BYTES = 2 * 2 * len(EVENTS) * TRACE_ITERS * RECORD.itemsize
_SEG_BYTES = SEG_CLUSTERS * SEG_SEGMENTS * 4 * 8
_WAIT_BYTES = WAIT_SLOTS * 2 * 8


def _read(handle, nbytes: int) -> tuple[np.ndarray, int]:
    h = _lib.lib() if handle is None else handle
    buf = np.zeros(nbytes, dtype=np.uint8)
    written = ctypes.c_uint64(0)
    rc = h.llmfa_trace_read(ctypes.c_void_p(buf.ctypes.data), buf.nbytes, ctypes.byref(written))
    _lib.check(rc, "llmfa_trace_read (library built without LLMFA_TRACE=1?)")
    return buf, written.value


def read_trace(handle=None) -> np.ndarray:
    """Structured array [cta rank 2][Q tile 2][event][iteration] of (globaltimer_ns, clock).
    `handle`: a library loaded with _lib.load (default: the product library)."""
    buf, _ = _read(handle, _EV_BYTES)
    return buf.view(RECORD).reshape(2, 2, len(EVENTS), TRACE_ITERS)


def read_all(handle=None) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """(events, segment timeline, wait statistics) in one read; the read clears the wait
    statistics. Segment timeline: uint64 [cluster][segment][4] = %globaltimer of the first
    QK, of the epilogue seeing O complete, of the epilogue done, then u * 65536 + len
    (zero for segments not run). Wait statistics: uint64 [16][2] (see WAIT_SITES)."""
    buf, written = _read(handle, _EV_BYTES + _SEG_BYTES + _WAIT_BYTES)
    if written < _EV_BYTES + _SEG_BYTES + _WAIT_BYTES:
        raise RuntimeError("library trace has no segment timeline / wait statistics")
    ev = buf[:_EV_BYTES].view(RECORD).reshape(2, 2, len(EVENTS), TRACE_ITERS)
    seg = buf[_EV_BYTES:_EV_BYTES + _SEG_BYTES].view(np.uint64).reshape(
        SEG_CLUSTERS, SEG_SEGMENTS, 4)
    wait = buf[_EV_BYTES + _SEG_BYTES:].view(np.uint64).reshape(WAIT_SLOTS, 2)
    return ev, seg, wait


def read_segments(handle=None) -> np.ndarray:
    """Segment timeline of every cluster (see read_all)."""
    return read_all(handle)[1]


def wait_table(wait: np.ndarray, clock_ghz: float) -> list[dict]:
    """Per wait site, over the waits that took more than 64 cycles: how many per CTA, their
    mean length, and the share of the waiting warps' time spent in them (cycles waited /
    (warps of the role x CTA run cycles))."""
    cta_cycles, ctas = float(wait[0, 0]), max(float(wait[0, 1]), 1.0)
    rows = []
    for site, (role, what) in WAIT_SITES.items():
        cyc, n = float(wait[site, 0]), float(wait[site, 1])
        if n == 0:
            continue
        rows.append({"site": site, "role": role, "waits_for": what,
                     "waits_per_cta": n / ctas,
                     "mean_wait_ns": cyc / n / clock_ghz,
                     "share_of_role_time": cyc / (ROLE_WARPS[role] * cta_cycles)})
    return rows


# The hand-off chain of one Q tile's KV iteration j, as causal edges (a, b, b's iteration
# offset): the softmax warps' program order, each barrier hand-off to the leader's MMA warp
# and the MMA warp's program order, and QK(j+1) -> S(j+1) visible.
CHAIN_EDGES = [
    ("s_ready", "ld_done", 0), ("ld_done", "stat", 0), ("stat", "p_half", 0),
    ("p_half", "p_full", 0),
    ("p_half", "mma_p_half", 0), ("p_full", "mma_p_full", 0),
    ("mma_p_half", "mma_p_full", 0), ("mma_p_full", "mma_qk_next", 0),
    ("mma_qk_next", "s_ready", 1),
]
CHAIN_EVENTS = ["s_ready", "ld_done", "stat", "p_half", "p_full", "mma_p_half", "mma_p_full",
                "mma_qk_next"]


def check_chain(tr: np.ndarray, slack_ns: float = 64.0) -> list[str]:
    """Walk every traced iteration's hand-off chain (CHAIN_EDGES) for both Q tiles and both
    CTAs; return the violations (empty = every event present and every edge in order).
    Within one SM (the leader CTA's softmax and MMA warps) the order is checked on
    %clock64; the peer CTA's softmax events against the leader's MMA events on
    %globaltimer, whose resolution is 32 ns, with `slack_ns` of tolerance. Edges into the
    next iteration are checked for all but the window's last iteration."""
    E = {e: i for i, e in enumerate(EVENTS)}
    bad = []
    for r in (0, 1):
        for t in (0, 1):
            for name in CHAIN_EVENTS:
                src = 0 if ROLES[name] == "mma" else r
                missing = np.nonzero(tr[src, t, E[name]]["globaltimer_ns"] == 0)[0]
                if len(missing):
                    bad.append(f"cta{r} tile{t}: {name} missing at iterations "
                               f"{[TRACE_FIRST + int(i) for i in missing]}")
            for i in range(TRACE_ITERS):
                for a, b, off in CHAIN_EDGES:
                    j_b = i + off
                    if j_b >= TRACE_ITERS:
                        continue
                    ra = 0 if ROLES[a] == "mma" else r
                    rb = 0 if ROLES[b] == "mma" else r
                    if ra == rb:  # same SM: cycle counter
                        ta = int(tr[ra, t, E[a]]["clock"][i])
                        tb = int(tr[rb, t, E[b]]["clock"][j_b])
                        ok = tb >= ta
                    else:
                        ta = float(tr[ra, t, E[a]]["globaltimer_ns"][i])
                        tb = float(tr[rb, t, E[b]]["globaltimer_ns"][j_b])
                        ok = tb + slack_ns >= ta
                    if not ok:
                        bad.append(f"cta{r} tile{t} iteration {TRACE_FIRST + i}: {a} -> {b} "
                                   f"out of order ({ta} > {tb})")
    return bad


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


def main() -> None:
    """python -m llm_fa_b200.trace [--config c3] [--chrome out.json]: run the configuration
    through the trace build (hand-off latencies, chain check) and the wait-statistics build
    (per-wait-site table, markdown), with each build's time beside the product's."""
    import argparse

    import torch

    from .attention import forward_with
    from .build import build_variant
    from .workloads import CONFIGS, make_inputs

    ap = argparse.ArgumentParser(description=main.__doc__.splitlines()[0])
    ap.add_argument("--config", default="c3")
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--chrome", default=None, help="write a Chrome trace-event JSON here")
    a = ap.parse_args()
    builds = {"product": _lib.lib(), "trace": _lib.load(build_variant("trace")),
              "waitstats": _lib.load(build_variant("waitstats"))}
    cfg = CONFIGS[a.config]
    dev = torch.device("cuda", 0)
    q, k, v = (t.to(dev) for t in make_inputs(cfg))
    o = torch.empty_like(q)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    got = {}
    for name, h in builds.items():
        for _ in range(a.warmup):
            forward_with(h, q, k, v, out=o)
        torch.cuda.synchronize()
        if name != "product":
            read_all(h)  # clears the wait statistics of the warm-up launches
        flush.zero_()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        forward_with(h, q, k, v, out=o)
        e1.record()
        torch.cuda.synchronize()
        got[name] = (e0.elapsed_time(e1), None if name == "product" else read_all(h))
    print(f"# {cfg.name} ({cfg.describe()}): " + ", ".join(
        f"{n} build {t:.3f} ms" for n, (t, _) in got.items()))
    ev = got["trace"][1][0]
    ghz = clock_ghz(ev)
    print(f"# SM clock from the trace: {ghz:.3f} GHz")
    print("\n## hand-off latencies of the trace build (median over the traced window, ns)\n")
    for name, val in hop_latencies(ev, ghz).items():
        print(f"- {name}: {val:.0f}")
    bad = check_chain(ev)
    print(f"\n## chain check: {'ok' if not bad else f'{len(bad)} violations'}")
    for b in bad[:20]:
        print(f"- {b}")
    ev2, _, wait = got["waitstats"][1]
    print("\n## wait sites of the wait-statistics build (all CTAs of the launch; waits longer "
          "than 64 cycles)\n")
    print("| site | role | waits for | waits per CTA | mean wait (ns) | share of the role's time |")
    print("|---|---|---|---|---|---|")
    for r in wait_table(wait, clock_ghz(ev2)):
        print(f"| {r['site']} | {r['role']} | {r['waits_for']} | {r['waits_per_cta']:.1f} | "
              f"{r['mean_wait_ns']:.0f} | {100 * r['share_of_role_time']:.1f} % |")
    if a.chrome:
        to_chrome_json(ev, a.chrome, ghz)


if __name__ == "__main__":
    main()
