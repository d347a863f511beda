"""Host-side trace tooling on a synthetic trace (no GPU, no traced library).

The traced library build writes records laid out [cta rank][Q tile][event]
[iteration]; these tests fill that layout with a known schedule and check that
the clock estimate, the per-hop medians and the Chrome trace export read it
back correctly.
"""
import json

import numpy as np

from llm_fa_b200 import trace


def _synthetic(ghz=1.8, period_ns=2000.0):
    tr = np.zeros((2, 2, len(trace.EVENTS), trace.TRACE_ITERS), dtype=trace.RECORD)
    offsets = {e: 10.0 * i for i, e in enumerate(trace.EVENTS)}  # ns after S visible
    for r in range(2):
        for t in range(2):
            for e, name in enumerate(trace.EVENTS):
                ns = np.arange(trace.TRACE_ITERS) * period_ns + offsets[name] + 700.0 * t + 5000.0
                tr[r, t, e]["globaltimer_ns"] = (ns // 32 * 32).astype(np.uint64) + 1_000_000
                tr[r, t, e]["clock"] = (ns * ghz).astype(np.int64) + 123_456 * (r + 1)
    return tr


def test_clock_estimate_and_hops():
    tr = _synthetic()
    ghz = trace.clock_ghz(tr)
    assert abs(ghz - 1.8) < 0.01
    hops = trace.hop_latencies(tr, ghz)
    assert abs(hops["cta0 tile0: period (S visible to S visible)"] - 2000.0) < 2.0
    assert abs(hops["cta1 tile1: softmax (S visible -> P full)"] - 40.0) < 2.0
    assert abs(hops["tile1 S visible - tile0 S visible (same j)"] - 700.0) < 2.0


def test_chrome_export(tmp_path):
    tr = _synthetic()
    path = tmp_path / "t.json"
    trace.to_chrome_json(tr, str(path), 1.8)
    events = json.loads(path.read_text())["traceEvents"]
    assert len(events) == 2 * 2 * len(trace.EVENTS) * trace.TRACE_ITERS
    assert {e["tid"] for e in events} >= {"softmax tile0", "mma tile1", "producer tile0"}
    assert min(e["ts"] for e in events) >= 0.0
    rows = trace.timeline(tr, 1.8, rank=0, first=2, count=1)
    assert rows[0][0] == 0.0 and rows[0][1].endswith("tile0 s_ready")
