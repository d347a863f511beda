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


def test_chain_check_accepts_the_schedule_and_reports_a_reordering():
    tr = _synthetic()
    assert trace.check_chain(tr) == []
    E = {e: i for i, e in enumerate(trace.EVENTS)}
    bad = tr.copy()
    # the leader's MMA warp "sees" tile 1's P half before CTA 0 published it
    bad[0, 1, E["mma_p_half"], 3]["clock"] = bad[0, 1, E["p_half"], 3]["clock"] - 100
    msgs = trace.check_chain(bad)
    assert msgs and all("p_half -> mma_p_half" in m for m in msgs), msgs
    gone = tr.copy()
    gone[1, 0, E["stat"], 5]["globaltimer_ns"] = 0
    assert any("stat missing" in m for m in trace.check_chain(gone))


def test_wait_table_shares():
    wait = np.zeros((trace.WAIT_SLOTS, 2), dtype=np.uint64)
    wait[0] = (2 * 1_000_000, 2)      # two CTAs of 1e6 cycles
    wait[6] = (8 * 2 * 250_000, 400)  # softmax S waits: 8 warps x 2 CTAs x 250k cycles
    wait[4] = (2 * 100_000, 60)       # MMA K/V waits
    rows = {r["site"]: r for r in trace.wait_table(wait, clock_ghz=2.0)}
    assert set(rows) == {4, 6}
    assert abs(rows[6]["share_of_role_time"] - 0.25) < 1e-12
    assert abs(rows[4]["share_of_role_time"] - 0.10) < 1e-12
    assert abs(rows[6]["waits_per_cta"] - 200.0) < 1e-12
    assert abs(rows[6]["mean_wait_ns"] - 2 * 8 * 250_000 / 400 / 2.0) < 1e-9
