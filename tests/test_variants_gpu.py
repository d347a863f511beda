"""GPU tests of the library's compile-time variants (built beside the product library).

* The trace build (-DLLMFA_TRACE=1) computes the same attention as the product,
  records every traced hand-off event of cluster 0's window, and its events
  follow the per-tile chain S(j) visible -> scores loaded -> rescale factor ->
  P half -> MMA sees P half / P full -> QK(j+1) -> S(j+1) visible: the
  verification the reference runs on its own traces (its trace conventions'
  checklist and its flow walker). The wait-statistics build (trace level 2)
  reports per-wait-site statistics within the hand-offs the schedule has.
* The ablation-ladder rungs (floor, faux, noexp) run to completion with a clean
  device status; their outputs are not attention and are not checked.
"""
import ctypes

import pytest
import torch

from llm_fa_b200 import _lib, trace
from llm_fa_b200.attention import forward_with
from llm_fa_b200.build import build_variant
from llm_fa_b200.workloads import Config, make_inputs
from oracle.sdpa_oracle import MAX_ABS_TOL, MEAN_ABS_TOL, compare, sdpa_fp32

pytestmark = pytest.mark.gpu


def _status(h) -> int:
    out = ctypes.c_int(0)
    _lib.check(h.llmfa_device_status(ctypes.byref(out), ctypes.c_void_p(
        torch.cuda.current_stream().cuda_stream)), "llmfa_device_status")
    return out.value


def _traced_forward(h, cfg):
    q, k, v = make_inputs(cfg)
    qd, kd, vd = q.cuda(), k.cuda(), v.cuda()
    forward_with(h, qd, kd, vd, split_kv=False)  # warm-up
    torch.cuda.synchronize()
    trace.read_all(h)  # clears the wait statistics
    o = forward_with(h, qd, kd, vd, split_kv=False)
    torch.cuda.synchronize()
    assert _status(h) == 0
    err = compare(o, sdpa_fp32(q, k, v))
    assert err["nonfinite"] == 0
    assert err["max_abs"] < MAX_ABS_TOL and err["mean_abs"] < MEAN_ABS_TOL, err
    return trace.read_all(h)


# 2 query blocks x 64 KV tiles, classic schedule (no workspace): cluster 0 runs unit 0 over
# all 64 tiles, which covers the traced iterations 32..47
TRACE_CFG = Config("tr", 1, 1, 1024, 8192, seed=77)


def test_trace_build_events_and_chain():
    h = _lib.load(build_variant("trace"))
    assert _lib.build_config(h) == {"ablation": 0, "ablation_name": "none", "trace": 1}
    ev, seg, wait = _traced_forward(h, TRACE_CFG)
    assert trace.check_chain(ev) == []
    E = {e: i for i, e in enumerate(trace.EVENTS)}
    for name in ("s_ready", "stat", "p_half", "p_full", "corr_stat", "corr_p_full", "prod_load"):
        for r in (0, 1):  # every CTA's own roles
            assert (ev[r, :, E[name]]["globaltimer_ns"] > 0).all(), (name, r)
    for name in ("mma_p_half", "mma_p_full", "mma_qk_next", "kv_landed"):  # leader only
        assert (ev[0, :, E[name]]["globaltimer_ns"] > 0).all(), name
    # the segment timeline has cluster 0's one segment: unit 0, 64 tiles
    assert int(seg[0, 0, 3]) == 0 * 65536 + 64 and seg[0, 0, 0] > 0
    assert not wait.any()  # no wait statistics below trace level 2


def test_waitstats_build_statistics():
    """Per-wait-site statistics: the counts stay within the hand-offs the schedule has
    (4 CTAs, 64 KV tiles per unit, one unit per cluster), the softmax warps wait for S,
    and every share of a role's time lies in [0, 1]."""
    h = _lib.load(build_variant("waitstats"))
    assert _lib.build_config(h)["trace"] == 2
    ev, seg, wait = _traced_forward(h, TRACE_CFG)
    assert trace.check_chain(ev) == []
    n_kv, ctas, leaders = 64, 4, 2
    assert int(wait[0, 1]) == ctas
    assert 0 < int(wait[6, 1]) <= ctas * 8 * n_kv      # softmax: S(j) of its tile
    assert int(wait[7, 1]) <= ctas * 4 * 2 * n_kv      # correction: both tiles' rescale factor
    assert int(wait[5, 1]) <= leaders * 4 * n_kv       # MMA: P half + P full of both tiles
    assert int(wait[2, 1]) <= ctas * 2 * n_kv          # producer: K and V stage per tile
    assert int(wait[3, 1]) <= leaders * 2              # MMA: both Q tiles of the unit
    rows = trace.wait_table(wait, trace.clock_ghz(ev))
    assert rows and all(0.0 <= r["share_of_role_time"] <= 1.0 for r in rows), rows


@pytest.mark.parametrize("rung,code", [("floor", 1), ("faux", 2), ("noexp", 3)])
def test_ablation_rungs_run_to_completion(rung, code):
    h = _lib.load(build_variant(rung))
    assert _lib.build_config(h)["ablation"] == code
    for B, H, Sq, Sk in ((1, 1, 2048, 4096), (1, 1, 16384, 2048)):  # classic and split KV
        q, k, v = (t.cuda() for t in make_inputs(Config("ab", B, H, Sq, Sk, seed=5)))
        o = forward_with(h, q, k, v)
        torch.cuda.synchronize()
        assert _status(h) == 0, rung
        assert o.shape == q.shape
