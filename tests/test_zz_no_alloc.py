"""GPU test of llmfa_forward_static_scratch, the entry point that allocates nothing.

It exists for callers that cannot allocate device memory themselves (a
foreign-language host that only holds device pointers it was given, or a
framework that plans all device memory up front and forbids allocation on the
request path): they cannot supply llmfa_forward's split-KV workspace, so this
entry point takes that scratch from a fixed array inside the library.

The test calls it through the C ABI twice in a row (the array keeps the first
call's contents) and requires each result to be bit-identical to llmfa_forward
given a normal workspace: both calls run the same kernels with the same
deterministic launch plan, so any difference means the fixed array was read
stale or overrun. It also checks sampled rows against the CPU oracle within
the parity tolerance of the other GPU tests, and that the split-KV path (the
one that uses the scratch) really ran where the shape calls for it. The file
is named so pytest collects it last.
"""
import ctypes
import math

import pytest
import torch

from llm_fa_b200 import _lib, device_status, launch_plan, reset_device_status
from llm_fa_b200.attention import workspace_size
from llm_fa_b200.workloads import Config, make_inputs, sample_rows
from oracle.sdpa_oracle import MAX_ABS_TOL, MEAN_ABS_TOL, compare, sdpa_fp32

pytestmark = pytest.mark.gpu


def _args(q, k, v, o):
    B, Sq, H, _ = q.shape
    return (ctypes.c_void_p(q.data_ptr()), _lib.strides3(q.stride()[:3]),
            ctypes.c_void_p(k.data_ptr()), _lib.strides3(k.stride()[:3]),
            ctypes.c_void_p(v.data_ptr()), _lib.strides3(v.stride()[:3]),
            ctypes.c_void_p(o.data_ptr()), _lib.strides3(o.stride()[:3]),
            B, H, Sq, k.shape[1], ctypes.c_float(1.0 / math.sqrt(128)))


# (1, 1, 16384, 4096) and (1, 2, 1000, 777) split KV ranges across clusters (the
# scratch is written and read); (2, 8, 2048, 1024) fills the GPU without a split.
@pytest.mark.parametrize("B,H,Sq,Sk,splits", [(1, 1, 16384, 4096, True),
                                               (2, 8, 2048, 1024, None),
                                               (1, 2, 1000, 777, True)])
def test_static_scratch_entry_point_matches_workspace_entry_point(B, H, Sq, Sk, splits):
    assert torch.cuda.is_available()
    reset_device_status()
    cfg = Config("na", B, H, Sq, Sk, seed=Sq + Sk + H)
    q_h, k_h, v_h = make_inputs(cfg)
    q, k, v = q_h.cuda(), k_h.cuda(), v_h.cuda()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    L = _lib.lib()
    plan = launch_plan(B, H, Sq, Sk)
    if splits:
        assert plan["kernels"] == 2 and plan["split_units"] > 0, plan

    # reference result: the existing entry point with a caller-allocated workspace
    ws_bytes = workspace_size()
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    o_ref = torch.empty_like(q)
    _lib.check(L.llmfa_forward(*_args(q, k, v, o_ref), ctypes.c_void_p(ws.data_ptr()), ws_bytes,
                               stream), "llmfa_forward")

    outs = []
    for _ in range(2):  # the fixed scratch still holds the previous call's contents
        o = torch.full_like(q, float("nan"))
        _lib.check(L.llmfa_forward_static_scratch(*_args(q, k, v, o), stream),
                   "llmfa_forward_static_scratch")
        outs.append(o)
    torch.cuda.synchronize()
    assert device_status() == 0
    for o in outs:
        assert torch.equal(o, o_ref), (compare(o, o_ref.float()), plan)
    rows = sample_rows(cfg, 256)
    err = compare(outs[1][:, rows].cpu(), sdpa_fp32(q_h, k_h, v_h, rows=rows))
    assert err["nonfinite"] == 0, err
    assert err["max_abs"] < MAX_ABS_TOL and err["mean_abs"] < MEAN_ABS_TOL, err

