"""GPU tests of llm_fa_b200.host.HostAttention (host tensors in, host O out, copies
overlapped across requests)."""
import pytest
import torch

from llm_fa_b200 import attention_forward, device_status
from llm_fa_b200.host import HostAttention
from llm_fa_b200.workloads import Config, make_inputs

pytestmark = pytest.mark.gpu


def test_pipelined_requests_match_device_calls():
    # four requests through two buffer slots: slot reuse must wait for the earlier
    # request's compute and copy-out
    cfgs = [Config("h", 1, 2, 1000, 2049, seed=s) for s in (11, 12, 13)] + \
           [Config("h", 2, 3, 700, 640, seed=14)]
    ha = HostAttention(torch.device("cuda", 0), depth=2)
    ins = [tuple(t.contiguous().pin_memory() for t in make_inputs(c)) for c in cfgs]
    outs = [torch.empty(q.shape, dtype=q.dtype).pin_memory() for q, _, _ in ins]
    events = [ha.submit(q, k, v, o) for (q, k, v), o in zip(ins, outs)]
    events[-1].synchronize()
    ha.synchronize()
    assert device_status() == 0
    for (q, k, v), o in zip(ins, outs):
        ref = attention_forward(q.cuda(), k.cuda(), v.cuda()).cpu()
        assert torch.equal(o, ref)


def test_pageable_inputs_and_argument_checks():
    q, k, v = make_inputs(Config("h", 1, 1, 512, 512, seed=21))
    ha = HostAttention(0, depth=1)
    o = torch.empty_like(q)
    ha.submit(q, k, v, o).synchronize()
    assert torch.equal(o, attention_forward(q.cuda(), k.cuda(), v.cuda()).cpu())
    with pytest.raises(RuntimeError):
        ha.submit(q.cuda(), k, v, o)
    with pytest.raises(RuntimeError):
        ha.submit(q, k, v, torch.empty(1, 512, 1, 128, dtype=torch.bfloat16)[:, :256])
