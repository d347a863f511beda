"""Multi-rank host logic on the CPU (gloo, world size 2).

bench.py shards configurations with several heads over ranks with no exchange
in the data path and gathers O afterwards only for validation. These tests run
that logic with two gloo ranks, the CPU oracle standing in for the kernel:
the gathered shards must equal the whole-problem oracle, and a rank that
leaves early must make its peer fail within the process-group timeout instead
of hanging.
"""
import os
import socket
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import bench
from llm_fa_b200.workloads import Config, make_inputs, shard_heads
from oracle.sdpa_oracle import sdpa_fp32

CFG = Config("shard", 2, 4, 192, 320, seed=31)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=20):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=timedelta(seconds=timeout_s))


def _shard_and_gather(rank, world, port, out_q):
    try:
        _init(rank, world, port)
        q, k, v = make_inputs(CFG)
        shard = bench.local_shard(CFG, world, rank)
        assert shard[0] == "heads"
        ql, kl, vl = bench.slice_inputs(q, k, v, shard)
        o_local = sdpa_fp32(ql, kl, vl).contiguous()
        parts = [torch.empty_like(o_local) for _ in range(world)]
        dist.all_gather(parts, o_local)
        if rank == 0:
            full = torch.cat(parts, dim=2)
            ref = sdpa_fp32(q, k, v)
            out_q.put(("ok", float((full - ref).abs().max())))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as exc:  # reported to the parent
        out_q.put(("error", repr(exc)))


def _peer_leaves(rank, world, port, out_q):
    _init(rank, world, port, timeout_s=5)
    if rank == 1:
        os._exit(0)  # leaves between steps, with no collective in flight
    t = torch.ones(4)
    try:
        dist.all_reduce(t)
        out_q.put(("no error", None))
    except Exception as exc:
        out_q.put(("raised", type(exc).__name__))


def _spawn(fn):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=fn, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
            pytest.fail("rank did not exit")
    return q


def test_head_sharding_covers_every_head_once():
    for world in (1, 2, 4, 8):
        owned = [bh for r in range(world) for bh in shard_heads(4, 32, world, r)]
        assert sorted(owned) == [(b, h) for b in range(4) for h in range(32)]
    assert bench.local_shard(CFG, 2, 1) == ("heads", 2, 4)
    assert bench.local_shard(Config("one", 1, 1, 64, 64, 0), 2, 0) == ("replica",)


def test_single_head_configs_shard_query_rows():
    """One (batch, head): whole 512-row query blocks per rank, K and V on every rank; the
    row shards of all ranks tile the query rows once."""
    from llm_fa_b200.workloads import CONFIGS
    c3 = CONFIGS["c3"]
    for world in (2, 4, 8):
        shards = [bench.local_shard(c3, world, r) for r in range(world)]
        assert all(s[0] == "rows" and (s[2] - s[1]) % 512 == 0 for s in shards)
        assert [s[1] for s in shards] == sorted(s[1] for s in shards)
        assert shards[0][1] == 0 and shards[-1][2] == c3.seq_q
        assert all(a[2] == b[1] for a, b in zip(shards, shards[1:]))
    cfg = Config("rows", 1, 1, 2048, 320, seed=33)
    q, k, v = make_inputs(cfg)
    parts = []
    for r in range(4):
        ql, kl, vl = bench.slice_inputs(q, k, v, bench.local_shard(cfg, 4, r))
        assert kl.shape == k.shape and vl.shape == v.shape
        parts.append(sdpa_fp32(ql, kl, vl))
    assert float((torch.cat(parts, dim=1) - sdpa_fp32(q, k, v)).abs().max()) < 1e-6


def test_two_gloo_ranks_gather_the_whole_output():
    q = _spawn(_shard_and_gather)
    status, err = q.get(timeout=10)
    assert status == "ok", err
    assert err < 1e-6


def test_rank_that_leaves_makes_peer_fail_not_hang():
    q = _spawn(_peer_leaves)
    status, what = q.get(timeout=10)
    assert status == "raised", (status, what)
