"""Attention on host-resident tensors with the copies overlapped.

For callers whose Q, K, V live in host memory and who want O back in host
memory (a request loop that receives inputs from the CPU side), copying in,
computing and copying out one request at a time leaves the GPU idle during
every copy. `HostAttention` keeps `depth` sets of device buffers and three
CUDA streams (host-to-device, compute, device-to-host), so while request i
computes, request i+1's inputs are being copied in and request i-1's output
is being copied out. Each request still copies all of its inputs in and all of
its output back; nothing is cached between requests.

    ha = HostAttention(torch.device("cuda", 0))
    done = ha.submit(q_host, k_host, v_host, o_host)   # returns at once
    done.synchronize()                                   # o_host is filled

Host tensors should be in pinned memory (`tensor.pin_memory()`); pageable
memory works but its copies are synchronous and do not overlap.
"""
from __future__ import annotations

import torch

from .attention import HEAD_DIM, attention_forward


class HostAttention:
    """Pipelined attention_forward for host (CPU) tensors; see the module docstring."""

    def __init__(self, device: torch.device | int | None = None, depth: int = 2):
        if depth < 1:
            raise ValueError("depth must be >= 1")
        self.device = torch.device("cuda", torch.cuda.current_device() if device is None else
                                   (device if isinstance(device, int) else device.index))
        self.depth = depth
        with torch.cuda.device(self.device):
            self.s_in = torch.cuda.Stream(self.device)
            self.s_compute = torch.cuda.Stream(self.device)
            self.s_out = torch.cuda.Stream(self.device)
        self._slots: list[dict | None] = [None] * depth
        self._n = 0

    def _slot(self, i: int, q, k, v):
        key = (tuple(q.shape), tuple(k.shape))
        slot = self._slots[i]
        if slot is None or slot["key"] != key:
            mk = lambda t: torch.empty(t.shape, dtype=torch.bfloat16, device=self.device)  # noqa: E731
            slot = {"key": key, "q": mk(q), "k": mk(k), "v": mk(v), "o": mk(q),
                    "computed": None, "copied_out": None}
            self._slots[i] = slot
        return slot

    @staticmethod
    def _check(t: torch.Tensor, name: str) -> None:
        if t.is_cuda:
            raise RuntimeError(f"{name} must be a host (CPU) tensor; use attention_forward "
                               "for device tensors")
        if t.dtype != torch.bfloat16 or t.shape[-1] != HEAD_DIM or not t.is_contiguous():
            raise RuntimeError(f"{name} must be contiguous bfloat16 with head dim {HEAD_DIM}")

    def submit(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
               out: torch.Tensor, softmax_scale: float | None = None) -> torch.cuda.Event:
        """Queue O = attention(Q, K, V) into the host tensor `out`; returns an event that
        completes when `out` holds the result. Inputs must stay unchanged, and `out`
        unread, until then."""
        for t, nm in ((q, "Q"), (k, "K"), (v, "V"), (out, "out")):
            self._check(t, nm)
        if out.shape != q.shape:
            raise RuntimeError(f"out shape {tuple(out.shape)} must equal Q shape {tuple(q.shape)}")
        i = self._n % self.depth
        self._n += 1
        slot = self._slot(i, q, k, v)
        with torch.cuda.device(self.device):
            # copy in, once the compute that last read this slot's inputs is done
            if slot["computed"] is not None:
                self.s_in.wait_event(slot["computed"])
            with torch.cuda.stream(self.s_in):
                slot["q"].copy_(q, non_blocking=True)
                slot["k"].copy_(k, non_blocking=True)
                slot["v"].copy_(v, non_blocking=True)
                copied_in = torch.cuda.Event()
                copied_in.record(self.s_in)
            # compute, once the inputs landed and the slot's last output was copied out
            self.s_compute.wait_event(copied_in)
            if slot["copied_out"] is not None:
                self.s_compute.wait_event(slot["copied_out"])
            with torch.cuda.stream(self.s_compute):
                attention_forward(slot["q"], slot["k"], slot["v"], out=slot["o"],
                                  softmax_scale=softmax_scale)
                computed = torch.cuda.Event()
                computed.record(self.s_compute)
            # copy out
            self.s_out.wait_event(computed)
            with torch.cuda.stream(self.s_out):
                out.copy_(slot["o"], non_blocking=True)
                copied_out = torch.cuda.Event()
                copied_out.record(self.s_out)
            # The slot's buffers come from the caching allocator on the current
            # stream; when a later request of another shape replaces them, they
            # must not be handed out again before this work on the three
            # streams has finished.
            for name, streams in (("q", (self.s_in, self.s_compute)),
                                  ("k", (self.s_in, self.s_compute)),
                                  ("v", (self.s_in, self.s_compute)),
                                  ("o", (self.s_compute, self.s_out))):
                for st in streams:
                    slot[name].record_stream(st)
        slot["computed"], slot["copied_out"] = computed, copied_out
        return copied_out

    def synchronize(self) -> None:
        """Wait until every submitted request's output is in host memory."""
        for s in (self.s_in, self.s_compute, self.s_out):
            s.synchronize()
