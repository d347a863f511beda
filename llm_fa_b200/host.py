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


class _Slot:
    """One set of device buffers and the events that order its reuse."""

    def __init__(self, q_shape, kv_shape, device):
        mk = lambda shape: torch.empty(shape, dtype=torch.bfloat16, device=device)  # noqa: E731
        self.key = (q_shape, kv_shape)
        self.q, self.k, self.v, self.o = mk(q_shape), mk(kv_shape), mk(kv_shape), mk(q_shape)
        self.copied_in = torch.cuda.Event()
        self.computed = torch.cuda.Event()
        self.copied_out = torch.cuda.Event()
        self.used = False


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
        self._slots: list[_Slot | None] = [None] * depth
        self._n = 0

    def _slot(self, i: int, q, k) -> _Slot:
        key = (tuple(q.shape), tuple(k.shape))
        slot = self._slots[i]
        if slot is None or slot.key != key:
            if slot is not None:
                # The old buffers come from the caching allocator on the current stream;
                # work queued on the three streams may still use them, so they must not be
                # handed out again before it has finished.
                for buf, streams in ((slot.q, (self.s_in, self.s_compute)),
                                     (slot.k, (self.s_in, self.s_compute)),
                                     (slot.v, (self.s_in, self.s_compute)),
                                     (slot.o, (self.s_compute, self.s_out))):
                    for st in streams:
                        buf.record_stream(st)
            with torch.cuda.device(self.device):
                slot = _Slot(key[0], key[1], self.device)
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
        if k.shape != v.shape:
            raise RuntimeError(f"K {tuple(k.shape)} and V {tuple(v.shape)} must have the same shape")
        slot = self._slot(self._n % self.depth, q, k)
        self._n += 1
        s_in, s_c, s_out = self.s_in, self.s_compute, self.s_out
        with torch.cuda.device(self.device):
            # copy in, once the compute that last read this slot's inputs is done
            if slot.used:
                s_in.wait_event(slot.computed)
            with torch.cuda.stream(s_in):
                slot.q.copy_(q, non_blocking=True)
                slot.k.copy_(k, non_blocking=True)
                slot.v.copy_(v, non_blocking=True)
            slot.copied_in.record(s_in)
            # compute, once the inputs landed and the slot's last output was copied out
            s_c.wait_event(slot.copied_in)
            if slot.used:
                s_c.wait_event(slot.copied_out)
            with torch.cuda.stream(s_c):
                attention_forward(slot.q, slot.k, slot.v, out=slot.o,
                                  softmax_scale=softmax_scale)
            slot.computed.record(s_c)
            # copy out
            s_out.wait_event(slot.computed)
            with torch.cuda.stream(s_out):
                out.copy_(slot.o, non_blocking=True)
            slot.copied_out.record(s_out)
            done = torch.cuda.Event()
            done.record(s_out)
        slot.used = True
        return done

    def synchronize(self) -> None:
        """Wait until every submitted request's output is in host memory."""
        for s in (self.s_in, self.s_compute, self.s_out):
            s.synchronize()
