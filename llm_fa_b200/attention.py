"""Torch-facing entry points over the C ABI.

`attention_forward` is the one compute call: bf16 Q/K/V with head dim 128,
either 2-D `(seq, 128)` (the reference's call shape, llm_fa.py:57-65) or 4-D
`[batch, seq, heads, 128]`, non-causal, returns bf16 O in the layout of Q.
PyTorch only supplies device memory and the current stream; the arithmetic is
the sm_100a kernel in libllm_fa_b200.so.
"""
from __future__ import annotations

import contextlib
import ctypes
import functools
import math

import torch

from . import _lib

HEAD_DIM = 128


def _as_bshd(t: torch.Tensor, name: str) -> torch.Tensor:
    if t.dim() == 2:
        return t.unsqueeze(0).unsqueeze(2)  # (S,128) -> (1,S,1,128), a view
    if t.dim() == 4:
        return t
    raise RuntimeError(f"{name} must be 2-D (seq, 128) or 4-D [batch, seq, heads, 128], "
                       f"got shape {tuple(t.shape)}")


def _check(t: torch.Tensor, name: str, device: torch.device) -> None:
    if not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor (there is no CPU path)")
    if t.device != device:
        raise RuntimeError(f"{name} is on {t.device}, expected {device}")
    if t.dtype != torch.bfloat16:
        raise RuntimeError(f"{name} must be bfloat16, got {t.dtype}")
    if t.shape[-1] != HEAD_DIM:
        raise RuntimeError(f"{name} head dim must be {HEAD_DIM}, got {t.shape[-1]}")
    if t.stride(-1) != 1:
        raise RuntimeError(f"{name} head dim must be contiguous (stride 1)")


def attention_forward(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *,
                      softmax_scale: float | None = None,
                      out: torch.Tensor | None = None, return_lse: bool = False):
    """O = softmax(Q K^T * softmax_scale) V on the current CUDA stream.

    softmax_scale defaults to 1/sqrt(128) (the reference's scale,
    validate.py:19-27). `out`, if given, must have Q's shape and be bf16.
    With return_lse, returns (O, lse): the fp32 natural-log log-sum-exp of each
    query row's scaled scores, shaped [B, H, Sq] for 4-D inputs and [Sq] for
    2-D ones (llmfa_forward_lse). Raises RuntimeError on invalid input or a
    nonzero library status.
    """
    return forward_with(_lib.lib(), q, k, v, softmax_scale=softmax_scale, out=out,
                        return_lse=return_lse)


def forward_with(handle, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *,
                 softmax_scale: float | None = None, out: torch.Tensor | None = None,
                 return_lse: bool = False, split_kv: bool = True):
    """attention_forward through one library build: `handle` is the product library or a
    trace/ablation variant loaded with _lib.load. split_kv=False passes no workspace, so
    every 512-row query block runs on one SM pair (the classic schedule)."""
    device = q.device
    for t, nm in ((q, "Q"), (k, "K"), (v, "V")):
        _check(t, nm, device)
    if not (q.dim() == k.dim() == v.dim()):
        raise RuntimeError("Q, K and V must have the same number of dimensions")
    q4, k4, v4 = _as_bshd(q, "Q"), _as_bshd(k, "K"), _as_bshd(v, "V")
    B, Sq, H, _ = q4.shape
    if k4.shape != v4.shape:
        raise RuntimeError(f"K {tuple(k.shape)} and V {tuple(v.shape)} must have the same shape")
    if k4.shape[0] != B or k4.shape[2] != H:
        raise RuntimeError(f"K/V batch and heads {tuple(k4.shape)} do not match Q {tuple(q4.shape)}")
    Sk = k4.shape[1]
    if Sq == 0 or Sk == 0 or B == 0 or H == 0:
        raise RuntimeError("empty Q/K/V are not supported")
    if out is None:
        out = torch.empty_like(q, memory_format=torch.contiguous_format)
    else:
        _check(out, "out", device)
        if out.shape != q.shape:
            raise RuntimeError(f"out shape {tuple(out.shape)} must equal Q shape {tuple(q.shape)}")
    o4 = _as_bshd(out, "out")
    scale = (1.0 / math.sqrt(HEAD_DIM)) if softmax_scale is None else float(softmax_scale)
    # the library launches on the current device: switch only when the tensors live elsewhere
    ctx = (torch.cuda.device(device) if device.index != torch.cuda.current_device()
           else contextlib.nullcontext())
    with ctx:
        # scratch for split KV ranges, from the caching allocator on this stream
        ws_bytes = workspace_size(device) if split_kv else 0
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=device) if split_kv else None
        stream = torch.cuda.current_stream(device).cuda_stream
        lse = torch.empty(B, H, Sq, dtype=torch.float32, device=device) if return_lse else None
        rc = handle.llmfa_forward_lse(
            q4.data_ptr(), _strides3(q4.stride()), k4.data_ptr(), _strides3(k4.stride()),
            v4.data_ptr(), _strides3(v4.stride()), o4.data_ptr(), _strides3(o4.stride()),
            lse.data_ptr() if return_lse else None, _lib.strides2((H * Sq, Sq)),
            B, H, Sq, Sk, scale, ws.data_ptr() if ws is not None else None, ws_bytes, stream)
    _lib.check(rc, "llmfa_forward_lse")
    if return_lse:
        return out, (lse if q.dim() == 4 else lse.reshape(Sq))
    return out


@functools.lru_cache(maxsize=256)
def _strides3(stride: tuple) -> ctypes.Array:
    """(batch, seq, head) element strides of a [B, S, H, 128] view, as the C array type
    (cached: a loop of calls on the same views reuses the converted array)."""
    return _lib.strides3(stride[:3])


_WS_BYTES: dict[int, int] = {}


def workspace_size(device: torch.device | int | None = None) -> int:
    """Bytes of split-KV scratch llmfa_forward can use on `device` (cached per device)."""
    idx = torch.cuda.current_device() if device is None else (
        device if isinstance(device, int) else device.index)
    got = _WS_BYTES.get(idx)
    if got is None:
        out = ctypes.c_uint64(0)
        with torch.cuda.device(idx):
            _lib.check(_lib.lib().llmfa_workspace_size(ctypes.byref(out)), "llmfa_workspace_size")
        got = _WS_BYTES[idx] = int(out.value)
    return got


def device_status(device: torch.device | int | None = None) -> int:
    """Device status word after the current stream drains (0 = no timeout)."""
    dev = torch.device("cuda", torch.cuda.current_device() if device is None else
                       (device if isinstance(device, int) else device.index))
    out = ctypes.c_int(0)
    with torch.cuda.device(dev):
        s = torch.cuda.current_stream(dev).cuda_stream
        _lib.check(_lib.lib().llmfa_device_status(ctypes.byref(out), ctypes.c_void_p(s)),
                   "llmfa_device_status")
    return out.value


def reset_device_status(device: torch.device | int | None = None) -> None:
    dev = torch.device("cuda", torch.cuda.current_device() if device is None else
                       (device if isinstance(device, int) else device.index))
    with torch.cuda.device(dev):
        s = torch.cuda.current_stream(dev).cuda_stream
        _lib.check(_lib.lib().llmfa_reset_device_status(ctypes.c_void_p(s)),
                   "llmfa_reset_device_status")


def set_wait_timeout_ms(ms: int) -> None:
    _lib.check(_lib.lib().llmfa_set_wait_timeout_ms(int(ms)), "llmfa_set_wait_timeout_ms")


def launch_plan(batch: int, heads: int, seq_q: int, seq_k: int,
                workspace_bytes: int | None = None) -> dict:
    """Kernels, clusters and split query blocks of one forward on the current device."""
    if workspace_bytes is None:
        workspace_bytes = workspace_size()
    k, c, s = ctypes.c_int(0), ctypes.c_int(0), ctypes.c_int(0)
    _lib.check(_lib.lib().llmfa_launch_plan(batch, heads, seq_q, seq_k, workspace_bytes,
                                            ctypes.byref(k), ctypes.byref(c), ctypes.byref(s)),
               "llmfa_launch_plan")
    return {"kernels": k.value, "clusters": c.value, "split_units": s.value}


def build_info() -> dict:
    """Compile-time configuration of the loaded library: ablation rung (0 = the product)
    and whether the event trace is compiled in."""
    return _lib.build_config()


def max_active_clusters() -> int:
    out = ctypes.c_int(0)
    _lib.check(_lib.lib().llmfa_max_active_clusters(ctypes.byref(out)), "llmfa_max_active_clusters")
    return out.value


def selftest_wait_timeout(timeout_us: int) -> None:
    """Launch the never-satisfied bounded wait (see include/llm_fa_b200.h)."""
    s = torch.cuda.current_stream().cuda_stream
    _lib.check(_lib.lib().llmfa_selftest_wait_timeout(int(timeout_us), ctypes.c_void_p(s)),
               "llmfa_selftest_wait_timeout")


def attention_flops(batch: int, heads: int, seq_q: int, seq_k: int, head_dim: int = HEAD_DIM) -> int:
    """Algorithmic FLOPs of one forward: two GEMMs, 4*B*H*Sq*Sk*D (softmax not counted)."""
    return 4 * batch * heads * seq_q * seq_k * head_dim
