"""CPU oracle for the attention forward — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg (and its
`--impl reference` CPU arm) may import this module, and only as the checker or
the timed CPU baseline; the product path (llm_fa_b200) never calls it.

The reference's semantics for its path is torch's scaled_dot_product_attention,
non-causal, scale 1/sqrt(D) (validate.py:19-27, the `torch_sdpa` reference of
`report`, validate.py:30-42); its kernel computes the same
softmax(Q K^T * scale) V with an online softmax (llm_fa.cu:805-1060,
1348-1406). Two restatements are kept:

* `sdpa_fp32` — torch SDPA on the CPU in fp32 on bf16-rounded inputs: the
  reference's own oracle path, run on host cores (configuration c1's method);
* `attention_np` — an independent numpy restatement of the math
  (max-subtracted exp, row sum, divide) in float64, used to pin `sdpa_fp32`.

Parity is pinned by tests/golden/*.npz, produced by tests/golden/make_golden.py
from the reference's own oracle path; the reference ships no golden vectors
or known-answer files of its own.
"""
from __future__ import annotations

import math

import numpy as np
import torch
import torch.nn.functional as F


def sdpa_fp32(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float | None = None,
              rows: torch.Tensor | None = None) -> torch.Tensor:
    """O in fp32 for [B,S,H,D] (or 2-D (S,D)) inputs; optional subset of query rows.

    Follows validate.py:19-27: F.scaled_dot_product_attention(..., is_causal=False,
    scale=1/sqrt(D)) on [B,H,S,D] views, here in fp32 on CPU tensors.
    """
    two_d = q.dim() == 2
    if two_d:
        q, k, v = q[None, :, None], k[None, :, None], v[None, :, None]
    D = q.shape[-1]
    scale = 1.0 / math.sqrt(D) if scale is None else scale
    if rows is not None:
        q = q[:, rows]
    qh = q.float().permute(0, 2, 1, 3)
    kh = k.float().permute(0, 2, 1, 3)
    vh = v.float().permute(0, 2, 1, 3)
    o = F.scaled_dot_product_attention(qh, kh, vh, is_causal=False, scale=scale)
    o = o.permute(0, 2, 1, 3).contiguous()
    return o[0, :, 0] if two_d else o


def attention_np(q: np.ndarray, k: np.ndarray, v: np.ndarray, scale: float) -> np.ndarray:
    """float64 softmax(q k^T * scale) v for [B,S,H,D] float arrays."""
    q = q.astype(np.float64)
    k = k.astype(np.float64)
    v = v.astype(np.float64)
    B, Sq, H, D = q.shape
    out = np.empty((B, Sq, H, D), dtype=np.float64)
    for b in range(B):
        for h in range(H):
            s = (q[b, :, h] @ k[b, :, h].T) * scale
            s -= s.max(axis=1, keepdims=True)
            p = np.exp(s)
            out[b, :, h] = (p @ v[b, :, h]) / p.sum(axis=1, keepdims=True)
    return out


def compare(out: torch.Tensor, ref: torch.Tensor) -> dict:
    """max/mean absolute error of `out` (any dtype) against fp32 `ref`."""
    d = (out.float().cpu() - ref.float().cpu()).abs()
    return {"max_abs": float(d.max()), "mean_abs": float(d.mean()),
            "nonfinite": int((~torch.isfinite(out.float().cpu())).sum())}


# Parity tolerances on O: max-abs 2e-2, mean-abs 2e-3.
MAX_ABS_TOL = 2e-2
MEAN_ABS_TOL = 2e-3
