"""CPU emulation of the kernel's numerics (test helper, numpy float32).

Follows llm_fa_b200/csrc/fa_fwd_kernel.cuh step by step for one (batch,
head): 128-key tiles; row max of the raw scores times scale*log2(e); lazy
rescale only when the max grows by more than 8 (log2 units); exponentials
exp2(s*c - m) with the columns the kernel sends to the FMA-pipe polynomial
evaluated by the same polynomial (softmax_exp2.cuh); P rounded to bf16
before P@V; fp32 row sums of the exponentials plus, per tile, the bf16
rounding of the tile's largest one (computed as the kernel computes that
element); final O/l in bf16.
Lets the CPU suite check the algorithm (and the polynomial) against the
oracle without a GPU.
"""
from __future__ import annotations

import numpy as np

C0 = np.float32(float.fromhex("0x1.fff692p-1"))
C1 = np.float32(float.fromhex("0x1.62f31ap-1"))
C2 = np.float32(float.fromhex("0x1.f0de1ap-3"))
C3 = np.float32(float.fromhex("0x1.c3f76p-5"))
MAGIC = np.float32(12582912.0)
RESCALE_THRESHOLD = np.float32(8.0)
# pairs (within each 32-column chunk) that use the polynomial: the kernel's default
# (LLMFA_SOFTMAX_POLY_MASK in fa_fwd_kernel.cuh)
POLY_MASK = 0x0080


def bf16_round(x: np.ndarray) -> np.ndarray:
    """float32 -> nearest-even bf16 -> float32."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32)


def _fma32(a, b, c):
    return (a.astype(np.float64) * b + c).astype(np.float32)


def exp2_poly(x: np.ndarray) -> np.ndarray:
    """The kernel's FMA-pipe exp2 (softmax_exp2.cuh) in float32 arithmetic."""
    x = np.maximum(np.asarray(x, dtype=np.float32), np.float32(-125.0))
    t = (x + MAGIC).astype(np.float32)
    jf = (t - MAGIC).astype(np.float32)
    f = (x - jf).astype(np.float32)
    p = _fma32(np.full_like(f, C3), f, C2)
    p = _fma32(p, f, C1)
    p = _fma32(p, f, C0)
    bits = (p.view(np.uint32).astype(np.uint64) + (t.view(np.uint32).astype(np.uint64) << 23))
    return (bits & 0xFFFFFFFF).astype(np.uint32).view(np.float32)


def poly_columns(mask: int = POLY_MASK) -> np.ndarray:
    cols = np.zeros(128, dtype=bool)
    for c in range(4):
        for k in range(16):
            if (mask >> k) & 1:
                cols[32 * c + 2 * k] = cols[32 * c + 2 * k + 1] = True
    return cols


def attention_kernel_emulation(q: np.ndarray, k: np.ndarray, v: np.ndarray,
                               scale: float, poly_mask: int = POLY_MASK) -> np.ndarray:
    """q (Sq,D), k/v (Sk,D) float32 (bf16-valued) -> O (Sq,D) float32 (bf16-valued).

    `poly_mask` selects the column pairs whose exp2 uses the polynomial (0xFFFF
    sends every column through it, which stresses the polynomial)."""
    q = q.astype(np.float32)
    k = k.astype(np.float32)
    v = v.astype(np.float32)
    Sq, D = q.shape
    Sk = k.shape[0]
    c = np.float32(scale * 1.4426950408889634)
    m = np.zeros(Sq, np.float32)
    l = np.zeros(Sq, np.float32)
    o = np.zeros((Sq, D), np.float32)
    polyc = poly_columns(poly_mask)
    n_kv = (Sk + 127) // 128
    for j in range(n_kv):
        kt = k[128 * j:128 * (j + 1)]
        vt = v[128 * j:128 * (j + 1)]
        s = np.full((Sq, 128), -np.inf, np.float32)
        s[:, :kt.shape[0]] = q @ kt.T
        mt = (s.max(axis=1) * c).astype(np.float32)
        if j == 0:
            m = mt
        else:
            grow = mt > m + RESCALE_THRESHOLD
            sc = np.where(grow, np.exp2(m - mt), np.float32(1.0)).astype(np.float32)
            m = np.where(grow, mt, m)
            l = (l * sc).astype(np.float32)
            o = (o * sc[:, None]).astype(np.float32)
        x = _fma32(s, np.full_like(s, c), -m[:, None])
        e = np.exp2(x).astype(np.float32)
        e[:, polyc] = exp2_poly(x[:, polyc])
        l = (l + e.sum(axis=1, dtype=np.float32)).astype(np.float32)
        # the bf16 rounding of each row's largest probability of the tile (dominant_rounding)
        smax = s.max(axis=1)
        xmax = _fma32(smax, np.full_like(smax, c), -m)
        in_poly = (s[:, polyc] == smax[:, None]).any(axis=1)
        pm = np.where(in_poly, exp2_poly(xmax), np.exp2(xmax)).astype(np.float32)
        l = (l + (bf16_round(pm) - pm)).astype(np.float32)
        p = bf16_round(e)
        vpad = np.zeros((128, D), np.float32)
        vpad[:vt.shape[0]] = vt
        o = (o + p @ vpad).astype(np.float32)
    return bf16_round(o / l[:, None])
