"""Seeded synthetic inputs for the configurations the reference is measured on.

Inputs are drawn on the CPU with `torch.Generator().manual_seed(seed)` so the
CPU oracle, every GPU rank and every run see identical tensors (the reference
draws on the GPU RNG, validate.py:57-60, which cannot be replayed on a CPU).
Draw order: q, k, v, each `torch.randn(B, S, H, 128)` in fp32 then rounded to
bf16. For the softmax-stress configuration, after the three draws, q and then
k get round(0.05*S) rows per (batch, head) multiplied by 4, the rows chosen by
`torch.randperm(S)` from the same generator (batch-major, head-minor order).
No public dataset is involved; these stand in for the reference's random
single-head inputs (bench.py:63-76) at the benchmark configurations' shapes.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class Config:
    name: str
    batch: int
    heads: int
    seq_q: int
    seq_k: int
    seed: int
    stress_rows: bool = False  # scale 5% of q and k rows by 4 (online-max stress)
    head_dim: int = 128

    @property
    def scale(self) -> float:
        return 1.0 / math.sqrt(self.head_dim)

    @property
    def flops(self) -> int:
        return 4 * self.batch * self.heads * self.seq_q * self.seq_k * self.head_dim

    @property
    def io_bytes(self) -> int:
        """Algorithmic HBM bytes: read Q, K, V once, write O once (bf16)."""
        return 2 * self.head_dim * self.batch * self.heads * (2 * self.seq_q + 2 * self.seq_k)

    def describe(self) -> str:
        return (f"B{self.batch} H{self.heads} Sq{self.seq_q} Sk{self.seq_k} D{self.head_dim} "
                f"seed{self.seed}{' stress' if self.stress_rows else ''}")


# The benchmark configurations c1..c5, in order.
CONFIGS = {
    "c1": Config("c1", 1, 2, 1024, 1024, seed=0),
    "c2": Config("c2", 1, 1, 16384, 16384, seed=1),
    "c3": Config("c3", 1, 1, 32768, 131072, seed=2),
    "c4": Config("c4", 4, 32, 8192, 8192, seed=3),
    "c5": Config("c5", 1, 64, 32768, 32768, seed=4, stress_rows=True),
}


def make_inputs(cfg: Config, dtype: torch.dtype = torch.bfloat16):
    """(q, k, v) on the CPU, [B, S, H, D], rounded to bf16 (returned as `dtype`)."""
    g = torch.Generator().manual_seed(cfg.seed)
    B, H, D = cfg.batch, cfg.heads, cfg.head_dim
    q = torch.randn(B, cfg.seq_q, H, D, generator=g).to(torch.bfloat16)
    k = torch.randn(B, cfg.seq_k, H, D, generator=g).to(torch.bfloat16)
    v = torch.randn(B, cfg.seq_k, H, D, generator=g).to(torch.bfloat16)
    if cfg.stress_rows:
        for t, S in ((q, cfg.seq_q), (k, cfg.seq_k)):
            nrows = int(round(0.05 * S))
            for b in range(B):
                for h in range(H):
                    rows = torch.randperm(S, generator=g)[:nrows]
                    t[b, rows, h, :] = (t[b, rows, h, :].float() * 4.0).to(torch.bfloat16)
    if dtype != torch.bfloat16:
        q, k, v = q.to(dtype), k.to(dtype), v.to(dtype)
    return q, k, v


def sample_rows(cfg: Config, n: int, salt: int = 1000) -> torch.Tensor:
    """A seeded, sorted subset of query rows (rows are independent in attention)."""
    g = torch.Generator().manual_seed(cfg.seed + salt)
    n = min(n, cfg.seq_q)
    return torch.randperm(cfg.seq_q, generator=g)[:n].sort().values


def shard_heads(batch: int, heads: int, world: int, rank: int) -> list[tuple[int, int]]:
    """Contiguous block of (batch, head) pairs owned by `rank` (no exchange needed)."""
    total = batch * heads
    lo = (total * rank) // world
    hi = (total * (rank + 1)) // world
    return [(i // heads, i % heads) for i in range(lo, hi)]
