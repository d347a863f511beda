"""Drop-in mirror of the reference module `llm_fa.py` (llm_fa.py:37-78).

Same names and meaning:
  * `mod.llm_fa_forward(Q, K, V)` -> `[O, prof_buf, prof_count]`
    (llm_fa.cu:1418-1475): prof_buf is int32 (16384*6,), prof_count int32 (1,),
    both zero (the reference's values too unless built with ENABLE_PROF=1);
  * `forward(Q, K, V)` -> O (llm_fa.py:57-65);
  * `run(q, sk, seed)` draws Q/K/V with `torch.manual_seed(seed)` on the GPU
    and returns the 3-list (llm_fa.py:68-78).

Differences, all supersets: Q/K/V may also be 4-D [B, S, H, 128]; any q >= 1
and sk >= 1 are accepted (the reference requires q % 512 == 0, sk % 128 == 0,
sk >= 256); the call is stream-ordered instead of ending in
cudaDeviceSynchronize. Errors raise RuntimeError, as TORCH_CHECK does.
"""
from __future__ import annotations

import torch

from .attention import attention_forward

PROF_MAX_EVENTS = 16384  # reference profiler ring capacity (llm_fa.cu, prof_buf size / 6)


class _Module:
    """Stands in for the JIT-built pybind module `mod` of the reference."""

    def __init__(self) -> None:
        self._placeholders: dict[torch.device, tuple[torch.Tensor, torch.Tensor]] = {}

    def _prof(self, device: torch.device):
        ph = self._placeholders.get(device)
        if ph is None:
            ph = (torch.zeros(PROF_MAX_EVENTS * 6, dtype=torch.int32, device=device),
                  torch.zeros(1, dtype=torch.int32, device=device))
            self._placeholders[device] = ph
        return ph

    def llm_fa_forward(self, Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor):
        O = attention_forward(Q, K, V)
        prof_buf, prof_count = self._prof(Q.device)
        return [O, prof_buf, prof_count]


mod = _Module()


def forward(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor) -> torch.Tensor:
    """Full attention forward: O = softmax(Q K^T / sqrt(128)) V."""
    return mod.llm_fa_forward(Q, K, V)[0]


def run(q: int = 32768, sk: int = 131072, seed: int = 0):
    """Random Q/K/V of the given shape (GPU RNG, as the reference), one call."""
    torch.manual_seed(seed)
    Q = torch.randn(q, 128, device="cuda", dtype=torch.bfloat16)
    K = torch.randn(sk, 128, device="cuda", dtype=torch.bfloat16)
    V = torch.randn(sk, 128, device="cuda", dtype=torch.bfloat16)
    return mod.llm_fa_forward(Q, K, V)
