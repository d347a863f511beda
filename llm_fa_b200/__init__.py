"""llm_fa_b200: FlashAttention forward (bf16, head dim 128, non-causal) for B200.

The compute path is the sm_100a kernel in libllm_fa_b200.so behind the C ABI
of include/llm_fa_b200.h; this package is the host-side mirror of the
reference's Python surface (`llm_fa.mod.llm_fa_forward`, `llm_fa.forward`).
"""
from .attention import (HEAD_DIM, attention_flops, attention_forward, build_info,
                        device_status, launch_plan, max_active_clusters, reset_device_status,
                        selftest_wait_timeout, set_wait_timeout_ms, workspace_size)

__all__ = [
    "HEAD_DIM", "attention_flops", "attention_forward", "build_info", "device_status",
    "launch_plan",
    "max_active_clusters", "reset_device_status", "selftest_wait_timeout", "set_wait_timeout_ms",
    "workspace_size",
]
__version__ = "0.1.0"
