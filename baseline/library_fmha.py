"""A library attention kernel on the same box, for comparison only: flashinfer's CUTLASS
Blackwell FMHA (`flashinfer.prefill.fmha_varlen`, the sm100a `fmha_cutlass_sm100a`
module: tcgen05 MMAs, TMEM accumulators, TMA loads).

The FA4 kernel (`flash_attn.cute`) is not installed in this image; this is the
tcgen05-native attention kernel that is. flashinfer compiles the module just in time
from its CUDA sources; `build()` does that once, offline, into baseline/_fi (about
20 minutes of nvcc on the CPU), and `load()` loads that prebuilt library directly, so
that a GPU run never compiles. Nothing on this repository's product path uses it.

    python -m baseline.library_fmha      # build baseline/_fi
"""
from __future__ import annotations

import os
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
WORKSPACE = ROOT / "baseline" / "_fi"
MODULE = "fmha_cutlass_sm100a"


def _prebuilt() -> Path | None:
    found = sorted(WORKSPACE.glob(f".cache/flashinfer/*/100a/cached_ops/{MODULE}/{MODULE}.so"))
    return found[-1] if found else None


def build() -> Path:
    """Compile flashinfer's sm100a FMHA module (bf16 in and out, head dim 128, no
    positional encoding, no sliding window or logit cap) into baseline/_fi."""
    os.environ["FLASHINFER_WORKSPACE_BASE"] = str(WORKSPACE)
    os.environ.setdefault("FLASHINFER_CUDA_ARCH_LIST", "10.0a")
    import torch
    from flashinfer.jit.attention.modules import gen_fmha_cutlass_sm100a_module
    spec = gen_fmha_cutlass_sm100a_module(torch.bfloat16, torch.bfloat16, torch.bfloat16,
                                          torch.int32, 128, 128, 0, False, False)
    spec.build(verbose=False)
    so = _prebuilt()
    if so is None:
        raise RuntimeError(f"flashinfer build finished but {MODULE}.so is not under {WORKSPACE}")
    return so


class LibraryFMHA:
    """One forward over [B, S, H, 128] bf16 tensors through flashinfer's `fmha_varlen`
    (batch entries as equal-length segments), with its plan and output buffer made once."""

    def __init__(self, q, k, v, scale: float):
        import torch
        so = _prebuilt()
        if so is None:
            raise FileNotFoundError("flashinfer sm100a FMHA not built (python -m baseline.library_fmha)")
        os.environ.setdefault("FLASHINFER_WORKSPACE_BASE", str(WORKSPACE))
        import flashinfer
        import flashinfer.prefill as prefill
        import tvm_ffi
        module = tvm_ffi.load_module(str(so))
        # fmha_varlen looks its module up through get_fmha_module, which would compile
        # (or re-check) the sources; hand it the prebuilt library instead
        prefill.get_fmha_module = lambda *a, **kw: module
        self.version = f"flashinfer {flashinfer.__version__} {MODULE} (CUTLASS sm100 FMHA)"
        B, Sq, H, D = q.shape
        Sk = k.shape[1]
        dev = q.device
        qo = torch.arange(B + 1, device=dev, dtype=torch.int32) * Sq
        kvo = torch.arange(B + 1, device=dev, dtype=torch.int32) * Sk
        plan = prefill.fmha_varlen_plan(module, qo, kvo, H, False)
        # the library's own output allocation: rows before the first segment are writable
        pad = max(Sq, 128)
        out = torch.empty(B * Sq + pad, H, D, device=dev, dtype=q.dtype)[pad:]
        qf = q.contiguous().view(B * Sq, H, D)
        kf = k.contiguous().view(B * Sk, H, D)
        vf = v.contiguous().view(B * Sk, H, D)
        self.out = out.view(B, Sq, H, D)

        def call():
            prefill.fmha_varlen(qf, kf, vf, qo, kvo, plan_info=plan, max_qo_len=Sq, out=out,
                                causal=False, sm_scale=scale)
        self._call = call

    def __call__(self):
        self._call()


if __name__ == "__main__":
    print(build())
