"""Measured tcgen05.mma rates of the operand forms the attention kernel issues.

    python -m llm_fa_b200.mma_rate [--n-mma 2048]

Runs the microbenchmark of csrc/mma_rate.cu (its own library file,
libllm_fa_b200_mmarate.so): per form, one warp of each issuing CTA issues
`n_mma` MMAs back to back (one elected lane per instruction, as the attention
kernel issues them), on one CTA pair and on every SM at once. Prints one JSON
line per form and grid: SM cycles per MMA from the first issue to completion,
cycles per MMA spent issuing, the cycles the first eight issues took (from an
idle tensor pipe), and multiply-accumulates per cycle per SM; once from unrolled
groups of eight MMAs with their descriptors in registers (the tensor pipe's own
rate) and once from a rolled loop that selects the form and builds the
descriptors at run time for every MMA (what a longer issue path costs).

The attention kernel's two forms are QK (A = the Q tile from shared memory)
and PV (A = P from tensor memory); the others show how the rate of the shared-
memory form changes with the CTA group and N.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import statistics

import torch

from .build import build_mmarate

# form -> (description, M, N, CTAs per MMA)
FORMS = {
    0: ("QK: SS cta_group::2 M=256 N=128 (A Q tile, B K tile, both shared memory)", 256, 128, 2),
    1: ("PV: TS cta_group::2 M=256 N=128 (A P in tensor memory, B V tile)", 256, 128, 2),
    2: ("SS cta_group::1 M=128 N=128", 128, 128, 1),
    3: ("SS cta_group::2 M=256 N=256", 256, 256, 2),
    4: ("SS cta_group::2 M=256 N=64", 256, 64, 2),
    5: ("SS cta_group::2 M=256 N=128, B MN-major (PV's V layout, A from shared memory)", 256, 128, 2),
}
K_STEP = 16  # bf16 K per MMA


def _lib() -> ctypes.CDLL:
    h = ctypes.CDLL(str(build_mmarate()))
    h.llmfa_mma_rate.restype = ctypes.c_int
    h.llmfa_mma_rate.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                 ctypes.c_void_p, ctypes.c_void_p]
    return h


def measure(form: int, n_mma: int, ctas: int, handle: ctypes.CDLL | None = None,
            runtime_loop: bool = False) -> dict:
    """One launch of `form` on `ctas` CTAs; statistics over the issuing CTAs. With
    `runtime_loop` the MMAs come from a rolled loop that selects the form and builds the
    descriptors at run time (a longer issue path per MMA)."""
    h = handle or _lib()
    desc, m, n, cg = FORMS[form]
    out = torch.zeros(4 * ctas, dtype=torch.int64, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    rc = h.llmfa_mma_rate(form, n_mma, ctas, int(runtime_loop), ctypes.c_void_p(out.data_ptr()),
                          ctypes.c_void_p(stream))
    if rc != 0:
        raise RuntimeError(f"llmfa_mma_rate(form {form}) launch failed: cudaError {rc}")
    torch.cuda.synchronize()
    res = out.view(ctas, 4).cpu()
    issuing = res[::cg]
    if bool(issuing[:, 3].any()):
        raise RuntimeError(f"form {form}: an MMA completion wait gave up")
    total = [int(x) for x in issuing[:, 0]]
    cyc = statistics.median(total) / n_mma
    macs_per_sm = m * n * K_STEP / cg  # each SM of the group computes M / cg rows
    return {"form": form, "what": desc, "ctas": ctas, "n_mma": n_mma,
            "issue_loop": "rolled, run-time form" if runtime_loop else "unrolled, descriptors in registers",
            "cycles_per_mma": round(cyc, 2),
            "cycles_per_mma_max": round(max(total) / n_mma, 2),
            "issue_cycles_per_mma": round(statistics.median(int(x) for x in issuing[:, 1]) / n_mma, 2),
            "first8_issue_cycles": int(statistics.median(int(x) for x in issuing[:, 2])),
            "macs_per_cycle_per_sm": round(macs_per_sm / cyc, 1)}


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--n-mma", type=int, default=2048)
    a = ap.parse_args()
    h = _lib()
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    for form in FORMS:
        measure(form, 64, 2, h)  # warm-up: module load, first launch
        for rolled in (False, True):
            for ctas in (2, sms - sms % 2):
                print(json.dumps(measure(form, a.n_mma, ctas, h, rolled)), flush=True)


if __name__ == "__main__":
    main()
