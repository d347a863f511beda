"""The tensor-core rate microbenchmark (llm_fa_b200.mma_rate, csrc/mma_rate.cu): its
library builds and rejects bad arguments without a GPU; on a GPU every form completes
with a per-MMA time in a plausible range."""
import ctypes

import pytest

from llm_fa_b200 import mma_rate


def test_mma_rate_library_rejects_bad_arguments_without_cuda():
    h = mma_rate._lib()
    out = ctypes.c_void_p(16)
    invalid = 1  # cudaErrorInvalidValue
    assert h.llmfa_mma_rate(6, 64, 2, 0, out, None) == invalid      # no such form
    assert h.llmfa_mma_rate(0, 0, 2, 0, out, None) == invalid       # no MMAs
    assert h.llmfa_mma_rate(0, 12, 2, 0, out, None) == invalid      # not whole 8-MMA groups
    assert h.llmfa_mma_rate(0, 64, 3, 0, out, None) == invalid      # pairs need an even grid
    assert h.llmfa_mma_rate(2, 64, 1, 0, None, None) == invalid     # no output


@pytest.mark.gpu
@pytest.mark.parametrize("form", sorted(mma_rate.FORMS))
@pytest.mark.parametrize("rolled", [False, True])
def test_mma_rate_forms_complete(form, rolled):
    r = mma_rate.measure(form, 512, 2, runtime_loop=rolled)
    # an MMA of these shapes takes tens of cycles at least, and far fewer than 1000
    assert 16 <= r["cycles_per_mma"] <= 1000, r
    assert r["issue_cycles_per_mma"] <= r["cycles_per_mma"] * 1.05, r
