"""CPU tests of the C ABI: the library loads without a GPU, exports every
function include/llm_fa_b200.h declares, and rejects bad arguments with
status codes before making any CUDA call."""
import ctypes
import re
from pathlib import Path

import pytest

from llm_fa_b200 import _lib
from llm_fa_b200.build import build

HEADER = Path(__file__).resolve().parents[1] / "include" / "llm_fa_b200.h"


@pytest.fixture(scope="module")
def L():
    build()
    return _lib.lib()


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(llmfa_\w+)\s*\(", text)))


def test_header_declares_the_bound_functions():
    assert declared_functions() == sorted(_lib.SIGNATURES)


def test_library_exports_every_declared_symbol(L):
    for name in declared_functions():
        assert hasattr(L, name), name


def test_version_and_error_strings(L):
    assert L.llmfa_version() == 100
    for code in range(7):
        assert _lib.error_string(code)
    assert _lib.error_string(0) == "ok"
    assert "unknown" in _lib.error_string(99)


def _call(L, q=16, k=16, v=16, o=16, qs=(1024 * 128, 128, 128), ks=(1024 * 128, 128, 128),
          B=1, H=1, Sq=1024, Sk=1024, scale=0.088):
    # fake, never-dereferenced addresses: validation fails before any CUDA call
    ptr = lambda a: ctypes.c_void_p(a) if a else None  # noqa: E731
    return L.llmfa_forward(ptr(q), _lib.strides3(qs), ptr(k), _lib.strides3(ks), ptr(v),
                           _lib.strides3(ks), ptr(o), _lib.strides3(qs), B, H, Sq, Sk,
                           ctypes.c_float(scale), None, 0, None)


@pytest.mark.parametrize("kw,code", [
    (dict(q=0), _lib.LLMFA_ERR_INVALID_ARGUMENT),
    (dict(o=0), _lib.LLMFA_ERR_INVALID_ARGUMENT),
    (dict(B=0), _lib.LLMFA_ERR_INVALID_ARGUMENT),
    (dict(Sq=0), _lib.LLMFA_ERR_INVALID_ARGUMENT),
    (dict(Sk=-5), _lib.LLMFA_ERR_INVALID_ARGUMENT),
    (dict(scale=0.0), _lib.LLMFA_ERR_INVALID_ARGUMENT),
    (dict(scale=-1.0), _lib.LLMFA_ERR_INVALID_ARGUMENT),
    (dict(scale=float("nan")), _lib.LLMFA_ERR_INVALID_ARGUMENT),
    (dict(scale=float("inf")), _lib.LLMFA_ERR_INVALID_ARGUMENT),
    (dict(k=24), _lib.LLMFA_ERR_UNSUPPORTED),                       # not 16-byte aligned
    (dict(qs=(1024 * 128, 100, 128)), _lib.LLMFA_ERR_UNSUPPORTED),  # row stride % 8 != 0
    (dict(B=2, qs=(0, 128, 128)), _lib.LLMFA_ERR_UNSUPPORTED),      # zero batch stride
    (dict(Sq=1 << 31), _lib.LLMFA_ERR_UNSUPPORTED),
])
def test_bad_arguments_are_rejected_without_cuda(L, kw, code):
    assert _call(L, **kw) == code


def test_lse_entry_point_rejects_bad_lse_arguments_without_cuda(L):
    ptr = ctypes.c_void_p
    qs = _lib.strides3((1024 * 128, 128, 128))

    def call(lse, lse_strides, B=1, H=1):
        return L.llmfa_forward_lse(ptr(16), qs, ptr(16), qs, ptr(16), qs, ptr(16), qs,
                                   ptr(lse) if lse else None, lse_strides, B, H, 1024, 1024,
                                   ctypes.c_float(0.088), None, 0, None)

    assert call(64, None) == _lib.LLMFA_ERR_INVALID_ARGUMENT              # no strides
    assert call(66, _lib.strides2((1024, 1024))) == _lib.LLMFA_ERR_INVALID_ARGUMENT  # misaligned
    assert call(64, _lib.strides2((0, 1024)), B=2) == _lib.LLMFA_ERR_INVALID_ARGUMENT  # batch stride
    # the shared argument checks still run first
    assert L.llmfa_forward_lse(None, qs, ptr(16), qs, ptr(16), qs, ptr(16), qs, None, None, 1, 1,
                               1024, 1024, ctypes.c_float(0.088), None, 0,
                               None) == _lib.LLMFA_ERR_INVALID_ARGUMENT


def test_static_scratch_entry_point_checks_arguments_without_cuda(L):
    """llmfa_forward_static_scratch refuses invalid arguments with llmfa_forward's status
    codes before its first CUDA call (the device-address lookup of its fixed array)."""
    st = _lib.strides3((1024 * 128, 128, 128))
    p = ctypes.c_void_p(16)
    scale = ctypes.c_float(0.088)

    def call(q=p, k=p, Sq=1024, sc=scale):
        return L.llmfa_forward_static_scratch(q, st, k, st, p, st, p, st, 1, 1, Sq, 1024, sc,
                                              None)

    assert call(q=None) == _lib.LLMFA_ERR_INVALID_ARGUMENT
    assert call(sc=ctypes.c_float(0.0)) == _lib.LLMFA_ERR_INVALID_ARGUMENT
    assert call(Sq=0) == _lib.LLMFA_ERR_INVALID_ARGUMENT
    assert call(k=ctypes.c_void_p(24)) == _lib.LLMFA_ERR_UNSUPPORTED  # not 16-byte aligned


def test_small_helpers_validate(L):
    assert L.llmfa_set_wait_timeout_ms(0) == _lib.LLMFA_ERR_INVALID_ARGUMENT
    assert L.llmfa_device_status(None, None) == _lib.LLMFA_ERR_INVALID_ARGUMENT
    assert L.llmfa_max_active_clusters(None) == _lib.LLMFA_ERR_INVALID_ARGUMENT
    assert L.llmfa_selftest_wait_timeout(0, None) == _lib.LLMFA_ERR_INVALID_ARGUMENT
    assert L.llmfa_workspace_size(None) == _lib.LLMFA_ERR_INVALID_ARGUMENT


def test_python_wrapper_rejects_cpu_tensors():
    import torch

    from llm_fa_b200 import attention_forward
    x = torch.zeros(512, 128, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="CUDA"):
        attention_forward(x, x, x)


def test_product_build_has_no_ablation_or_trace(L):
    """The default library is the product: no ablation-ladder rung, no event trace."""
    cfg = _lib.build_config(L)
    assert cfg == {"ablation": 0, "ablation_name": "none", "trace": 0}
    a, t = ctypes.c_int(-1), ctypes.c_int(-1)
    assert L.llmfa_build_config(None, ctypes.byref(t)) == _lib.LLMFA_ERR_INVALID_ARGUMENT
    assert L.llmfa_build_config(ctypes.byref(a), ctypes.byref(t)) == _lib.LLMFA_OK


def test_ablation_variant_reports_its_rung():
    """A ladder rung is a separate library file that says what it is (no GPU needed)."""
    from llm_fa_b200.build import build_variant
    h = _lib.load(build_variant("floor"))
    assert _lib.build_config(h) == {"ablation": 1, "ablation_name": "floor", "trace": 0}


def test_bench_refuses_an_ablation_build(monkeypatch):
    """bench.py times only the product: a library reporting an ablation rung is refused
    before any GPU work."""
    import argparse

    import llm_fa_b200

    import bench
    from llm_fa_b200.workloads import CONFIGS
    monkeypatch.setattr(llm_fa_b200, "build_info",
                        lambda: {"ablation": 1, "ablation_name": "floor", "trace": 0})
    args = argparse.Namespace(warmup=3, steps=1, no_e2e=True, no_cpu_baseline=True,
                              validate=False, cpu_seconds=1.0)
    with pytest.raises(RuntimeError, match="ablation"):
        bench.run_ours(args, CONFIGS["c1"], 1, 0, 0)
