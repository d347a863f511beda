"""ctypes binding of the C ABI in include/llm_fa_b200.h.

The shared library is the only compute path: if it is missing or cannot be
loaded, every entry point raises instead of falling back to anything else.
"""
from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libllm_fa_b200.so"

# status codes (include/llm_fa_b200.h)
LLMFA_OK = 0
LLMFA_ERR_INVALID_ARGUMENT = 1
LLMFA_ERR_UNSUPPORTED = 2
LLMFA_ERR_TENSOR_MAP = 3
LLMFA_ERR_LAUNCH = 4
LLMFA_ERR_CUDA = 5
LLMFA_ERR_DEVICE_TIMEOUT = 6
DEVICE_STATUS_TIMEOUT_BASE = 0x1000

_I64x3 = ctypes.c_int64 * 3
_I64x2 = ctypes.c_int64 * 2
_lock = threading.Lock()
_lib = None

# name -> (restype, argtypes); every function declared in include/llm_fa_b200.h
SIGNATURES = {
    "llmfa_forward": (ctypes.c_int, [
        ctypes.c_void_p, _I64x3, ctypes.c_void_p, _I64x3, ctypes.c_void_p, _I64x3,
        ctypes.c_void_p, _I64x3, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
        ctypes.c_int64, ctypes.c_float, ctypes.c_void_p, ctypes.c_uint64, ctypes.c_void_p]),
    "llmfa_forward_lse": (ctypes.c_int, [
        ctypes.c_void_p, _I64x3, ctypes.c_void_p, _I64x3, ctypes.c_void_p, _I64x3,
        ctypes.c_void_p, _I64x3, ctypes.c_void_p, ctypes.POINTER(ctypes.c_int64),
        ctypes.c_int64, ctypes.c_int64,
        ctypes.c_int64, ctypes.c_int64, ctypes.c_float, ctypes.c_void_p, ctypes.c_uint64,
        ctypes.c_void_p]),
    "llmfa_workspace_size": (ctypes.c_int, [ctypes.POINTER(ctypes.c_uint64)]),
    "llmfa_forward_static_scratch": (ctypes.c_int, [
        ctypes.c_void_p, _I64x3, ctypes.c_void_p, _I64x3, ctypes.c_void_p, _I64x3,
        ctypes.c_void_p, _I64x3, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
        ctypes.c_int64, ctypes.c_float, ctypes.c_void_p]),
    "llmfa_forward_2d": (ctypes.c_int, [
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
        ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p, ctypes.c_uint64, ctypes.c_void_p]),
    "llmfa_device_status": (ctypes.c_int, [ctypes.POINTER(ctypes.c_int), ctypes.c_void_p]),
    "llmfa_reset_device_status": (ctypes.c_int, [ctypes.c_void_p]),
    "llmfa_set_wait_timeout_ms": (ctypes.c_int, [ctypes.c_uint32]),
    "llmfa_max_active_clusters": (ctypes.c_int, [ctypes.POINTER(ctypes.c_int)]),
    "llmfa_launch_plan": (ctypes.c_int, [ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                         ctypes.c_int64, ctypes.c_uint64,
                                         ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int),
                                         ctypes.POINTER(ctypes.c_int)]),
    "llmfa_error_string": (ctypes.c_char_p, [ctypes.c_int]),
    "llmfa_version": (ctypes.c_int, []),
    "llmfa_build_config": (ctypes.c_int, [ctypes.POINTER(ctypes.c_int),
                                          ctypes.POINTER(ctypes.c_int)]),
    "llmfa_selftest_wait_timeout": (ctypes.c_int, [ctypes.c_uint32, ctypes.c_void_p]),
    "llmfa_trace_read": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_uint64,
                                        ctypes.POINTER(ctypes.c_uint64)]),
}


class LlmfaError(RuntimeError):
    """A nonzero llmfa status code."""

    def __init__(self, code: int, what: str):
        self.code = code
        super().__init__(f"{what}: {error_string(code)} (status {code})")


def load(path: Path | str) -> ctypes.CDLL:
    """Load one build of the library (the product, or a trace/ablation variant built by
    llm_fa_b200.build.build_variant) as its own handle, with every signature set."""
    path = Path(path)
    if not path.exists():
        raise ImportError(f"{path.name} is not built; run `python -m llm_fa_b200.build` "
                          "(there is no non-CUDA fallback)")
    handle = ctypes.CDLL(str(path), mode=os.RTLD_NOW | os.RTLD_LOCAL)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(handle, name)
        fn.restype = res
        fn.argtypes = args
    return handle


def lib() -> ctypes.CDLL:
    """Load the product library once; raise if it is not there."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                _lib = load(LIB_PATH)
    return _lib


ABLATION_NAMES = {0: "none", 1: "floor", 2: "faux", 3: "noexp"}


def build_config(handle: ctypes.CDLL | None = None) -> dict:
    """Compile-time configuration of a library build (llmfa_build_config)."""
    h = lib() if handle is None else handle
    a, t = ctypes.c_int(-1), ctypes.c_int(-1)
    check(h.llmfa_build_config(ctypes.byref(a), ctypes.byref(t)), "llmfa_build_config")
    return {"ablation": a.value, "ablation_name": ABLATION_NAMES.get(a.value, str(a.value)),
            "trace": t.value}


def error_string(code: int) -> str:
    return lib().llmfa_error_string(int(code)).decode()


def check(code: int, what: str) -> None:
    if code != LLMFA_OK:
        raise LlmfaError(code, what)


def strides3(st) -> ctypes.Array:
    return _I64x3(*[int(x) for x in st])


def strides2(st) -> ctypes.Array:
    return _I64x2(*[int(x) for x in st])
