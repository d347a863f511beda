"""Build the in-tree CUDA library `libllm_fa_b200.so` for sm_100a.

One nvcc invocation, no torch dependency in the binary (static cudart); the
driver entry point for tensor-map encoding is resolved at run time, so the
library builds on a machine without a GPU and loads on a machine with one.

    python -m llm_fa_b200.build [--force] [-v] [--variant NAME|all]

Besides the product library, the same source builds variants (compile-time
switches, each in its own library file, never loaded in place of the product):
`trace` (-DLLMFA_TRACE=1: event trace and segment timeline), `waitstats`
(-DLLMFA_TRACE=2: the trace plus per-wait-site statistics, which time every
bounded wait and perturb the schedule more) and the
ablation-ladder rungs `floor`, `faux`, `noexp` (-DLLMFA_ABLATE=1..3: the TMA +
MMA floor, no softmax math, no exponentials; their output is not attention).
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
INCLUDE = PKG.parent / "include"
LIB = PKG / "libllm_fa_b200.so"
SOURCES = [CSRC / "llm_fa_api.cu"]
DEPS = SOURCES + sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-shared", "-Xcompiler", "-fPIC",
    "-Xptxas", "-v",
]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found (set NVCC or put the CUDA toolkit on PATH)")


# variant name -> extra nvcc defines
VARIANTS = {
    "trace": ["-DLLMFA_TRACE=1"],
    "waitstats": ["-DLLMFA_TRACE=2"],
    "floor": ["-DLLMFA_ABLATE=1"],
    "faux": ["-DLLMFA_ABLATE=2"],
    "noexp": ["-DLLMFA_ABLATE=3"],
}


def variant_path(name: str) -> Path:
    return PKG / f"libllm_fa_b200_{name}.so"


# The tensor-core rate microbenchmark (llm_fa_b200.mma_rate): its own source and library.
MMARATE_LIB = PKG / "libllm_fa_b200_mmarate.so"
MMARATE_SOURCES = [CSRC / "mma_rate.cu"]
MMARATE_DEPS = MMARATE_SOURCES + [CSRC / "ptx.cuh"]


def is_stale(lib: Path = LIB, deps: list[Path] = DEPS) -> bool:
    if not lib.exists():
        return True
    t = lib.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile the product library if it is missing or older than its sources."""
    return _compile(LIB, [], force, verbose)


def build_variant(name: str, force: bool = False, verbose: bool = False) -> Path:
    """Compile one variant library (see VARIANTS) if missing or stale."""
    if name not in VARIANTS:
        raise ValueError(f"unknown variant {name!r}; one of {sorted(VARIANTS)}")
    return _compile(variant_path(name), VARIANTS[name], force, verbose)


def build_mmarate(force: bool = False, verbose: bool = False) -> Path:
    """Compile the tensor-core rate microbenchmark library if missing or stale."""
    return _compile(MMARATE_LIB, [], force, verbose, MMARATE_SOURCES, MMARATE_DEPS)


def build_all(force: bool = False, verbose: bool = False) -> list[Path]:
    """The product library, every variant and the microbenchmark, compiled concurrently
    (one nvcc each)."""
    import concurrent.futures
    jobs = [(LIB, [], SOURCES, DEPS)] + [(variant_path(n), d, SOURCES, DEPS)
                                         for n, d in VARIANTS.items()]
    jobs.append((MMARATE_LIB, [], MMARATE_SOURCES, MMARATE_DEPS))
    with concurrent.futures.ThreadPoolExecutor(max_workers=len(jobs)) as pool:
        return list(pool.map(lambda j: _compile(j[0], j[1], force, verbose, j[2], j[3]), jobs))


def _compile(lib: Path, defines: list[str], force: bool, verbose: bool,
             sources: list[Path] = SOURCES, deps: list[Path] = DEPS) -> Path:
    if not force and not is_stale(lib, deps):
        return lib
    tmp = lib.with_name(lib.name + f".{os.getpid()}.tmp")
    cmd = [nvcc_path(), *NVCC_FLAGS, *defines, "-o", str(tmp), *map(str, sources)]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if verbose or proc.returncode != 0:
        sys.stderr.write(proc.stdout + proc.stderr)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed ({proc.returncode}): {' '.join(cmd)}")
    # ptxas -v: report every kernel that spills, by name
    entry = "?"
    for line in (proc.stdout + proc.stderr).splitlines():
        if "Compiling entry function" in line:
            entry = line.split("'")[1] if "'" in line else line.strip()
        elif "spill stores" in line and not line.strip().startswith("0 bytes stack frame, 0 bytes spill"):
            sys.stderr.write(f"warning: {lib.name}: {entry}: ptxas reports {line.strip()}\n")
    os.replace(tmp, lib)
    return lib


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("--variant", choices=[*VARIANTS, "all"])
    a = ap.parse_args()
    if a.variant is None:
        print(build(force=a.force, verbose=a.verbose))
    else:
        for name in (VARIANTS if a.variant == "all" else [a.variant]):
            print(build_variant(name, force=a.force, verbose=a.verbose))
