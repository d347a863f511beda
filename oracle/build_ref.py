"""Build the reference kernel (llm_fa.cu) from its own sources into oracle/_ref/.

TEST/BASELINE INFRASTRUCTURE ONLY. The reference's path is one CUDA file plus
one header (llm_fa.cu, profiler.cuh) compiled as a torch extension with the
flags of llm_fa.py:46-51. This recipe compiles those files where they lie in
the reference checkout (nothing is copied into this repository) together with
oracle/ref_binding.cpp, a pybind binding of its `llm_fa_forward` written
here, and keeps only the resulting `oracle/_ref/llm_fa_ref*.so`
(git-ignored; it travels to the GPU box with the working tree).

Users: bench.py --impl reference (the reference arm) and the GPU tests.
"""
from __future__ import annotations

import os
import shutil
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"
DEFAULT_REF = Path(os.environ.get("LLMFA_REFERENCE_DIR", "/root/reference"))


def built_module_path() -> Path | None:
    hits = sorted(OUT.glob("llm_fa_ref*.so"))
    return hits[0] if hits else None


def build(ref_dir: Path = DEFAULT_REF, verbose: bool = False) -> Path:
    from torch.utils.cpp_extension import load as _load_and_import

    src = ref_dir / "llm_fa.cu"
    if not src.exists():
        raise FileNotFoundError(src)
    build_dir = OUT / "build"
    build_dir.mkdir(parents=True, exist_ok=True)
    try:
        _load_and_import(
        name="llm_fa_ref",
        sources=[str(HERE / "ref_binding.cpp"), str(src)],
        extra_cuda_cflags=["-O3", "-gencode=arch=compute_100a,code=sm_100a", "--use_fast_math",
                           "-std=c++17", "-lineinfo", "-DENABLE_PROF=0", f"-I{ref_dir}"],
        extra_ldflags=["-lcuda"],
        build_directory=str(build_dir),
        verbose=verbose,
        is_python_module=True,
        )
    except ImportError:
        pass  # built, but this machine has no driver (libcuda) to import it with
    hits = sorted(build_dir.glob("llm_fa_ref*.so"))
    if not hits:
        raise RuntimeError("reference extension build produced no module")
    so = hits[0]
    dst = OUT / so.name
    shutil.copy2(so, dst)
    shutil.rmtree(build_dir)  # objects and generated build files stay out of the tree
    return dst


def build_if_possible() -> Path | None:
    """Build when the reference checkout is present and the module is missing."""
    have = built_module_path()
    if have is not None or not (DEFAULT_REF / "llm_fa.cu").exists():
        return have
    try:
        return build()
    except Exception as exc:  # the comparison baseline is optional; the product is not
        sys.stderr.write(f"reference kernel not built: {exc}\n")
        return None


def load_module():
    """Import the built reference extension (pybind module `llm_fa_ref`)."""
    import importlib.machinery
    import importlib.util

    import torch  # noqa: F401  (the extension links against libtorch)

    so = built_module_path()
    if so is None:
        raise ImportError("reference kernel not built (oracle/build_ref.py)")
    loader = importlib.machinery.ExtensionFileLoader("llm_fa_ref", str(so))
    spec = importlib.util.spec_from_loader("llm_fa_ref", loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    print(build(Path(sys.argv[1]) if len(sys.argv) > 1 else DEFAULT_REF, verbose=True))
