"""Build the reference's kernels from their own sources into oracle/_ref/.

TEST AND COMPARISON INFRASTRUCTURE ONLY. The reference's path is one CUDA file plus
one header (llm_fa.cu, profiler.cuh) compiled as a torch extension with the
flags of llm_fa.py:46-51; its ablation-ladder kernels scaffolding.cu and
faux.cu (scaffolding.py, faux.py) are built the same way. This recipe compiles
those files where they lie in the reference checkout (nothing is copied into
this repository) together with oracle/ref_binding.cpp, a pybind binding of
each launcher written here, and keeps only the resulting
`oracle/_ref/<name>*.so` (git-ignored; they travel to the GPU box with the
working tree).

Users: bench.py --impl reference (the reference arm) and the GPU tests (the
reference's validate.py run against this repository's mirror module).
"""
from __future__ import annotations

import os
import shutil
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"


def reference_dir() -> Path | None:
    """The reference checkout: $LLMFA_REFERENCE_DIR, else the `reference_path` that the
    repository's BASELINE.json records; None when neither names an existing directory."""
    cand = os.environ.get("LLMFA_REFERENCE_DIR")
    if not cand:
        try:
            import json
            cand = json.loads((HERE.parent / "BASELINE.json").read_text()).get("reference_path")
        except (OSError, ValueError):
            cand = None
    if cand and Path(cand).is_dir():
        return Path(cand)
    return None


# module name -> (reference source, launcher, extra defines), as the reference's own
# launch modules build them (llm_fa.py, scaffolding.py, faux.py)
REF_MODULES = {
    "llm_fa_ref": ("llm_fa.cu", "llm_fa_forward", []),
    "scaffolding_ref": ("scaffolding.cu", "redist_v6_forward", ["-DSKIP_SM_FULL=0"]),
    "faux_ref": ("faux.cu", "fa4_faux_attn_forward", []),
}


def built_module_path(name: str = "llm_fa_ref") -> Path | None:
    hits = sorted(OUT.glob(f"{name}*.so"))
    return hits[0] if hits else None


def build(ref_dir: Path, name: str = "llm_fa_ref", verbose: bool = False) -> Path:
    from torch.utils.cpp_extension import load as _load_and_import

    source, launcher, defines = REF_MODULES[name]
    src = ref_dir / source
    if not src.exists():
        raise FileNotFoundError(src)
    build_dir = OUT / f"build_{name}"
    build_dir.mkdir(parents=True, exist_ok=True)
    try:
        _load_and_import(
            name=name,
            sources=[str(HERE / "ref_binding.cpp"), str(src)],
            extra_cflags=[f"-DREF_FN={launcher}"],
            extra_cuda_cflags=["-O3", "-gencode=arch=compute_100a,code=sm_100a",
                               "--use_fast_math", "-std=c++17", "-lineinfo", "-DENABLE_PROF=0",
                               *defines, f"-I{ref_dir}"],
            extra_ldflags=["-lcuda"],
            build_directory=str(build_dir),
            verbose=verbose,
            is_python_module=True,
        )
    except ImportError:
        pass  # built, but this machine has no driver (libcuda) to import it with
    hits = sorted(build_dir.glob(f"{name}*.so"))
    if not hits:
        raise RuntimeError(f"reference extension {name} build produced no module")
    so = hits[0]
    dst = OUT / so.name
    shutil.copy2(so, dst)
    shutil.rmtree(build_dir)  # objects and generated build files stay out of the tree
    return dst


def build_if_possible() -> Path | None:
    """Build every reference module that is missing, when the reference checkout is
    present; returns the llm_fa_ref module path (or None)."""
    import concurrent.futures
    import multiprocessing

    ref = reference_dir()
    todo = [name for name, (source, _, _) in REF_MODULES.items()
            if built_module_path(name) is None and ref is not None and (ref / source).exists()]
    if todo:
        # one process per module (each is a separate extension build in its own directory)
        with concurrent.futures.ProcessPoolExecutor(
                max_workers=len(todo), mp_context=multiprocessing.get_context("spawn")) as pool:
            futures = {name: pool.submit(build, ref, name) for name in todo}
            for name, fut in futures.items():
                try:
                    fut.result()
                except Exception as exc:  # the comparison baselines are optional; the product is not
                    sys.stderr.write(f"reference module {name} not built: {exc}\n")
    return built_module_path("llm_fa_ref")


def load_module(name: str = "llm_fa_ref"):
    """Import one built reference extension (pybind module `name`, see REF_MODULES)."""
    import importlib.machinery
    import importlib.util

    import torch  # noqa: F401  (the extension links against libtorch)

    so = built_module_path(name)
    if so is None:
        raise ImportError(f"reference module {name} not built (oracle/build_ref.py)")
    loader = importlib.machinery.ExtensionFileLoader(name, str(so))
    spec = importlib.util.spec_from_loader(name, loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    ref = Path(sys.argv[1]) if len(sys.argv) > 1 else reference_dir()
    if ref is None:
        sys.exit("usage: python oracle/build_ref.py <reference checkout> "
                 "(or set LLMFA_REFERENCE_DIR)")
    for name in REF_MODULES:
        print(build(ref, name, verbose=True))
