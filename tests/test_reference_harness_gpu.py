"""The reference's own validation harness, run unchanged against this repository.

`validate.py` (validate.py:44-66) imports `scaffolding`, `faux` and `llm_fa`,
draws Q/K/V of 4096 x 128 with the GPU RNG, runs the two ladder kernels (their
output is intentionally wrong; it only prints them) and checks `llm_fa.forward`
against bf16 torch SDPA, printing PASS below a max-abs error of 5e-3
(validate.py:30-42). Here `llm_fa` is this repository's drop-in mirror module
(llm_fa_b200.llm_fa) and `scaffolding` / `faux` expose the reference's own
ladder kernels, built from its sources by oracle/build_ref.py (the same
launchers its scaffolding.py / faux.py build just in time).

The harness is read from the reference installed into baseline/_ref (the
offline `pip install --target baseline/_ref` of the reference package, whose
modules include validate.py) or from the checkout named by the environment
variable LLMFA_REFERENCE_DIR; without either, or without the prebuilt ladder
modules, the test is skipped.
"""
import importlib.util
import os
import re
import sys
import types
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]


def _harness_dir() -> Path | None:
    for cand in (os.environ.get("LLMFA_REFERENCE_DIR"), ROOT / "baseline" / "_ref"):
        if cand and (Path(cand) / "validate.py").exists():
            return Path(cand)
    return None


def _ladder_module(name: str, launcher: str) -> types.ModuleType:
    """A stand-in for the reference's scaffolding.py / faux.py: the same `forward`
    (Q, K, V) -> O over the same kernel, prebuilt instead of built just in time."""
    from oracle.build_ref import load_module
    ext = load_module(f"{name}_ref")
    mod = types.ModuleType(name)
    mod.forward = lambda Q, K, V: getattr(ext, launcher)(Q, K, V)[0]
    return mod


def test_reference_validate_py_passes_with_the_mirror_module(monkeypatch, capsys):
    from oracle.build_ref import built_module_path
    harness = _harness_dir()
    if harness is None:
        pytest.skip("reference harness (validate.py) not installed")
    if built_module_path("scaffolding_ref") is None or built_module_path("faux_ref") is None:
        pytest.skip("reference ladder modules not built (oracle/build_ref.py)")
    from llm_fa_b200 import llm_fa as mirror

    # sys.modules and sys.path are restored after the test (validate.py prepends its own
    # directory to sys.path when imported)
    monkeypatch.setattr(sys, "path", list(sys.path))
    for name, mod in (("llm_fa", mirror),
                      ("scaffolding", _ladder_module("scaffolding", "redist_v6_forward")),
                      ("faux", _ladder_module("faux", "fa4_faux_attn_forward"))):
        monkeypatch.setitem(sys.modules, name, mod)
    spec = importlib.util.spec_from_file_location("ref_validate_harness", harness / "validate.py")
    validate = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(validate)
    monkeypatch.setattr(sys, "argv", ["validate.py"])  # its defaults: q = sk = 4096, seed 0
    validate.main()
    out = capsys.readouterr().out
    sys.stdout.write(out)
    assert "=== scaffolding ===" in out and "=== faux ===" in out
    section = out.split("=== llm_fa ===", 1)[1]
    assert re.search(r"status\s*:\s*PASS", section), section
    max_abs = float(re.search(r"max_abs vs ref\s*:\s*(\S+)", section).group(1))
    assert max_abs < 5e-3
