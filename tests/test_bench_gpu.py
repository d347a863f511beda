"""GPU check of bench.py's comparison sweep on one small shape: this kernel, the same
kernel on the reference's grid, the reference kernel (built from its sources into
oracle/_ref) and the optional library kernel all run, and the row reports each of them."""
import argparse
import json
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
pytestmark = pytest.mark.gpu


def test_sweep_row_on_one_small_shape(monkeypatch, capsys):
    from oracle.build_ref import built_module_path
    if built_module_path("llm_fa_ref") is None:
        pytest.skip("reference kernel module not built (oracle/build_ref.py)")
    sys.path.insert(0, str(ROOT))
    import bench
    monkeypatch.setattr(bench, "SWEEP_SHAPES", [(1024, 2048)])
    bench.run_sweep(argparse.Namespace(steps=2, warmup=1))
    rows = [json.loads(line) for line in capsys.readouterr().out.splitlines()
            if line.startswith("{")]
    assert len(rows) == 1
    r = rows[0]
    for key in ("ours_us", "reference_us", "ours_on_reference_grid_us", "speedup",
                "speedup_on_reference_grid", "max_abs_diff_vs_reference", "library"):
        assert key in r, key
    assert r["ours_us"] > 0 and r["reference_us"] > 0 and r["ours_on_reference_grid_us"] > 0
    # both kernels compute the same attention (bf16 outputs, parity-level agreement)
    assert r["max_abs_diff_vs_reference"] < 2e-2
    lib = r["library"]
    assert "unavailable" in lib or (lib["us"] > 0 and lib["max_abs_diff_vs_this_kernel"] < 2e-2)
