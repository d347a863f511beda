"""CPU check of bench.py's reference-arm line (without a GPU it times the CPU oracle path):
one JSON line with the contract's keys."""
import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def test_reference_arm_line_on_cpu():
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference",
                          "--config", "c1", "--steps", "1", "--warmup", "0",
                          "--cpu-seconds", "0.3"],
                         capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    line = json.loads(out.stdout.strip().splitlines()[-1])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "higher_is_better",
                "impl", "cpu_baseline", "e2e", "config"):
        assert key in line, key
    assert line["impl"] == "reference" and line["unit"] == "TFLOP/s"
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0
    assert line["cpu_baseline"]["cores"] >= 1 and line["value"] > 0


def test_library_comparison_reports_unavailable_without_its_build(monkeypatch):
    """The same-box library column never fails the bench: without its prebuilt module it
    says why instead."""
    import argparse

    import torch

    sys.path.insert(0, str(ROOT))
    import bench
    from baseline import library_fmha
    monkeypatch.setattr(library_fmha, "_prebuilt", lambda: None)
    x = torch.zeros(1, 256, 1, 128, dtype=torch.bfloat16)
    args = argparse.Namespace(warmup=3, steps=1)
    got = bench.time_library(x, x, x, x, 1, args, None, 1.0)
    assert set(got) == {"unavailable"} and "not built" in got["unavailable"]
