"""Generate the golden attention vectors in tests/golden/golden.npz.

Outputs come from the reference's own oracle function `torch_sdpa`
(validate.py:19-27), imported from the reference checkout and run on the CPU
in fp32 on bf16-rounded inputs, one (batch, head) slice at a time (it takes
2-D (q, D) tensors). Inputs are regenerated from seeds by
llm_fa_b200.workloads.make_inputs; an input checksum is stored so that a
change of the generator is detected instead of silently changing the pin.

Run in a checkout that has the reference mounted:
    python tests/golden/make_golden.py /path/to/reference
"""
from __future__ import annotations

import importlib.util
import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
from llm_fa_b200.workloads import CONFIGS, Config, make_inputs, sample_rows  # noqa: E402

# name -> (config, number of sampled query rows or None for all rows)
CASES = {
    "small": (Config("small", 1, 1, 256, 256, seed=100), None),
    "ragged": (Config("ragged", 2, 2, 130, 333, seed=101), 24),
    "stress": (Config("stress", 1, 2, 256, 640, seed=102, stress_rows=True), 32),
    "c1": (CONFIGS["c1"], 64),
}


def load_reference_sdpa(ref_dir: Path):
    spec = importlib.util.spec_from_file_location("ref_validate", ref_dir / "validate.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)  # defines functions only; main() is not run
    return mod.torch_sdpa


def input_checksum(q, k, v) -> np.ndarray:
    return np.array([t.float().double().sum().item() for t in (q, k, v)], dtype=np.float64)


def main() -> None:
    if len(sys.argv) < 2:
        sys.exit("usage: python tests/golden/make_golden.py <reference checkout>")
    ref_dir = Path(sys.argv[1])
    torch_sdpa = load_reference_sdpa(ref_dir)
    out = {}
    for name, (cfg, nrows) in CASES.items():
        q, k, v = make_inputs(cfg)
        rows = sample_rows(cfg, nrows) if nrows else torch.arange(cfg.seq_q)
        o = torch.empty(cfg.batch, len(rows), cfg.heads, cfg.head_dim)
        full_sum = np.zeros((cfg.batch, cfg.heads))
        full_abs = np.zeros((cfg.batch, cfg.heads))
        for b in range(cfg.batch):
            for h in range(cfg.heads):
                ob = torch_sdpa(q[b, :, h].float(), k[b, :, h].float(), v[b, :, h].float())
                o[b, :, h] = ob[rows]
                full_sum[b, h] = ob.double().sum().item()
                full_abs[b, h] = ob.double().abs().sum().item()
        out[f"{name}/config"] = np.array([cfg.batch, cfg.heads, cfg.seq_q, cfg.seq_k, cfg.seed,
                                          int(cfg.stress_rows)], dtype=np.int64)
        out[f"{name}/rows"] = rows.numpy().astype(np.int64)
        out[f"{name}/o"] = o.numpy().astype(np.float32)
        out[f"{name}/o_sum"] = full_sum
        out[f"{name}/o_abs_sum"] = full_abs
        out[f"{name}/input_checksum"] = input_checksum(q, k, v)
        print(f"{name}: {cfg.describe()} rows={len(rows)} o_sum={full_sum.ravel()[:2]}")
    np.savez_compressed(Path(__file__).with_name("golden.npz"), **out)


if __name__ == "__main__":
    main()
