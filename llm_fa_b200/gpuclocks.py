"""SM clock and throttle-reason samples of one GPU while a timed region runs.

Used by bench.py and the ladder tool to report the clocks a measurement saw
(a number taken under thermal or hardware slowdown, or with the SM clock held
below its maximum, is not comparable). It only reads nvidia-smi samples; it
changes no GPU setting.
"""
from __future__ import annotations

import os
import statistics
import subprocess


class ClockSampler:
    """nvidia-smi samples (200 ms) of one GPU while the timed region runs.

    nvidia-smi writes its samples to a file (`-f`), read after the timed region: a
    Python thread reading a pipe would take the interpreter lock during the timed
    steps and delay their launches."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []
        self.path = None

    def start(self):
        import tempfile
        fd, self.path = tempfile.mkstemp(prefix="llmfa_clocks_", suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200", "-f", self.path],
                stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
        except (OSError, ValueError):
            self.proc = None

    def stop(self) -> dict | None:
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        try:
            with open(self.path) as f:
                self.lines = [ln.strip() for ln in f]
            os.unlink(self.path)
        except OSError:
            self.lines = []
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[0]))
                mx.append(float(parts[1]))
            except ValueError:
                continue
            for nm, val in zip(names, parts[4:8]):
                if val.lower() == "active":
                    reasons.add(nm)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}
