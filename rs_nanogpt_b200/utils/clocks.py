"""Samples GPU clocks and throttle reasons with nvidia-smi while a timed
region runs (read-only queries; no GPU setting is changed)."""
import statistics
import subprocess
import tempfile
from typing import Dict, Optional

FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
          "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
          "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
REASONS = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]


class ClockSampler:
    def __init__(self, interval_ms: int = 200):
        self.interval_ms = interval_ms
        self.proc: Optional[subprocess.Popen] = None
        self.file = None

    def __enter__(self):
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={FIELDS}", "--format=csv,noheader,nounits", "-lms", str(self.interval_ms)],
                stdout=self.file, stderr=subprocess.DEVNULL)
        except (OSError, ValueError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> Dict:
        if self.proc is None or self.file is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        self.file.flush()
        with open(self.file.name) as f:
            rows = [r.split(", ") for r in f.read().strip().splitlines() if r.count(",") >= 8]
        sm, smax, reasons = [], None, set()
        for r in rows:
            try:
                sm.append(float(r[1]))
                smax = float(r[2])
            except ValueError:
                continue
            for name, val in zip(REASONS, r[5:9]):
                if val.strip() == "Active":
                    reasons.add(name)
        load = [s for s in sm if smax and s > 0.5 * smax] or sm
        return {"sm_mhz": statistics.median(load) if load else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}
