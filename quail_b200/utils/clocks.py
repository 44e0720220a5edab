"""SM clock and throttle-reason sampling during a timed region (nvidia-smi)."""

from __future__ import annotations

import os
import statistics
import subprocess
import tempfile

QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")


class ClockSampler:
    """Runs `nvidia-smi -lms 200` for one GPU while active; summarizes on stop."""

    def __init__(self, gpu_index: int | None = None, period_ms: int = 200):
        self.gpu = gpu_index
        self.period = period_ms
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(prefix="qb_clocks_", suffix=".csv")
        os.close(fd)
        cmd = ["nvidia-smi", f"--query-gpu={QUERY}", "--format=csv,noheader,nounits", f"-lms={self.period}"]
        if self.gpu is not None:
            cmd.insert(1, f"--id={self.gpu}")
        try:
            self.proc = subprocess.Popen(cmd, stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except (FileNotFoundError, OSError):
            self.proc = None
        return self

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    rows.append((float(parts[1]), float(parts[2]), float(parts[3]), parts[5:9]))
                except ValueError:
                    continue
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        max_mhz = max(r[1] for r in rows)
        loaded = [r for r in rows if r[2] > 200.0] or rows
        reasons = set()
        for r in loaded:
            for name, flag in zip(REASONS, r[3]):
                if flag.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(r[0] for r in loaded), "sm_max_mhz": max_mhz,
                "reasons": sorted(reasons), "samples": len(rows), "samples_under_load": len(loaded),
                "power_w_max": max(r[2] for r in rows)}
