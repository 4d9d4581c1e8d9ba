"""GPU clock / throttle sampling during a timed region (reads only).

Runs ``nvidia-smi --query-gpu=... -lms 200`` in the background and summarises
the samples: median SM clock under load, max clock, and the throttle reasons
that were active. Nothing here changes a GPU setting.
"""
from __future__ import annotations

import os
import statistics
import subprocess
import tempfile

FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,utilization.gpu,clocks_event_reasons.active,"
          "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
          "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")


class ClockSampler:
    def __init__(self, gpu_index: int | None = None, period_ms: int = 200):
        self.gpu = gpu_index
        self.period = period_ms
        self.proc = None
        self.path = None

    def __enter__(self):
        self.start()
        return self

    def __exit__(self, *a):
        self.stop()

    def start(self):
        fd, self.path = tempfile.mkstemp(prefix="clocks_", suffix=".csv")
        os.close(fd)
        cmd = ["nvidia-smi", f"--query-gpu={FIELDS}", "--format=csv,noheader,nounits", f"-lms={self.period}"]
        if self.gpu is not None:
            cmd.insert(1, f"--id={self.gpu}")
        try:
            self.proc = subprocess.Popen(cmd, stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except (FileNotFoundError, OSError):
            self.proc = None

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict | None:
        if self.path is None or not os.path.exists(self.path):
            return None
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 10:
                    continue
                try:
                    rows.append(dict(sm=float(parts[1]), smax=float(parts[2]), util=float(parts[4] or 0),
                                     flags={r: parts[6 + i] == "Active" for i, r in enumerate(REASONS)}))
                except ValueError:
                    continue
        os.unlink(self.path)
        if not rows:
            return None
        loaded = [r for r in rows if r["util"] > 10] or rows
        reasons = sorted({k for r in loaded for k, v in r["flags"].items() if v})
        return {"sm_mhz": statistics.median(r["sm"] for r in loaded), "sm_max_mhz": max(r["smax"] for r in rows),
                "reasons": reasons, "samples": len(rows)}
