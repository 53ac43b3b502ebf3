"""Samples GPU clocks and throttle reasons with nvidia-smi during a timed region.

Reading clocks is harmless; nothing here changes a GPU setting.
"""
from __future__ import annotations

import os
import shutil
import signal
import statistics
import subprocess
import tempfile
from typing import Dict, List, Optional

_FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
           "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
           "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
_REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")


class ClockSampler:
    """``with ClockSampler(gpu) as c: ...`` then ``c.summary()``."""

    def __init__(self, gpu: int, period_ms: int = 200):
        self.gpu = gpu
        self.period_ms = period_ms
        self.proc: Optional[subprocess.Popen] = None
        self.path = ""

    def __enter__(self) -> "ClockSampler":
        if shutil.which("nvidia-smi") is None:
            return self
        fd, self.path = tempfile.mkstemp(prefix="cail_clocks_", suffix=".csv")
        os.close(fd)
        self.proc = subprocess.Popen(
            ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={_FIELDS}", "--format=csv,noheader,nounits",
             "-lms", str(self.period_ms)],
            stdout=open(self.path, "w"), stderr=subprocess.DEVNULL, start_new_session=True)
        return self

    def __exit__(self, *exc) -> None:
        if self.proc is not None:
            self.proc.send_signal(signal.SIGTERM)
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def samples(self) -> List[List[str]]:
        if not self.path or not os.path.exists(self.path):
            return []
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        return rows

    def summary(self) -> Optional[Dict]:
        rows = self.samples()
        if self.path and os.path.exists(self.path):
            os.unlink(self.path)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        reasons = set()
        for r in rows:
            for name, val in zip(_REASONS, r[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(rows)}
