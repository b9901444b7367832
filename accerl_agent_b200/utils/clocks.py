"""Sample SM clocks and throttle reasons with nvidia-smi while a timed region runs."""

from __future__ import annotations

import statistics
import subprocess
import threading
from typing import Dict, List, Optional

QUERY = (
    "index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
    "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
    "clocks_event_reasons.sw_power_cap"
)
REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")


class ClockSampler:
    """``with ClockSampler(gpu_index) as cs: ...`` then ``cs.summary()``."""

    def __init__(self, gpu_index: int = 0, interval_ms: int = 200):
        self.gpu_index = gpu_index
        self.interval_ms = interval_ms
        self.proc: Optional[subprocess.Popen] = None
        self.lines: List[str] = []
        self._thread: Optional[threading.Thread] = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={QUERY}", "--format=csv,noheader,nounits", f"-i={self.gpu_index}",
                 f"-lms={self.interval_ms}"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True,
            )
            self._thread = threading.Thread(target=self._read, daemon=True)
            self._thread.start()
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def _read(self):
        assert self.proc is not None and self.proc.stdout is not None
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        if self._thread is not None:
            self._thread.join(timeout=2)
        return False

    def summary(self) -> Dict:
        sm, mx, power, reasons = [], [], [], set()
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
                power.append(float(parts[3]))
            except ValueError:
                continue
            for name, flag in zip(REASONS, parts[5:9]):
                if flag.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {
            "sm_mhz": statistics.median(sm),
            "sm_max_mhz": max(mx),
            "power_w_max": max(power),
            "reasons": sorted(reasons),
            "samples": len(sm),
        }
