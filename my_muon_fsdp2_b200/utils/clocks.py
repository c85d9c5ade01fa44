"""Sample GPU SM clocks and throttle reasons with ``nvidia-smi`` while a region runs (read-only)."""
from __future__ import annotations

import os
import shutil
import statistics
import subprocess
import tempfile
from typing import Dict, List, Optional

FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
          "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
          "clocks_event_reasons.sw_power_cap")
REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")


def physical_gpu_index(local_device: int) -> int:
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        parts = [p.strip() for p in vis.split(",") if p.strip()]
        if local_device < len(parts) and parts[local_device].isdigit():
            return int(parts[local_device])
    return local_device


class ClockSampler:
    def __init__(self, gpu_index: int, period_ms: int = 200):
        self.gpu_index = gpu_index
        self.period_ms = period_ms
        self.proc: Optional[subprocess.Popen] = None
        self._file = None

    def start(self) -> None:
        if shutil.which("nvidia-smi") is None:
            return
        self._file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.proc = subprocess.Popen(
            ["nvidia-smi", f"--query-gpu={FIELDS}", "--format=csv,noheader,nounits", f"-lms={self.period_ms}",
             f"--id={self.gpu_index}"], stdout=self._file, stderr=subprocess.DEVNULL)

    def stop(self) -> Dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:  # pragma: no cover
            self.proc.kill()
        self._file.flush()
        self._file.seek(0)
        rows = [r.strip() for r in self._file.read().splitlines() if r.strip()]
        self._file.close()
        os.unlink(self._file.name)
        return summarize(rows)


def _active(v: str) -> bool:
    return v.strip().lower() in ("active", "1", "yes", "true")


def summarize(rows: List[str]) -> Dict:
    sm, mx, power, reasons = [], [], [], set()
    for r in rows:
        parts = [p.strip() for p in r.split(",")]
        if len(parts) < 9:
            continue
        try:
            sm.append(float(parts[1]))
            mx.append(float(parts[2]))
            power.append(float(parts[3]))
        except ValueError:
            continue
        for name, val in zip(REASONS, parts[5:9]):
            if _active(val):
                reasons.add(name)
    if not sm:
        return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "samples": 0}
    # "under load": samples at or above the 25th percentile (drops idle edges of the window)
    srt = sorted(sm)
    cut = srt[len(srt) // 4]
    loaded = [s for s in sm if s >= cut]
    return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
            "samples": len(sm), "power_w_max": max(power) if power else None}
