"""nvidia-smi clock and throttle sampling during a timed region (read-only).

Starts ``nvidia-smi ... -lms`` in the background, keeps the samples, and
reports the median SM clock under load, the maximum clock and every clock
event reason seen active. Nothing here changes a GPU setting.
"""

from __future__ import annotations

import shutil
import statistics
import subprocess
import threading
import time

FIELDS = (
    "index,clocks.sm,clocks.max.sm,power.draw,utilization.gpu,clocks_event_reasons.active"
)

#: Bits of ``clocks_event_reasons.active`` (NVML's documented reason masks).
REASONS = {
    0x1: "gpu_idle",
    0x2: "applications_clocks_setting",
    0x4: "sw_power_cap",
    0x8: "hw_slowdown",
    0x20: "sw_thermal_slowdown",
    0x40: "hw_thermal_slowdown",
    0x80: "hw_power_brake_slowdown",
    0x100: "display_clock_setting",
}
REJECTING = {"hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "hw_power_brake_slowdown"}


def _num(v: str) -> float | None:
    try:
        return float(v.strip())
    except ValueError:
        return None


class ClockSampler:
    """Background sampler for one GPU index."""

    def __init__(self, index: int, interval_ms: int = 50) -> None:
        self.index = index
        self.interval_ms = interval_ms
        self.samples: list[tuple[float, float | None, float | None, float | None, float | None, int]] = []
        self._proc: subprocess.Popen | None = None
        self._thread: threading.Thread | None = None

    def start(self) -> "ClockSampler":
        exe = shutil.which("nvidia-smi")
        if exe is None:
            return self
        self._proc = subprocess.Popen(
            [exe, f"--query-gpu={FIELDS}", "--format=csv,noheader,nounits", "-i", str(self.index),
             f"-lms={self.interval_ms}"],
            stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True,
        )
        self._thread = threading.Thread(target=self._read, daemon=True)
        self._thread.start()
        return self

    def _read(self) -> None:
        assert self._proc is not None and self._proc.stdout is not None
        for line in self._proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 6:
                continue
            try:
                mask = int(parts[5], 16) if parts[5].lower().startswith("0x") else int(parts[5])
            except ValueError:
                mask = 0
            self.samples.append((time.monotonic(), _num(parts[1]), _num(parts[2]), _num(parts[3]),
                                 _num(parts[4]), mask))

    def stop(self) -> dict:
        if self._proc is not None:
            self._proc.terminate()
            try:
                self._proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self._proc.kill()
        if self._thread is not None:
            self._thread.join(timeout=5)
        return self.summary()

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0, "note": "no nvidia-smi samples"}
        loaded = [s for s in self.samples if (s[4] or 0) >= 50] or self.samples
        sm = [s[1] for s in loaded if s[1] is not None]
        mx = [s[2] for s in self.samples if s[2] is not None]
        mask = 0
        for s in loaded:
            mask |= s[5]
        reasons = sorted(name for bit, name in REASONS.items() if mask & bit and name != "gpu_idle")
        return {
            "sm_mhz": statistics.median(sm) if sm else None,
            "sm_max_mhz": max(mx) if mx else None,
            "reasons": reasons,
            "samples": len(self.samples),
            "samples_under_load": len(loaded),
            "power_w_max": max((s[3] for s in loaded if s[3] is not None), default=None),
            "rejecting_reason_seen": bool(set(reasons) & REJECTING),
        }
