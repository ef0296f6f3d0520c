"""Clock and throttle sampling during a timed region (read-only).

:class:`NvmlSampler` polls NVML from a background thread every few
milliseconds (SM clock, its maximum, power, utilization and the active
clock event reasons), so a timed region of ~100 ms still yields dozens of
samples; :class:`ClockSampler` runs ``nvidia-smi ... -lms`` instead, for
machines without NVML bindings. Both report the median SM clock under load,
the maximum clock and every clock event reason seen active, restricted to
the window marked with :meth:`mark_start` / :meth:`mark_end` when one was
marked. Nothing here changes a GPU setting.
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


Sample = tuple[float, "float | None", "float | None", "float | None", "float | None", int]


def summarize(samples: list, window: tuple[float, float] | None = None, source: str = "") -> dict:
    """Median SM clock under load, max clock, reasons seen; over `window` (monotonic seconds) if given."""
    in_window = None
    if window is not None:
        inside = [s for s in samples if window[0] <= s[0] <= window[1]]
        in_window = len(inside)
        samples = inside or samples
    if not samples:
        return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0, "note": "no clock samples"}
    loaded = [s for s in samples if (s[4] or 0) >= 50] or samples
    sm = [s[1] for s in loaded if s[1] is not None]
    mx = [s[2] for s in samples if s[2] is not None]
    mask = 0
    for s in loaded:
        mask |= s[5]
    reasons = sorted(name for bit, name in REASONS.items() if mask & bit and name != "gpu_idle")
    out = {
        "sm_mhz": statistics.median(sm) if sm else None,
        "sm_max_mhz": max(mx) if mx else None,
        "reasons": reasons,
        "samples": len(samples),
        "samples_under_load": len(loaded),
        "power_w_max": max((s[3] for s in loaded if s[3] is not None), default=None),
        "rejecting_reason_seen": bool(set(reasons) & REJECTING),
    }
    if in_window is not None:
        out["samples_in_timed_region"] = in_window
    if source:
        out["source"] = source
    return out


class _Window:
    def __init__(self) -> None:
        self._t0: float | None = None
        self._t1: float | None = None

    def mark_start(self) -> None:
        self._t0 = time.monotonic()

    def mark_end(self) -> None:
        self._t1 = time.monotonic()

    def window(self) -> tuple[float, float] | None:
        return (self._t0, self._t1) if self._t0 is not None and self._t1 is not None else None


class NvmlSampler(_Window):
    """Background NVML poller for the GPU with this UUID (or NVML index)."""

    def __init__(self, uuid: str | None, index: int, interval_ms: float = 5.0) -> None:
        super().__init__()
        self.uuid, self.index, self.interval = uuid, index, interval_ms / 1000.0
        self.samples: list[Sample] = []
        self._stop = threading.Event()
        self._thread: threading.Thread | None = None
        self._nvml = None
        self._handle = None

    def start(self) -> "NvmlSampler":
        import pynvml

        pynvml.nvmlInit()
        self._nvml = pynvml
        h = None
        if self.uuid:
            try:
                h = pynvml.nvmlDeviceGetHandleByUUID(self.uuid)
            except pynvml.NVMLError:
                h = None
        self._handle = h if h is not None else pynvml.nvmlDeviceGetHandleByIndex(self.index)
        self._max = float(pynvml.nvmlDeviceGetMaxClockInfo(self._handle, pynvml.NVML_CLOCK_SM))
        reasons_fn = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            pynvml.nvmlDeviceGetCurrentClocksThrottleReasons
        self._reasons = reasons_fn
        self._thread = threading.Thread(target=self._run, daemon=True)
        self._thread.start()
        return self

    def _run(self) -> None:
        nv, h = self._nvml, self._handle
        while not self._stop.is_set():
            try:
                sm = float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM))
                pw = nv.nvmlDeviceGetPowerUsage(h) / 1000.0
                util = float(nv.nvmlDeviceGetUtilizationRates(h).gpu)
                mask = int(self._reasons(h))
                self.samples.append((time.monotonic(), sm, self._max, pw, util, mask))
            except nv.NVMLError:
                pass
            self._stop.wait(self.interval)

    def stop(self) -> dict:
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=5)
        try:
            self._nvml.nvmlShutdown()
        except Exception:  # noqa: BLE001 - shutdown is best effort
            pass
        return summarize(self.samples, self.window(), "nvml")


def start_sampler(device_index: int) -> "NvmlSampler | ClockSampler":
    """An NVML sampler for this CUDA device when NVML is usable, else nvidia-smi."""
    uuid = None
    try:
        import torch

        u = torch.cuda.get_device_properties(device_index).uuid
        uuid = f"GPU-{u}"
    except Exception:  # noqa: BLE001 - fall back to the index
        uuid = None
    try:
        return NvmlSampler(uuid, device_index).start()
    except Exception:  # noqa: BLE001 - no NVML bindings or library here
        return ClockSampler(device_index).start()


class ClockSampler(_Window):
    """Background nvidia-smi sampler for one GPU index."""

    def __init__(self, index: int, interval_ms: int = 50) -> None:
        super().__init__()
        self.index = index
        self.interval_ms = interval_ms
        self.samples: list[Sample] = []
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
        return summarize(self.samples, self.window(), "nvidia-smi")
