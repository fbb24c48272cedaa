"""Sample GPU clocks and throttle reasons while a timed region runs.

A background ``nvidia-smi --query-gpu ... -lms`` process writes CSV lines;
``summary()`` reports the median SM clock under load, the max SM clock and
every throttle reason seen active. Reading settings only: nothing here
changes a GPU setting.
"""

from __future__ import annotations

import shutil
import statistics
import subprocess
import tempfile

FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,utilization.gpu,clocks_event_reasons.active,"
          "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
          "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")


class ClockSampler:
    def __init__(self, gpus: str | None = None, interval_ms: int = 200):
        self.gpus = gpus
        self.interval_ms = interval_ms
        self.proc = None
        self.out = None

    def start(self) -> "ClockSampler":
        exe = shutil.which("nvidia-smi")
        if exe is None:
            return self
        self.out = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        cmd = [exe, f"--query-gpu={FIELDS}", "--format=csv,noheader,nounits", f"-lms={self.interval_ms}"]
        if self.gpus:
            cmd.append(f"--id={self.gpus}")
        self.proc = subprocess.Popen(cmd, stdout=self.out, stderr=subprocess.DEVNULL)
        return self

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:  # pragma: no cover
            self.proc.kill()
        self.out.flush()
        self.out.seek(0)
        return summarize(self.out.read())


def summarize(csv_text: str) -> dict:
    sm, sm_load, smax, reasons, n = [], [], [], set(), 0
    for line in csv_text.strip().splitlines():
        parts = [p.strip() for p in line.split(",")]
        if len(parts) < 10:
            continue
        try:
            clk, mx, util = float(parts[1]), float(parts[2]), float(parts[4])
        except ValueError:
            continue
        n += 1
        sm.append(clk)
        smax.append(mx)
        if util >= 50:
            sm_load.append(clk)
        for name, val in zip(REASONS, parts[6:10]):
            if val.lower() == "active":
                reasons.add(name)
    src = sm_load or sm
    return {
        "sm_mhz": statistics.median(src) if src else None,
        "sm_max_mhz": max(smax) if smax else None,
        "reasons": sorted(reasons),
        "samples": n,
        "samples_under_load": len(sm_load),
    }
