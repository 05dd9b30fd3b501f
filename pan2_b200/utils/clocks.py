"""Background ``nvidia-smi`` sampler of SM clocks and throttle reasons (read-only queries)."""
from __future__ import annotations

import csv
import io
import statistics
import subprocess
from typing import Dict, List, Optional

FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
          "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
          "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")


class ClockSampler:
    def __init__(self, interval_ms: int = 200):
        self.interval_ms = interval_ms
        self.proc: Optional[subprocess.Popen] = None

    def start(self) -> None:
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={FIELDS}", "--format=csv,noheader,nounits",
                                          f"-lms", str(self.interval_ms)], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except (FileNotFoundError, OSError):
            self.proc = None

    def stop(self, gpus: Optional[List[int]] = None) -> Dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=10)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        rows = list(csv.reader(io.StringIO(out)))
        sm, smax, reasons, power = [], [], set(), []
        for r in rows:
            if len(r) < 9:
                continue
            try:
                idx = int(r[0])
            except ValueError:
                continue
            if gpus is not None and idx not in gpus:
                continue
            try:
                pw = float(r[3])
                clk = float(r[1])
            except ValueError:
                continue
            power.append(pw)
            sm.append((pw, clk))
            try:
                smax.append(float(r[2]))
            except ValueError:
                pass
            for name, val in zip(REASONS, r[5:9]):
                if val.strip().lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        # "under load": samples drawing at least half of the peak power seen
        peak = max(p for p, _ in sm)
        loaded = [c for p, c in sm if p >= 0.5 * peak] or [c for _, c in sm]
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm), "power_w_max": peak}
