"""Background ``nvidia-smi`` sampler of SM clocks and throttle reasons (read-only queries)."""
from __future__ import annotations

import csv
import io
import statistics
import subprocess
from typing import Dict, List, Optional

FIELDS = ("index,uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
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
        """Summary of the samples of this process's visible CUDA devices (matched by UUID, so the
        physical GPUs behind ``CUDA_VISIBLE_DEVICES`` are the ones reported); ``gpus`` lists the
        visible device ordinals to include (all visible devices by default)."""
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=10)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        rows = [r for r in csv.reader(io.StringIO(out)) if len(r) >= 10]
        wanted = _visible_uuids(gpus)
        if wanted is not None and not any(r[1].strip().lower() in wanted for r in rows):
            wanted = None  # UUIDs not comparable here: fall back to the nvidia-smi indices
        idx_ok = set(gpus) if gpus is not None else None
        sm, smax, reasons, power = [], [], set(), []
        for r in rows:
            if wanted is not None:
                if r[1].strip().lower() not in wanted:
                    continue
            elif idx_ok is not None:
                try:
                    if int(r[0]) not in idx_ok:
                        continue
                except ValueError:
                    continue
            try:
                pw = float(r[4])
                clk = float(r[2])
            except ValueError:
                continue
            power.append(pw)
            sm.append((pw, clk))
            try:
                smax.append(float(r[3]))
            except ValueError:
                pass
            for name, val in zip(REASONS, r[6:10]):
                if val.strip().lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        # "under load": samples drawing at least half of the peak power seen
        peak = max(p for p, _ in sm)
        loaded = [c for p, c in sm if p >= 0.5 * peak] or [c for _, c in sm]
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm), "power_w_max": peak}


def _visible_uuids(gpus: Optional[List[int]]) -> Optional[set]:
    """``nvidia-smi`` UUID strings (``gpu-...``) of the given visible CUDA ordinals, or None when
    they cannot be read (then every sampled GPU counts)."""
    try:
        import torch
        if not torch.cuda.is_available():
            return None
        ordinals = gpus if gpus is not None else list(range(torch.cuda.device_count()))
        out = set()
        for d in ordinals:
            if d >= torch.cuda.device_count():
                continue
            out.add("gpu-" + str(torch.cuda.get_device_properties(d).uuid).lower())
        return out or None
    except Exception:  # noqa: BLE001 - sampling is best effort
        return None
