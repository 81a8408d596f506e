"""Clock sampling for benchmarks.

``ClockSampler`` runs ``nvidia-smi`` in the background during a timed region
(read-only queries; no GPU setting is changed) and summarizes the SM clock
under load and any active throttle reasons.
"""

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
    def __init__(self, interval_ms: int = 200, gpus: list[int] | None = None):
        self.interval_ms = interval_ms
        self.gpus = gpus
        self.proc = None
        self.path = None
        self._out = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        cmd = ["nvidia-smi", f"--query-gpu={QUERY}", "--format=csv,noheader,nounits",
               "-lms", str(self.interval_ms)]
        if self.gpus is not None:
            cmd[1:1] = ["-i", ",".join(str(g) for g in self.gpus)]
        try:
            self._out = open(self.path, "w")
            self.proc = subprocess.Popen(cmd, stdout=self._out, stderr=subprocess.DEVNULL)
        except (FileNotFoundError, OSError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        if self._out is not None:
            self._out.close()
        return False

    def summary(self) -> dict:
        rows = []
        if self.path and os.path.exists(self.path):
            with open(self.path) as f:
                for line in f:
                    parts = [p.strip() for p in line.split(",")]
                    if len(parts) < 9:
                        continue
                    try:
                        power = float(parts[3]) if parts[3] not in ("[N/A]", "") else 0.0
                        rows.append({"sm": float(parts[1]), "max": float(parts[2]), "power": power,
                                     **{r: parts[5 + i] == "Active" for i, r in enumerate(REASONS)}})
                    except ValueError:
                        continue
            os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        loaded = [r for r in rows if r["power"] > 200.0] or rows
        reasons = sorted({r for row in loaded for r in REASONS if row[r]})
        return {"sm_mhz": statistics.median(r["sm"] for r in loaded), "sm_max_mhz": max(r["max"] for r in rows),
                "reasons": reasons, "samples": len(rows), "samples_under_load": len(loaded),
                "power_w_max": max(r["power"] for r in rows)}
