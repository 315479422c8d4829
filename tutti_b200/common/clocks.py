"""GPU clock and throttle-reason sampling around a timed region.

``ClockSampler(gpus).start()`` runs one ``nvidia-smi -lms 100`` sampler;
``stop()`` returns ``{"sm_mhz": median under load, "sm_max_mhz", "reasons":
[active slowdown reasons], "samples"}``. Reading clocks changes no setting.
"""
from __future__ import annotations

import shutil
import statistics
import subprocess
import threading
import time


class ClockSampler:
    """Samples nvidia-smi clocks/throttle reasons every 100 ms during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus):
        self.gpus = set(gpus)
        self.rows = []
        self._proc = None
        self._t = None

    def start(self):
        if shutil.which("nvidia-smi") is None:
            return self
        # one long-running sampler (-lms) instead of a process per sample
        self._proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                       "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)

        def run():
            for line in self._proc.stdout:
                f = [x.strip() for x in line.split(",")]
                try:
                    if len(f) >= 8 and int(f[0]) in self.gpus:
                        self.rows.append(f)
                except ValueError:
                    continue

        self._t = threading.Thread(target=run, daemon=True)
        self._t.start()
        time.sleep(0.3)  # first sample before the timed region starts
        return self

    def stop(self):
        if self._proc is not None:
            self._proc.terminate()
            try:
                self._proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self._proc.kill()
        if self._t:
            self._t.join(timeout=5)
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4) if r[4 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows)}
