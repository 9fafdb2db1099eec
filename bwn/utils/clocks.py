"""Sample SM clocks and throttle reasons with ``nvidia-smi`` while a timed
region runs (read-only queries; no GPU setting is changed)."""
from __future__ import annotations

import os
import shutil
import statistics
import subprocess
import threading

_FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
           "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
           "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
_REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")


def job_gpu_ids(local_world: int) -> list[str]:
    """``nvidia-smi -i`` ids of this node's GPUs 0..local_world-1 of the job
    (through ``CUDA_VISIBLE_DEVICES`` when it is set)."""
    cvd = os.environ.get("CUDA_VISIBLE_DEVICES", "").strip()
    if cvd:
        ids = [x.strip() for x in cvd.split(",") if x.strip()]
        return ids[:local_world]
    return [str(i) for i in range(local_world)]


class ClockSampler:
    """``gpu_index``: one id or a list of ids (one sampler per node covers every
    GPU of the job, so N ranks do not each start an ``nvidia-smi``)."""

    def __init__(self, gpu_index=0, period_ms: int = 100):
        self.idx = ",".join(str(i) for i in gpu_index) if isinstance(gpu_index, (list, tuple)) else str(gpu_index)
        self.period = period_ms
        self.proc = None
        self.lines: list[str] = []
        self._t = None

    def __enter__(self):
        if shutil.which("nvidia-smi") is None:
            return self
        self.proc = subprocess.Popen(
            ["nvidia-smi", f"--query-gpu={_FIELDS}", "--format=csv,noheader,nounits", f"-lms={self.period}",
             f"-i={self.idx}"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        self._t = threading.Thread(target=self._read, daemon=True)
        self._t.start()
        # nvidia-smi takes a while to start: return once sampling is live, so a
        # short timed region is still covered
        import time
        t0 = time.monotonic()
        while not self.lines and time.monotonic() - t0 < 10 and self.proc.poll() is None:
            time.sleep(0.01)
        self.lines.clear()
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            if self._t is not None:
                self._t.join(timeout=2)
        return False

    def summary(self) -> dict:
        sm, mx, reasons = [], None, set()
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for name, val in zip(_REASONS, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        med = statistics.median(sm)
        out = {"sm_mhz": med, "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}
        # the run is not trustworthy under thermal / hardware slowdown, or with the
        # clock held well below its maximum for no listed reason (a leftover lock)
        bad = sorted(reasons & {"hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown"})
        if bad:
            out["suspect"] = "throttled: " + ",".join(bad)
        elif mx and med < 0.8 * mx and not reasons:
            out["suspect"] = "SM clock held below max with no throttle reason"
        return out
