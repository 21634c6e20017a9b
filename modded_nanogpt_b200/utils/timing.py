"""Device timing helpers: CUDA events on the launching stream, max over ranks, plus a sampler
of SM clocks and throttle reasons while a region runs."""
from __future__ import annotations

import statistics
import subprocess
import threading
import time

import torch
import torch.distributed as dist


class DeviceTimer:
    """`with timer.region("name"):` accumulates device milliseconds per name (host clock on CPU)."""

    def __init__(self, enabled: bool = True):
        self.enabled = enabled
        self.records: dict[str, list] = {}
        self._pending = []

    class _Region:
        def __init__(self, t, name):
            self.t, self.name = t, name

        def __enter__(self):
            if self.t.enabled and torch.cuda.is_available():
                self.a = torch.cuda.Event(enable_timing=True)
                self.b = torch.cuda.Event(enable_timing=True)
                self.a.record()
            else:
                self.t0 = time.perf_counter()
            return self

        def __exit__(self, *exc):
            if self.t.enabled and torch.cuda.is_available():
                self.b.record()
                self.t._pending.append((self.name, self.a, self.b))
            else:
                self.t.records.setdefault(self.name, []).append(1000 * (time.perf_counter() - self.t0))

    def region(self, name: str):
        return DeviceTimer._Region(self, name)

    def flush(self):
        if self._pending:
            torch.cuda.synchronize()
            for name, a, b in self._pending:
                self.records.setdefault(name, []).append(a.elapsed_time(b))
            self._pending.clear()
        return self.records

    def summary(self):
        self.flush()
        return {k: (sum(v) / len(v), len(v)) for k, v in self.records.items()}


def max_over_ranks(value: float, device=None) -> float:
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return value
    t = torch.tensor([value], dtype=torch.float64, device=device or ("cuda" if torch.cuda.is_available() else "cpu"))
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


_SMI_FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
               "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
               "clocks_event_reasons.sw_power_cap")


class ClockSampler:
    """Polls `nvidia-smi` for one GPU in a background thread (read-only queries)."""

    def __init__(self, gpu_index: int = 0, period_s: float = 0.2):
        self.gpu, self.period = gpu_index, period_s
        self.samples = []
        self._stop = threading.Event()
        self._thread = None

    def _poll(self):
        cmd = ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={_SMI_FIELDS}", "--format=csv,noheader,nounits"]
        while not self._stop.is_set():
            try:
                out = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True, timeout=5).stdout
                parts = [p.strip() for p in out.strip().split(",")]
                if len(parts) >= 7:
                    self.samples.append(parts)
            except Exception:
                pass
            self._stop.wait(self.period)

    def start(self):
        self._thread = threading.Thread(target=self._poll, daemon=True)
        self._thread.start()
        return self

    def stop(self) -> dict:
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=10)
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for s in self.samples:
            try:
                sm.append(float(s[0]))
                mx.append(float(s[1]))
            except ValueError:
                continue
            for n, v in zip(names, s[3:7]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}
