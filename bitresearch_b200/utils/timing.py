"""Device timing helpers: CUDA-event phase timers, NVTX ranges and a clock sampler.

* ``PhaseTimer`` records CUDA events around named phases (forward, backward, reduce-scatter,
  optimizer, all-gather) on the launching stream and reports milliseconds once synchronised.
* ``nvtx`` is a no-op context manager when CUDA is absent.
* ``ClockSampler`` polls ``nvidia-smi`` in a background process during a timed region and
  summarises the SM clock and the throttle reasons it saw (read-only: it changes no setting).
"""
from __future__ import annotations

import contextlib
import os
import signal
import statistics
import subprocess
import tempfile

import torch


class PhaseTimer:
    def __init__(self, enabled: bool = True):
        self.enabled = enabled and torch.cuda.is_available()
        self.events: list[tuple[str, torch.cuda.Event, torch.cuda.Event]] = []

    @contextlib.contextmanager
    def phase(self, name: str):
        if not self.enabled:
            yield
            return
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        try:
            yield
        finally:
            b.record()
            self.events.append((name, a, b))

    def collect(self) -> dict[str, float]:
        out: dict[str, float] = {}
        for name, a, b in self.events:
            b.synchronize()
            out[name] = out.get(name, 0.0) + a.elapsed_time(b)
        self.events.clear()
        return out


@contextlib.contextmanager
def traced(timer: "PhaseTimer | None", name: str):
    """One phase: an NVTX range (seen by Nsight / torch.profiler) and, with a timer, CUDA events on the
    current stream. A no-op without a timer."""
    if timer is None or not timer.enabled:
        yield
        return
    torch.cuda.nvtx.range_push(name)
    try:
        with timer.phase(name):
            yield
    finally:
        torch.cuda.nvtx.range_pop()


@contextlib.contextmanager
def nvtx(name: str):
    if torch.cuda.is_available():
        torch.cuda.nvtx.range_push(name)
        try:
            yield
        finally:
            torch.cuda.nvtx.range_pop()
    else:
        yield


_QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
          "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
          "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")


class ClockSampler:
    """SM clock and clock-event reasons of one GPU between ``start()`` and ``stop()``.

    Reads NVML (read-only queries) every ``period_ms`` on a thread and always once at ``start()`` and
    once at ``stop()``, so a timed region shorter than the period still has samples; falls back to
    ``nvidia-smi -lms`` when NVML is unavailable."""

    # clock-event reason bits (nvml.h): the ones a benchmark must report
    _REASONS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40}

    def __init__(self, gpu_index: int | None = None, period_ms: int = 50):
        self.gpu_index = gpu_index
        self.period_ms = period_ms
        self.proc = None
        self.path = None
        self._nvml = None
        self._handle = None
        self._samples: list[tuple[float, float, int]] = []
        self._stop = None
        self._thread = None

    def _nvml_handle(self):
        import pynvml
        pynvml.nvmlInit()
        idx = self.gpu_index or 0
        try:  # match the CUDA device to its NVML handle by PCI address (CUDA_VISIBLE_DEVICES may remap)
            import torch
            pr = torch.cuda.get_device_properties(idx)
            bus = f"{pr.pci_domain_id:08x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
            return pynvml, pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:
            return pynvml, pynvml.nvmlDeviceGetHandleByIndex(idx)

    def _sample(self):
        n, h = self._nvml, self._handle
        try:
            sm = n.nvmlDeviceGetClockInfo(h, n.NVML_CLOCK_SM)
            smax = n.nvmlDeviceGetMaxClockInfo(h, n.NVML_CLOCK_SM)
            get = getattr(n, "nvmlDeviceGetCurrentClocksEventReasons", None) or n.nvmlDeviceGetCurrentClocksThrottleReasons
            self._samples.append((float(sm), float(smax), int(get(h))))
        except Exception:
            pass

    def start(self):
        import threading
        try:
            self._nvml, self._handle = self._nvml_handle()
        except Exception:
            self._nvml = None
        if self._nvml is not None:
            self._samples = []
            self._sample()
            self._stop = threading.Event()

            def loop():
                while not self._stop.wait(self.period_ms / 1000.0):
                    self._sample()

            self._thread = threading.Thread(target=loop, daemon=True)
            self._thread.start()
            return self
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        cmd = ["nvidia-smi", f"--query-gpu={_QUERY}", "--format=csv,noheader,nounits", f"-lms={max(self.period_ms, 100)}"]
        if self.gpu_index is not None:
            cmd.insert(1, f"--id={self.gpu_index}")
        try:
            self.proc = subprocess.Popen(cmd, stdout=open(self.path, "w"), stderr=subprocess.DEVNULL,
                                         start_new_session=True)
        except Exception:
            self.proc = None
        return self

    def stop(self) -> dict:
        if self._nvml is not None:
            self._stop.set()
            self._thread.join(timeout=5)
            self._sample()
            if not self._samples:
                return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "samples": 0}
            sm = [x[0] for x in self._samples]
            reasons = sorted({name for _, _, r in self._samples for name, bit in self._REASONS.items() if r & bit})
            loaded = [v for v in sm if v > 0.3 * max(sm)] or sm
            return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": max(x[1] for x in self._samples),
                    "reasons": reasons, "samples": len(sm), "source": "nvml"}
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        try:
            os.killpg(self.proc.pid, signal.SIGTERM)
        except Exception:
            pass
        self.proc.wait(timeout=10)
        return summarise_clock_csv(self.path)


def summarise_clock_csv(path: str) -> dict:
    sm, smax, reasons = [], [], set()
    names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
    with open(path) as f:
        for line in f:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
    if not sm:
        return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "samples": 0}
    # median over samples taken under load (clock above idle)
    loaded = [s for s in sm if s > 0.3 * max(sm)] or sm
    return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": max(smax), "reasons": sorted(reasons),
            "samples": len(sm)}
