# SPDX-License-Identifier: Apache-2.0
"""Device timing, L2 flushing and clock sampling for benchmarks.

The reference's bench times rank 0's host wall clock (reference:
bench/vccl_bench.cc:211-221); here every number is device time, the
maximum over ranks.

* Times are CUDA-event durations on the launching stream, taken after
  warm-up with a synchronize on both sides; multi-GPU numbers are the
  maximum over ranks.
* ``L2Flusher`` writes a buffer larger than the 126 MB L2 between timed
  iterations so every iteration starts cold.
* ``ClockSampler`` runs nvidia-smi in the background during the timed
  region and summarises SM clocks and throttle reasons (read-only; no GPU
  setting is ever changed).
"""

from __future__ import annotations

import csv
import io
import statistics
import subprocess
from typing import Callable, Optional

import torch


class L2Flusher:
    def __init__(self, nbytes: int = 256 << 20, device: str = "cuda"):
        self.buf = torch.empty(nbytes // 4, dtype=torch.int32, device=device)

    def __call__(self) -> None:
        self.buf.fill_(0)


def gpu_lead(ms: float = 5.0) -> None:
    """Keep the stream busy for about `ms` so the host can enqueue the timed
    steps before the GPU reaches them: a host pause (Python GC, page faults)
    between an event record and the next launch then cannot land inside a
    timed interval."""
    sleep = getattr(torch.cuda, "_sleep", None)
    if sleep is not None:
        sleep(int(ms * 2.0e6))  # cycles at ~2 GHz


def time_steps(step: Callable[[], None], steps: int, flush: Optional[L2Flusher] = None,
               align_ranks: bool = False) -> list:
    """Per-step device times in microseconds (events around each step).

    The steps are enqueued behind a short GPU sleep (gpu_lead) so host
    latency stays out of the timed intervals.  align_ranks: synchronize the
    device and barrier all ranks before every step (outside the timed
    events), so each step starts with the ranks aligned, as it would after a
    preceding collective.
    """
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    torch.cuda.synchronize()
    if not align_ranks:
        # Enough lead for the host to enqueue every step (two fused calls and a
        # flush each, ~0.1-0.3 ms of host work) with room for host pauses and
        # for a host slowed several-fold by other processes on its cores.
        gpu_lead(10.0 + 1.5 * steps)
    for i in range(steps):
        if align_ranks:
            import torch.distributed as dist

            torch.cuda.synchronize()
            if dist.is_initialized() and dist.get_world_size() > 1:
                dist.barrier()
            gpu_lead(0.5)
        if flush is not None:
            flush()
        starts[i].record()
        step()
        ends[i].record()
    torch.cuda.synchronize()
    return [s.elapsed_time(e) * 1000.0 for s, e in zip(starts, ends)]


def max_over_ranks(value: float) -> float:
    import torch.distributed as dist

    if not dist.is_available() or not dist.is_initialized() or dist.get_world_size() == 1:
        return value
    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")


class ClockSampler:
    """nvidia-smi --query-gpu ... -lms <period> in the background."""

    def __init__(self, period_ms: int = 50):
        self.period_ms = period_ms
        self.proc: Optional[subprocess.Popen] = None
        self.out = ""

    def start(self) -> None:
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={QUERY}", "--format=csv,noheader,nounits", f"-lms={self.period_ms}"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        self.proc.terminate()
        try:
            self.out, _ = self.proc.communicate(timeout=10)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            self.out, _ = self.proc.communicate()
        return summarize(self.out)


def _nvml_handle(device_index: int):
    """NVML handle of a CUDA device (matched by PCI bus id, so it honours
    CUDA_VISIBLE_DEVICES), or None."""
    try:
        import pynvml

        pynvml.nvmlInit()
        props = torch.cuda.get_device_properties(device_index)
        bus = f"{getattr(props, 'pci_domain_id', 0):08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
        return pynvml, pynvml.nvmlDeviceGetHandleByPciBusId(bus)
    except Exception:  # noqa: BLE001 - no NVML
        return None


def bind_to_gpu_cpus(device_index: int) -> bool:
    """Restrict this process to the CPU cores NVML reports as closest to the
    GPU, so pinned host buffers (allocated on first touch) sit on the GPU's
    NUMA node and host-device copies do not cross sockets.  Read-only NVML
    query; returns False (and changes nothing) when it is unavailable."""
    import os

    got = _nvml_handle(device_index)
    if got is None:
        return False
    nv, h = got
    try:
        words = nv.nvmlDeviceGetCpuAffinity(h, 16)
        cpus = {64 * w + b for w, mask in enumerate(words) for b in range(64) if (int(mask) >> b) & 1}
        cpus &= set(os.sched_getaffinity(0))  # stay inside the cores this process may use
        if not cpus:
            return False
        os.sched_setaffinity(0, cpus)
        return True
    except Exception:  # noqa: BLE001
        return False


class NvmlClockSampler:
    """Samples this process's GPU through NVML every `period_s` on a thread.

    Timed regions here are tens of milliseconds, shorter than nvidia-smi's
    start-up; NVML queries are read-only (clock and clocks-event-reason
    readings), nothing about the GPU is changed.
    """

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown"}

    def __init__(self, device_index: int, period_s: float = 0.005):
        import threading

        self.period_s = period_s
        self.samples = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        self.ok = False
        got = _nvml_handle(device_index)
        if got is not None:
            try:
                self.nvml, self.handle = got
                self.max_mhz = self.nvml.nvmlDeviceGetMaxClockInfo(self.handle, self.nvml.NVML_CLOCK_SM)
                self.ok = True
            except Exception:  # noqa: BLE001 - no NVML: report unavailable
                self.ok = False

    def _run(self):
        nv = self.nvml
        while not self._stop.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(self.handle, nv.NVML_CLOCK_SM)
                reasons = nv.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
                self.samples.append((mhz, reasons))
            except Exception:  # noqa: BLE001
                pass
            self._stop.wait(self.period_s)

    def start(self) -> None:
        import threading

        if self.ok:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()

    def stop(self) -> dict:
        if not self.ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvml unavailable"], "samples": 0}
        self._stop.set()
        if self._thread:
            self._thread.join(timeout=5)
        mhz = [m for m, _ in self.samples]
        reasons = set()
        for _, bits in self.samples:
            for bit, name in self.REASONS.items():
                if bits & bit:
                    reasons.add(name)
        return {"sm_mhz": statistics.median(mhz) if mhz else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(reasons), "samples": len(mhz), "source": "nvml"}


def summarize(text: str) -> dict:
    sm, smax, reasons = [], [], set()
    names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
    for row in csv.reader(io.StringIO(text)):
        if len(row) < 9:
            continue
        try:
            sm.append(float(row[1]))
            smax.append(float(row[2]))
        except ValueError:
            continue
        for name, val in zip(names, row[5:9]):
            if val.strip().lower() == "active":
                reasons.add(name)
    return {
        "sm_mhz": statistics.median(sm) if sm else None,
        "sm_max_mhz": max(smax) if smax else None,
        "reasons": sorted(reasons),
        "samples": len(sm),
    }
