"""GPU clock / throttle sampling during a timed region (read-only NVML queries).

Nothing here changes a GPU setting; it only reads SM clocks, power and the active
clock-event (throttle) reasons every ``period_s`` on a background thread.
"""
from __future__ import annotations

import os
import statistics
import threading
import time
from typing import List, Optional

_REASONS = {
    0x1: "gpu_idle",
    0x2: "applications_clocks_setting",
    0x4: "sw_power_cap",
    0x8: "hw_slowdown",
    0x20: "sync_boost",
    0x40: "sw_thermal_slowdown",
    0x80: "hw_thermal_slowdown",
    0x100: "hw_power_brake_slowdown",
    0x200: "display_clock_setting",
}


def decode_reasons(mask: int) -> List[str]:
    return [name for bit, name in _REASONS.items() if mask & bit]


def _nvml_handle(pynvml, device_index: int):
    """NVML handle of CUDA device `device_index` of this process.  NVML numbers the GPUs of
    the machine and ignores CUDA_VISIBLE_DEVICES, so the CUDA index is mapped through the
    device's PCI bus id (or, failing that, through CUDA_VISIBLE_DEVICES)."""
    try:
        import torch

        pr = torch.cuda.get_device_properties(device_index)
        bus = "%08x:%02x:%02x.0" % (pr.pci_domain_id, pr.pci_bus_id, pr.pci_device_id)
        return pynvml.nvmlDeviceGetHandleByPciBusId(bus)
    except Exception:  # noqa: BLE001
        pass
    vis = os.environ.get("CUDA_VISIBLE_DEVICES", "").strip()
    if vis:
        ent = [e.strip() for e in vis.split(",") if e.strip()]
        if device_index < len(ent):
            e = ent[device_index]
            if e.isdigit():
                return pynvml.nvmlDeviceGetHandleByIndex(int(e))
            return pynvml.nvmlDeviceGetHandleByUUID(e)
    return pynvml.nvmlDeviceGetHandleByIndex(device_index)


class ClockSampler:
    def __init__(self, device_index: int = 0, period_s: float = 0.2):
        self.index = device_index
        self.period = period_s
        self.samples: List[dict] = []
        self._stop = threading.Event()
        self._thread: Optional[threading.Thread] = None
        self.ok = False
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nvml = pynvml
            self._h = _nvml_handle(pynvml, device_index)
            self.max_sm = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:  # noqa: BLE001
            self.max_sm = None

    def _sample(self) -> None:
        n = self._nvml
        try:
            sm = n.nvmlDeviceGetClockInfo(self._h, n.NVML_CLOCK_SM)
            pw = n.nvmlDeviceGetPowerUsage(self._h) / 1000.0
            try:
                mask = n.nvmlDeviceGetCurrentClocksEventReasons(self._h)
            except Exception:  # noqa: BLE001
                mask = n.nvmlDeviceGetCurrentClocksThrottleReasons(self._h)
            util = n.nvmlDeviceGetUtilizationRates(self._h).gpu
            self.samples.append(dict(t=time.time(), sm=sm, power=pw, mask=int(mask), util=util))
        except Exception:  # noqa: BLE001
            pass

    def _loop(self) -> None:
        while not self._stop.is_set():
            self._sample()
            self._stop.wait(self.period)

    def start(self) -> None:
        if not self.ok:
            return
        self._stop.clear()
        self._thread = threading.Thread(target=self._loop, daemon=True)
        self._thread.start()

    def stop(self) -> dict:
        if not self.ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvml unavailable"]}
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=2)
        self._sample()
        busy = [s for s in self.samples if s["util"] > 50] or self.samples
        reasons = set()
        for s in busy:
            reasons.update(decode_reasons(s["mask"]))
        reasons.discard("gpu_idle")
        return {
            "sm_mhz": statistics.median(s["sm"] for s in busy) if busy else None,
            "sm_max_mhz": self.max_sm,
            "reasons": sorted(reasons),
            "power_w_max": max((s["power"] for s in busy), default=None),
            "samples": len(self.samples),
        }
