"""Node health probes: NVML (XID events, uncorrected ECC, clock/throttle side information)
and InfiniBand port state from sysfs.

Every probe degrades to a no-op when its facility is missing, so the same agent runs on a
CPU-only host.  ``NVMLProbe`` takes an injectable ``nvml`` module so tests drive it with a
fake.  The probes only read device state; nothing here changes a GPU setting.
(Reference: ``resihp/control/health.py:13-120``; the fatal XID set is the same.)
"""

from __future__ import annotations

from dataclasses import dataclass
from pathlib import Path

# XIDs after which the GPU is lost for this job.
FATAL_XIDS = frozenset({48, 61, 62, 63, 64, 74, 79, 92, 94, 95, 119, 120, 140})


@dataclass(frozen=True)
class HealthEvent:
    device: str          # "cuda:<i>" or "*" for the whole node
    kind: str            # xid | ecc | ib_port
    fatal: bool
    detail: str = ""

    def matches(self, worker_device: str) -> bool:
        return self.device == "*" or self.device == worker_device

    def describe(self) -> str:
        return f"{self.kind} on {self.device}: {self.detail}"


class NVMLProbe:
    def __init__(self, nvml=None, device_indices: list[int] | None = None):
        self.nvml = nvml
        self._ok = False
        self._handles: dict[int, object] = {}
        self._events = None
        self._last_ecc: dict[int, int] = {}
        try:
            if self.nvml is None:
                import pynvml  # nvidia-ml-py

                self.nvml = pynvml
            self.nvml.nvmlInit()
            count = self.nvml.nvmlDeviceGetCount()
            for i in (device_indices if device_indices is not None else range(count)):
                self._handles[i] = self.nvml.nvmlDeviceGetHandleByIndex(i)
            self._events = self.nvml.nvmlEventSetCreate()
            for h in self._handles.values():
                try:
                    self.nvml.nvmlDeviceRegisterEvents(h, self.nvml.nvmlEventTypeXidCriticalError, self._events)
                except Exception:  # noqa: BLE001 - XID events unsupported on this SKU
                    pass
            self._ok = True
        except Exception:  # noqa: BLE001 - no NVML on this host
            self._ok = False

    @property
    def available(self) -> bool:
        return self._ok

    def _index_of(self, handle) -> int:
        for i, h in self._handles.items():
            if h == handle:
                return i
        return -1

    def poll(self) -> list[HealthEvent]:
        if not self._ok:
            return []
        events: list[HealthEvent] = []
        while True:
            try:
                ev = self.nvml.nvmlEventSetWait(self._events, 0)
            except Exception:  # noqa: BLE001 - timeout: nothing pending
                break
            idx = self._index_of(ev.device)
            xid = int(ev.eventData)
            events.append(HealthEvent(f"cuda:{idx}" if idx >= 0 else "*", "xid", xid in FATAL_XIDS, f"XID {xid}"))
        for i, h in self._handles.items():
            try:
                n = self.nvml.nvmlDeviceGetTotalEccErrors(h, self.nvml.NVML_MEMORY_ERROR_TYPE_UNCORRECTED,
                                                          self.nvml.NVML_VOLATILE_ECC)
            except Exception:  # noqa: BLE001
                continue
            if n > self._last_ecc.get(i, n):
                events.append(HealthEvent(f"cuda:{i}", "ecc", True, f"uncorrected ECC count {n}"))
            self._last_ecc[i] = n
        return events

    def throttle(self, index: int) -> dict:
        """Clock, temperature and throttle-reason readings: side information for the fail-slow
        detector, never a trigger on their own."""
        if not self._ok or index not in self._handles:
            return {}
        h, nv = self._handles[index], self.nvml
        out = {}
        for key, fn in (("sm_clock", lambda: nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)),
                        ("temp", lambda: nv.nvmlDeviceGetTemperature(h, nv.NVML_TEMPERATURE_GPU)),
                        ("throttle", lambda: nv.nvmlDeviceGetCurrentClocksThrottleReasons(h))):
            try:
                out[key] = fn()
            except Exception:  # noqa: BLE001
                pass
        return out


class IBPortProbe:
    """One rail down degrades the node (a fail-slow candidate); every rail down isolates it."""

    def __init__(self, root: str = "/sys/class/infiniband"):
        self.root = Path(root)

    def poll(self) -> list[HealthEvent]:
        if not self.root.exists():
            return []
        states = sorted(self.root.glob("*/ports/*/state"))
        down = []
        for st in states:
            text = st.read_text().strip()
            if "ACTIVE" not in text:
                down.append(f"{st.parts[-4]} port {st.parts[-2]} {text}")
        fatal = bool(down) and len(down) == len(states)
        return [HealthEvent("*", "ib_port", fatal, d) for d in down]


class CompositeProbe:
    def __init__(self, *probes):
        self.probes = probes

    def poll(self) -> list[HealthEvent]:
        out: list[HealthEvent] = []
        for p in self.probes:
            out.extend(p.poll())
        return out
