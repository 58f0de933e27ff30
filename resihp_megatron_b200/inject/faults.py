"""Fault injection.

* ``FaultInjector`` lives inside a worker and fires at deterministic hook points
  ``(iteration >= iter, phase)`` -- phases ``forward``, ``backward``, ``reduce``, ``step``,
  ``loss``, and ``boundary`` (after an iteration committed, with the GPU synchronised, so a
  killed GPU worker leaves no kernel or collective in flight) -- or after a wall-clock offset: SIGKILL itself, SIGSTOP itself (optionally resumed by
  a SIGCONT timer), pad its compute by busy waiting (fail-slow) or delay a link.  All of it happens
  on the host: a killed or stopped process leaves between kernel launches, never inside a GPU
  operation.
* ``ExternalInjector`` builds (and, when allowed, runs) host commands that emulate hardware
  faults on a cluster: kill / stop, NIC down, bandwidth contention and -- only with
  ``allow_device_settings=True`` -- SM clock locks, power caps and DCGM XID injection.  It is a
  dry run by default; on shared GPUs the device-setting faults stay dry runs.

Spec grammar (``RESIHP_FAULTS`` or ``parse_faults``), kept from the reference
(``resihp/inject/faults.py:35-287``) because users write it::

    kind@key=value:key=value;kind@...     e.g.  kill@iter=5:target=n0g1;slow@iter=10:target=n1g0:factor=2

Reserved keys: target, iter, time, duration, factor, phase; any other key goes to ``params``.
"""

from __future__ import annotations

import os
import shlex
import signal
import subprocess
import time
from dataclasses import dataclass, field
from enum import Enum
from typing import Callable

from ..utils.log import get_logger

log = get_logger(__name__)


class FaultKind(str, Enum):
    KILL = "kill"
    HANG = "hang"
    SLOW_COMPUTE = "slow"
    SLOW_LINK = "slow_link"
    XID = "xid"
    NIC_DOWN = "nic_down"
    POWER_CAP = "power_cap"


DEVICE_SETTING_KINDS = frozenset({FaultKind.XID, FaultKind.POWER_CAP})

# reserved key -> (FaultSpec field, parser); the field order is the order ``to_spec`` writes
_FIELDS = {"target": ("target", str), "iter": ("at_iteration", int), "time": ("at_time", float),
           "duration": ("duration", float), "factor": ("factor", float), "phase": ("phase", str)}


@dataclass(frozen=True)
class FaultSpec:
    kind: FaultKind
    target: str
    at_iteration: int | None = None
    at_time: float | None = None
    duration: float | None = None
    factor: float = 1.0
    phase: str = "forward"
    params: tuple[tuple[str, str], ...] = field(default_factory=tuple)

    def param(self, key: str, default: str | None = None) -> str | None:
        return dict(self.params).get(key, default)

    def to_spec(self) -> str:
        """The grammar form; fields at their defaults are left out."""
        defaults = {"at_iteration": None, "at_time": None, "duration": None, "factor": 1.0, "phase": "forward"}
        pairs = []
        for key, (attr, _) in _FIELDS.items():
            value = getattr(self, attr)
            if attr == "target" or value != defaults[attr]:
                pairs.append(f"{key}={value}")
        pairs += [f"{k}={v}" for k, v in self.params]
        return f"{self.kind.value}@{':'.join(pairs)}"


def _parse_one(item: str) -> FaultSpec:
    kind, at, body = item.partition("@")
    if not at:
        raise ValueError(f"fault {item!r} must look like kind@key=value:...")
    values: dict[str, str] = {}
    for token in filter(None, body.split(":")):
        key, eq, value = token.partition("=")
        if not eq:
            raise ValueError(f"bad token {token!r} in fault {item!r}")
        values[key.strip()] = value.strip()
    if "target" not in values:
        raise ValueError(f"fault {item!r} has no target")
    fields = {attr: cast(values[key]) for key, (attr, cast) in _FIELDS.items() if key in values}
    extra = tuple(sorted((k, v) for k, v in values.items() if k not in _FIELDS))
    return FaultSpec(kind=FaultKind(kind.strip()), params=extra, **fields)


def parse_faults(spec: str | None) -> list[FaultSpec]:
    return [_parse_one(item) for item in (s.strip() for s in (spec or "").split(";")) if item]


class FaultInjector:
    def __init__(self, worker_id: str, faults: list[FaultSpec], *, start_time: float | None = None,
                 kill_fn: Callable[[], None] | None = None):
        self.worker_id = worker_id
        self.faults = [f for f in faults if f.target in ("*", worker_id)]
        self.fired: set[int] = set()
        self.start_time = start_time if start_time is not None else time.monotonic()
        self._kill_fn = kill_fn
        self._slow_factor, self._slow_until = 1.0, None
        self._link_delay: dict[str, float] = {}
        self._actions = {FaultKind.KILL: self._kill, FaultKind.HANG: self._hang,
                         FaultKind.SLOW_COMPUTE: self._slow, FaultKind.SLOW_LINK: self._slow_link}

    def _due(self, f: FaultSpec, iteration: int, phase: str, now: float) -> bool:
        if f.at_iteration is None and f.at_time is None:
            return False
        if f.at_iteration is not None and (iteration < f.at_iteration or phase != f.phase):
            return False
        return f.at_time is None or now - self.start_time >= f.at_time

    def on_hook(self, iteration: int, phase: str) -> None:
        now = time.monotonic()
        for i, f in enumerate(self.faults):
            if i not in self.fired and self._due(f, iteration, phase, now):
                self.fired.add(i)
                log.warning("injecting %s on %s", f.to_spec(), self.worker_id)
                action = self._actions.get(f.kind)
                if action is None:
                    raise ValueError(f"{f.kind.value} cannot be injected in-process; use ExternalInjector")
                action(f, now)

    def _kill(self, f: FaultSpec, now: float) -> None:
        stamp = os.environ.get("RESIHP_FAULT_STAMP")
        if stamp:  # the fault instant on the machine-wide monotonic clock, for recovery timing
            with open(stamp, "a") as fh:
                fh.write(f"{self.worker_id} {time.monotonic():.6f}\n")
        if self._kill_fn is not None:
            self._kill_fn()
        else:
            os.kill(os.getpid(), signal.SIGKILL)

    def _hang(self, f: FaultSpec, now: float) -> None:
        if f.duration is not None:  # a helper wakes this process up again
            subprocess.Popen(["sh", "-c", f"sleep {f.duration}; kill -CONT {os.getpid()}"])
        os.kill(os.getpid(), signal.SIGSTOP)

    def _slow(self, f: FaultSpec, now: float) -> None:
        self._slow_factor = max(1.0, f.factor)
        self._slow_until = now + f.duration if f.duration is not None else None

    def _slow_link(self, f: FaultSpec, now: float) -> None:
        self._link_delay[f.param("peer", "*")] = float(f.param("delay_s", "0.01"))

    def compute_factor(self) -> float:
        if self._slow_until is not None and time.monotonic() > self._slow_until:
            self._slow_factor, self._slow_until = 1.0, None
        return self._slow_factor

    def pad_compute(self, elapsed_s: float) -> float:
        """Busy-wait so that a chunk which took ``elapsed_s`` looks ``factor`` times slower."""
        extra = (self.compute_factor() - 1.0) * max(elapsed_s, 0.0)
        if extra <= 0.0:
            return 0.0
        until = time.perf_counter() + extra
        while time.perf_counter() < until:
            pass
        return extra

    def link_delay(self, peer: str) -> float:
        delay = self._link_delay.get(peer, self._link_delay.get("*", 0.0))
        if delay > 0:
            time.sleep(delay)
        return delay


_INJECTOR: FaultInjector | None = None


def get_injector() -> FaultInjector:
    """The process-wide injector built from ``RESIHP_FAULTS`` and ``RESIHP_WORKER_ID``."""
    global _INJECTOR
    if _INJECTOR is None:
        _INJECTOR = FaultInjector(os.environ.get("RESIHP_WORKER_ID", ""), parse_faults(os.environ.get("RESIHP_FAULTS")))
    return _INJECTOR


def reset_injector(injector: FaultInjector | None = None) -> None:
    global _INJECTOR
    _INJECTOR = injector


@dataclass
class ExternalCommand:
    apply: list[str]
    revert: list[str] | None = None


def _cmd_kill(f):
    return ExternalCommand(["kill", "-9", f.param("pid", "0")])


def _cmd_hang(f):
    pid = f.param("pid", "0")
    return ExternalCommand(["kill", "-STOP", pid], ["kill", "-CONT", pid])


def _cmd_slow(f):
    locked = str(int(float(f.param("base_mhz", "1965")) / max(f.factor, 1.0)))
    gpu = f.param("gpu", "0")
    return ExternalCommand(["nvidia-smi", "-i", gpu, "-lgc", f"{locked},{locked}"], ["nvidia-smi", "-i", gpu, "-rgc"])


def _cmd_power_cap(f):
    gpu = f.param("gpu", "0")
    return ExternalCommand(["nvidia-smi", "-i", gpu, "-pl", f.param("watts", "500")],
                           ["nvidia-smi", "-i", gpu, "-pl", f.param("default_watts", "1000")])


def _cmd_xid(f):
    # DCGM field 230 carries XID errors: this exercises the agents' health-probe path
    return ExternalCommand(["dcgmi", "test", "--inject", "--gpuid", f.param("gpu", "0"), "-f", "230", "-v",
                            f.param("xid", "79")])


def _cmd_nic_down(f):
    iface = f.param("iface", "ib0")
    return ExternalCommand(["ip", "link", "set", "dev", iface, "down"], ["ip", "link", "set", "dev", iface, "up"])


def _cmd_slow_link(f):
    return ExternalCommand(["python", "-m", "resihp_megatron_b200.inject.contention", "--host",
                            f.param("peer", "127.0.0.1"), "--port", f.param("port", "29700"), "--seconds",
                            str(f.duration or 60)])


_COMMANDS = {FaultKind.KILL: _cmd_kill, FaultKind.HANG: _cmd_hang, FaultKind.SLOW_COMPUTE: _cmd_slow,
             FaultKind.POWER_CAP: _cmd_power_cap, FaultKind.XID: _cmd_xid, FaultKind.NIC_DOWN: _cmd_nic_down,
             FaultKind.SLOW_LINK: _cmd_slow_link}


class ExternalInjector:
    """Host-level fault emulation, a dry run unless ``dry_run=False``.  Commands that change a
    GPU's settings (clock lock, power cap, XID injection) also need ``allow_device_settings=True``
    and are refused otherwise."""

    def __init__(self, dry_run: bool = True, runner: Callable[[list[str]], int] | None = None,
                 allow_device_settings: bool = False):
        self.dry_run, self.allow_device_settings = dry_run, allow_device_settings
        self.executed: list[list[str]] = []
        self._runner = runner if runner is not None else subprocess.call

    @staticmethod
    def commands(f: FaultSpec) -> ExternalCommand:
        build = _COMMANDS.get(f.kind)
        if build is None:
            raise ValueError(f"unsupported external fault {f.kind}")
        return build(f)

    @staticmethod
    def changes_device_settings(f: FaultSpec) -> bool:
        return f.kind == FaultKind.SLOW_COMPUTE or f.kind in DEVICE_SETTING_KINDS

    def apply(self, f: FaultSpec) -> ExternalCommand:
        cmd = self.commands(f)
        self._run(cmd.apply, f)
        return cmd

    def revert(self, f: FaultSpec) -> None:
        undo = self.commands(f).revert
        if undo:
            self._run(undo, f)

    def _run(self, argv: list[str], f: FaultSpec) -> None:
        self.executed.append(argv)
        if self.dry_run:
            log.warning("[dry-run] %s", shlex.join(argv))
            return
        if self.changes_device_settings(f) and not self.allow_device_settings:
            raise PermissionError(f"{f.kind.value} changes GPU settings; pass allow_device_settings=True")
        code = self._runner(argv)
        if code != 0:
            raise RuntimeError(f"fault command failed ({code}): {shlex.join(argv)}")


def run_schedule(faults: list[FaultSpec], injector: ExternalInjector, *, clock: Callable[[], float] = time.monotonic,
                 sleep: Callable[[float], None] = time.sleep) -> list[tuple[float, FaultSpec, str]]:
    """Apply the time-triggered faults and their reverts in time order (a revert first when both
    fall on the same instant); returns ``(time, fault, action)`` per event."""
    timeline = []
    for f in filter(lambda f: f.at_time is not None, faults):
        timeline.append((f.at_time, 1, "apply", f))
        if f.duration is not None:
            timeline.append((f.at_time + f.duration, 0, "revert", f))
    timeline.sort(key=lambda e: (e[0], e[1]))
    started = clock()
    done = []
    for at, _, action, f in timeline:
        pause = at - (clock() - started)
        if pause > 0:
            sleep(pause)
        getattr(injector, action)(f)
        done.append((at, f, action))
    return done
