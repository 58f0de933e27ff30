"""ResilientCommManager: generation-scoped communicators that are rebuilt without hanging.

Each way a rebuild could hang is designed out:

* **Dead ranks in group creation** -- only survivors create: NCCL ``shrink_group`` (aborting
  what the dead ranks left in flight) when the new world keeps the old ranks' order and NCCL is
  >= 2.27.3; otherwise a fresh world on the generation's ``PrefixStore`` of the coordinator's
  ``TCPStore``.
* **Creation order depending on local state** -- a plan-derived canonical order: one
  ``split_group`` per layer of disjoint groups on NCCL, ``new_group`` for every group on every
  rank (in the same order) on gloo.
* **A rendezvous store on a training rank** -- the store lives on the coordinator.
* **Blocking forever in a collective** -- ``guarded_wait`` (abortable, with a deadline), and a
  validation all-reduce of ones on every group, under a deadline, before the generation may
  report READY; a failure raises ``GenerationBuildError`` naming the suspect ranks.

``abort()`` (called from the control-client thread) raises the abort flag, runs the abort hooks
(the device abort word that this package's peer-memory kernels poll, so survivors leave fused
kernels in flight at once) and aborts every live NCCL group.  Gloo groups are aborted when their
generation is torn down: a gloo op that lost its peer stays in flight until its timeout, and
destroying its group would wait for it while the next generation's rendezvous runs out of time.
Parity: ``resihp/comm/comm_manager.py:31-329`` (same build paths, validation and abort semantics).
"""

from __future__ import annotations

import contextlib
import datetime
import threading
import time
from dataclasses import dataclass, field
from typing import Any, Callable

import torch
import torch.distributed as dist
import torch.distributed.distributed_c10d as c10d

from .group_spec import GroupSpec, canonical_order, split_layers
from ..utils.log import get_logger

log = get_logger(__name__)


class CommAborted(RuntimeError):
    """The control plane aborted this generation's communicators."""


class CommTimeout(RuntimeError):
    """A guarded wait ran past its deadline."""


class GenerationBuildError(RuntimeError):
    def __init__(self, msg: str, suspects: tuple[int, ...] = ()):
        super().__init__(msg)
        self.suspects = suspects


@dataclass
class GenerationComms:
    generation: int
    rank: int
    world: tuple[str, ...]
    specs: dict[str, GroupSpec]
    groups: dict[str, Any]
    path: str
    build_seconds: float = 0.0
    stats: dict = field(default_factory=dict)

    @property
    def world_size(self) -> int:
        return len(self.world)

    def group(self, name: str):
        """The process group of ``name``; None when this rank is not a member or it has one rank."""
        if name not in self.specs:
            raise KeyError(f"unknown group {name}")
        return self.groups.get(name)

    def ranks(self, name: str) -> tuple[int, ...]:
        return self.specs[name].ranks

    def is_member(self, name: str) -> bool:
        return self.rank in self.specs[name].ranks

    def rank_of(self, worker_id: str) -> int:
        return self.world.index(worker_id)


def is_order_preserving_subset(new: list[str], old: tuple[str, ...]) -> bool:
    """Every member of ``new`` was in ``old``, in the same relative order."""
    where = {w: i for i, w in enumerate(old)}
    positions = [where.get(w) for w in new]
    return None not in positions and positions == sorted(positions)


def _nccl_at_least(version, wanted: tuple[int, ...]) -> bool:
    return version is not None and tuple(version) >= wanted


def _abort_quietly(pg) -> None:
    with contextlib.suppress(Exception):  # the NCCL watchdog is the backstop
        pg.abort()


class ResilientCommManager:
    def __init__(self, backend: str = "gloo", *, device: str | None = None, timeout_s: float = 60.0,
                 validate_timeout_s: float = 30.0, validate: bool = True, shrink: str = "auto",
                 subgroup_mode: str = "split", nccl_nonblocking: bool = True, poll_interval_s: float = 0.0005):
        if shrink not in ("auto", "never", "always"):
            raise ValueError(shrink)
        if subgroup_mode not in ("split", "local"):
            raise ValueError(subgroup_mode)
        self.backend, self.device = backend, device
        self.timeout = datetime.timedelta(seconds=timeout_s)
        self.validate_timeout_s, self.validate = validate_timeout_s, validate
        self.shrink, self.subgroup_mode, self.nccl_nonblocking = shrink, subgroup_mode, nccl_nonblocking
        self.poll_interval_s = poll_interval_s or 0.0005
        self.current: GenerationComms | None = None
        self._aborted = threading.Event()
        self._mu = threading.Lock()
        self._groups_alive: list[Any] = []
        self._store: tuple[tuple[str, int], Any] | None = None
        self._abort_hooks: list[Callable[[], None]] = []
        self._comms_aborted = False  # this generation's NCCL communicators were aborted

    # ------------------------------------------------------------------ capabilities
    @staticmethod
    def capabilities() -> dict:
        caps = dict(shrink_group=hasattr(dist, "shrink_group"), split_group=hasattr(dist, "split_group"),
                    nccl=dist.is_nccl_available(), gloo=dist.is_gloo_available(), nccl_version=None)
        if dist.is_nccl_available() and torch.cuda.is_available():
            with contextlib.suppress(Exception):
                caps["nccl_version"] = torch.cuda.nccl.version()
        return caps

    def can_shrink(self, new_world: list[str]) -> bool:
        """Whether the transition to ``new_world`` can use NCCL's in-place shrink."""
        if self.shrink == "never" or self.backend != "nccl" or self.current is None:
            return False
        if self._comms_aborted:  # aborted communicators cannot be shrunk: the next world starts fresh
            return False
        caps = self.capabilities()
        supported = caps["shrink_group"] and hasattr(c10d, "SHRINK_ABORT") and _nccl_at_least(caps["nccl_version"],
                                                                                              (2, 27, 3))
        smaller = len(new_world) < self.current.world_size
        return bool(supported and smaller and is_order_preserving_subset(new_world, self.current.world))

    def add_abort_hook(self, fn: Callable[[], None]) -> None:
        """An extra action on abort (e.g. raising the symmetric heap's device abort word)."""
        self._abort_hooks.append(fn)

    # ------------------------------------------------------------------ building
    def store_for(self, store_addr: tuple[str, int], prefix: str):
        """The generation's view (``prefix``) of the coordinator's store; one client per address."""
        addr = (store_addr[0], int(store_addr[1]))
        if self._store is None or self._store[0] != addr:
            client = dist.TCPStore(addr[0], addr[1], is_master=False, timeout=self.timeout, wait_for_workers=False)
            self._store = (addr, client)
        return dist.PrefixStore(prefix, self._store[1])

    def _finish(self, generation: int, world: list[str], rank: int, specs: list[GroupSpec], path: str,
                started: float) -> GenerationComms:
        with self._mu:
            self._groups_alive = [c10d._get_default_group()]
        t_world = time.monotonic()
        groups = self._subgroups(rank, specs)
        t_groups = time.monotonic()
        if self.validate:
            self._validate(len(world), groups, specs)
            self._check_epoch(generation, world)
        t_end = time.monotonic()
        comms = GenerationComms(generation, rank, tuple(world), {s.name: s for s in specs}, groups, path,
                                t_end - started)
        # where a generation build spends its time: the world (init / shrink / adopt), the plan's
        # groups, their validation collectives
        comms.stats["phases_s"] = {"world": round(t_world - started, 4), "groups": round(t_groups - t_world, 4),
                                   "validate": round(t_end - t_groups, 4),
                                   "groups_created": len({id(g) for g in groups.values() if g is not None})}
        self.current = comms
        log.info("generation %d built (%s) in %.3fs with %d groups", generation, path, comms.build_seconds,
                 len(groups))
        return comms

    def build(self, generation: int, world: list[str], my_id: str, specs: list[GroupSpec], *, store=None,
              store_addr: tuple[str, int] | None = None, store_prefix: str | None = None) -> GenerationComms:
        started = time.monotonic()
        self._aborted.clear()
        rank = world.index(my_id)
        outside = [s.name for s in specs if s.ranks and max(s.ranks) >= len(world)]
        if outside:
            raise ValueError(f"group {outside[0]} names a rank outside a world of {len(world)}")
        if self.can_shrink(world):
            dropped = [i for i, w in enumerate(self.current.world) if w not in set(world)]
            dist.shrink_group(dropped, group=None, shrink_flags=c10d.SHRINK_ABORT)
            return self._finish(generation, world, rank, specs, "shrink", started)
        if self.shrink == "always":
            raise RuntimeError("shrink requested but this transition cannot shrink")
        if store is None:
            if store_addr is None or store_prefix is None:
                raise ValueError("a fresh world needs a store (or store_addr + store_prefix)")
            store = self.store_for(store_addr, store_prefix)
        self._teardown()
        self._init_world(rank, len(world), store)
        return self._finish(generation, world, rank, specs, "fresh", started)

    def adopt(self, generation: int, world: list[str], my_id: str, specs: list[GroupSpec]) -> GenerationComms:
        """Take the already initialised default process group (a launcher's, e.g. ``torchrun``) as
        this generation's world and create the plan's subgroups on it."""
        started = time.monotonic()
        self._aborted.clear()
        rank = world.index(my_id)
        matches = dist.is_initialized() and dist.get_world_size() == len(world) and dist.get_rank() == rank
        if not matches:
            raise RuntimeError("adopt() needs an initialised default group matching the world")
        return self._finish(generation, world, rank, specs, "adopted", started)

    def _nccl_options(self):
        """Options of every NCCL communicator this manager creates: non-blocking, so that
        ``abort()`` from the control thread returns promptly even while a collective that lost
        its peer is in flight (a blocking communicator's abort waited for the watchdog)."""
        if self.backend != "nccl" or not self.nccl_nonblocking:
            return None
        opts = dist.ProcessGroupNCCL.Options()
        opts.config.blocking = 0
        return opts

    def _init_world(self, rank: int, world_size: int, store) -> None:
        options: dict = dict(backend=self.backend, store=store, rank=rank, world_size=world_size, timeout=self.timeout)
        if self.backend == "nccl":
            if self.device is not None:
                options["device_id"] = torch.device(self.device)
            if self.nccl_nonblocking:
                nccl_opts = dist.ProcessGroupNCCL.Options()
                nccl_opts.config.blocking = 0
                options["pg_options"] = nccl_opts
        dist.init_process_group(**options)

    def _subgroups(self, rank: int, specs: list[GroupSpec]) -> dict[str, Any]:
        """Create the plan's groups in canonical order; name -> group for the groups this rank is in."""
        mine: dict[tuple[int, ...], Any] = {}
        # split_group needs a device bound to the default group (NCCL with device_id); gloo uses new_group
        if self.subgroup_mode == "split" and self.backend == "nccl" and self.device is not None:
            for layer in split_layers(specs):
                self._raise_if_aborted()
                pg = dist.split_group(split_ranks=[list(s.ranks) for s in layer], timeout=self.timeout,
                                      pg_options=self._nccl_options(),
                                      group_desc=f"resihp:{layer[0].kind}:{len(layer)}")
                mine.update((s.ranks, pg) for s in layer if rank in s.ranks)
        else:
            # every rank (member or not) creates every group in the same order, so c10d derives the
            # same group names everywhere and creation cannot deadlock
            for ranks in dict.fromkeys(s.ranks for s in canonical_order(specs) if s.materialized):
                self._raise_if_aborted()
                pg = dist.new_group(list(ranks), timeout=self.timeout, group_desc=f"resihp:{ranks}",
                                    pg_options=self._nccl_options())
                if rank in ranks:
                    mine[ranks] = pg
        with self._mu:
            self._groups_alive += [pg for pg in mine.values() if pg not in self._groups_alive]
        return {s.name: mine.get(s.ranks) if (s.materialized and rank in s.ranks) else None for s in specs}

    def _check_epoch(self, generation: int, world: list[str]) -> None:
        """Generation handshake: every rank of the new world must be building the same
        generation (a straggler still in an older transaction would otherwise join collectives
        meant for another plan).  One MAX all-reduce of (generation, -generation)."""
        on_gpu = self.backend == "nccl" and self.device
        device = torch.device(self.device) if on_gpu else torch.device("cpu")
        epoch = torch.tensor([generation, -generation], dtype=torch.int64, device=device)
        self.guarded_wait(dist.all_reduce(epoch, op=dist.ReduceOp.MAX, async_op=True),
                          timeout=self.validate_timeout_s, what="generation handshake")
        highest, lowest = int(epoch[0].item()), -int(epoch[1].item())
        if highest != generation or lowest != generation:
            raise GenerationBuildError(f"ranks of the new world build generations {lowest}..{highest}, "
                                       f"this rank {generation}", suspects=tuple(range(len(world))))

    def _validate(self, world_size: int, groups: dict[str, Any], specs: list[GroupSpec]) -> None:
        """An all-reduce of ones under a deadline on the world and on every group of this rank."""
        on_gpu = self.backend == "nccl" and self.device
        device = torch.device(self.device) if on_gpu else torch.device("cpu")
        checks = [("world", c10d._get_default_group(), tuple(range(world_size)))]
        checks += [(s.name, groups[s.name], s.ranks) for s in canonical_order(specs) if groups.get(s.name) is not None]
        done: set[int] = set()
        for name, pg, ranks in checks:
            if id(pg) in done:
                continue
            done.add(id(pg))
            ones = torch.ones(1, device=device)
            try:
                self.guarded_wait(dist.all_reduce(ones, group=pg, async_op=True), timeout=self.validate_timeout_s,
                                  what=f"validate {name}")
            except CommAborted:
                raise
            except (CommTimeout, RuntimeError) as err:
                raise GenerationBuildError(f"group {name} failed validation: {err}", suspects=tuple(ranks)) from err
            if int(ones.item()) != pg.size():
                raise GenerationBuildError(f"group {name}: validation sum {ones.item()} != {pg.size()}", tuple(ranks))

    # ------------------------------------------------------------------ waiting / aborting
    def _raise_if_aborted(self) -> None:
        if self._aborted.is_set():
            raise CommAborted("communicators aborted by the control plane")

    def guarded_wait(self, work, timeout: float | None = None, what: str = "collective") -> None:
        """Wait for ``work`` honouring aborts and a deadline.  On NCCL ``wait()`` only orders
        streams and a hang is broken by ``abort()``; gloo cannot interrupt an op in flight, so its
        blocking wait runs on a helper thread while this thread polls."""
        if self.backend == "nccl":
            self._raise_if_aborted()
            work.wait()
            return
        if work.is_completed():
            work.wait()
            return
        finished = threading.Event()
        errors: list[BaseException] = []

        def block() -> None:
            try:
                work.wait()
            except BaseException as err:  # noqa: BLE001 -- handed to the caller's thread
                errors.append(err)
            finally:
                finished.set()

        threading.Thread(target=block, name="guarded-wait", daemon=True).start()
        give_up = None if timeout is None else time.monotonic() + timeout
        while not finished.wait(self.poll_interval_s):
            if self._aborted.is_set():
                raise CommAborted(f"{what} aborted by the control plane")
            if give_up is not None and time.monotonic() > give_up:
                raise CommTimeout(f"{what} timed out after {timeout}s")
        if errors:
            raise errors[0]

    def abort(self) -> None:
        """Thread safe; the control client calls it on RECONFIG_NOTICE."""
        self._aborted.set()
        for hook in self._abort_hooks:
            try:
                hook()
            except Exception:  # noqa: BLE001 -- best effort
                log.exception("abort hook raised")
        if self.backend == "nccl":
            with self._mu:
                groups = list(self._groups_alive)
                self._comms_aborted = bool(groups)
            # Every communicator is aborted on its own thread, subgroups first: a subgroup split
            # from the world communicator shares its proxy, and on B200 the world's abort waited
            # (until the watchdog timeout) while a subgroup's collective was stuck on a dead peer,
            # so aborting them one after another in creation order never reached the stuck one.
            threads = [threading.Thread(target=_abort_quietly, args=(pg,), name="nccl-abort", daemon=True)
                       for pg in reversed(groups)]
            for t in threads:
                t.start()
            deadline = time.monotonic() + 2.0  # the control thread must not stall on a slow abort
            for t in threads:
                t.join(max(0.0, deadline - time.monotonic()))

    @property
    def aborted(self) -> bool:
        return self._aborted.is_set()

    def _teardown(self) -> None:
        if dist.is_initialized():
            try:
                if self.backend == "nccl":
                    c10d._abort_process_group(None)
                else:
                    # abort first: a gloo op that lost its peer would make the destroy wait
                    with self._mu:
                        groups = list(self._groups_alive)
                    for pg in groups:
                        with contextlib.suppress(Exception):  # older gloo builds: fall back to the wait
                            pg.abort()
                    dist.destroy_process_group()
            except Exception:  # noqa: BLE001
                log.exception("teardown of the previous generation failed; continuing")
        with self._mu:
            self._groups_alive = []
            self._comms_aborted = False
        self.current = None

    def destroy(self) -> None:
        self._teardown()
