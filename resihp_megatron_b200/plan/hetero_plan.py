"""HeteroParallelPlan: an explicit, generation-scoped layout of hybrid parallelism.

A plan is not a rectangular TP x PP x DP grid.  Each (replica, stage) group lists its own
devices -- TP-major, ``cp`` context-parallel slices of ``tp`` devices -- its half-open layer
range, and ``assignment[stage][mb]`` names the replica that runs micro-batch ``mb`` at that
stage.  The one table expresses plain DP, dropping a replica, a different TP degree per group
and stage-level micro-batch migration.  With interleaving (``vpp > 1``) stages are virtual:
virtual stage ``s`` runs on physical stage ``s % (num_stages // vpp)``, and every chunk of a
physical slot lists the same devices.

Interfaces kept from the reference (``resihp/plan/hetero_plan.py:21-280``) so that plans and
coordinator payloads interoperate: the JSON schema, the validation rules, and the derived
process-group names ``tp/r{r}/s{s}[/c{i}]``, ``cp/r{r}/s{s}/t{j}`` and ``dpshard/s{s}/{ranks}``.
The lookups here are served from indexes built once per plan object.
"""

from __future__ import annotations

import itertools
from dataclasses import dataclass, field, replace

from ..comm.group_spec import GroupSpec
from ..utils.intervals import even_split, locate, refine


@dataclass(frozen=True)
class StageGroup:
    replica: int
    stage: int
    devices: tuple[str, ...]
    layers: tuple[int, int]
    cp: int = 1

    @property
    def tp(self) -> int:
        return len(self.devices) // self.cp

    @property
    def num_layers(self) -> int:
        lo, hi = self.layers
        return hi - lo

    def slice(self, i: int) -> tuple[str, ...]:
        """CP slice ``i``: one TP group's devices."""
        width = self.tp
        return self.devices[width * i:width * (i + 1)]

    def cp_peers(self, j: int) -> tuple[str, ...]:
        """The devices at TP rank ``j`` of every CP slice: one CP group."""
        return tuple(self.devices[j + i * self.tp] for i in range(self.cp))

    def slice_of(self, device: str) -> int:
        return divmod(self.devices.index(device), self.tp)[0]

    def to_json(self) -> dict:
        out = dict(replica=self.replica, stage=self.stage, devices=list(self.devices), layers=list(self.layers))
        if self.cp > 1 or self.cp < 1:
            out["cp"] = self.cp
        return out

    @classmethod
    def from_json(cls, d: dict) -> "StageGroup":
        lo, hi = d["layers"]
        return cls(replica=d["replica"], stage=d["stage"], devices=tuple(d["devices"]), layers=(lo, hi),
                   cp=d.get("cp", 1))


def tp_group_name(replica: int, stage: int, cp_slice: int | None = None) -> str:
    name = f"tp/r{replica}/s{stage}"
    return name if cp_slice is None else name + f"/c{cp_slice}"


def cp_group_name(replica: int, stage: int, tp_rank: int) -> str:
    return f"cp/r{replica}/s{stage}/t{tp_rank}"


def dpshard_group_name(stage: int, ranks: tuple[int, ...]) -> str:
    return f"dpshard/s{stage}/{'-'.join(map(str, ranks))}"


def _scalar_fields():
    return ("generation", "num_layers", "num_stages", "num_replicas", "num_microbatches")


@dataclass(frozen=True)
class HeteroParallelPlan:
    generation: int
    world: tuple[str, ...]
    num_layers: int
    num_stages: int
    num_replicas: int
    stage_groups: tuple[StageGroup, ...]
    num_microbatches: int
    assignment: tuple[tuple[int, ...], ...]
    standby: tuple[str, ...] = ()
    sequence_parallel: bool = False
    meta: dict = field(default_factory=dict, compare=False)
    vpp: int = 1
    _keyed: dict = field(init=False, repr=False, compare=False, hash=False)
    _staged: dict = field(init=False, repr=False, compare=False, hash=False)
    _rank_of: dict = field(init=False, repr=False, compare=False, hash=False)

    def __post_init__(self):
        keyed, staged = {}, {}
        for g in self.stage_groups:
            keyed.setdefault((g.replica, g.stage), g)
            staged.setdefault(g.stage, []).append(g)
        for gs in staged.values():
            gs.sort(key=lambda g: g.replica)
        object.__setattr__(self, "_keyed", keyed)
        object.__setattr__(self, "_staged", staged)
        object.__setattr__(self, "_rank_of", {d: i for i, d in reversed(list(enumerate(self.world)))})

    # ------------------------------------------------------------------ lookups
    def group(self, replica: int, stage: int) -> StageGroup | None:
        return self._keyed.get((replica, stage))

    def groups_at(self, stage: int) -> list[StageGroup]:
        return list(self._staged.get(stage, ()))

    @property
    def num_physical_stages(self) -> int:
        return self.num_stages // self.vpp

    def physical_key(self, replica: int, stage: int) -> tuple[int, int]:
        return replica, stage % self.num_physical_stages

    def chunk_stages(self, replica: int, physical_stage: int) -> list[int]:
        """The virtual stages of ``replica`` that run on ``physical_stage``, in order."""
        virtual = range(physical_stage, self.num_stages, self.num_physical_stages)
        return [s for s in virtual if (replica, s) in self._keyed]

    def groups_of_device(self, device: str) -> list[StageGroup]:
        return sorted(filter(lambda g: device in g.devices, self.stage_groups), key=lambda g: g.stage)

    def group_of_device(self, device: str) -> StageGroup | None:
        return next(iter(self.groups_of_device(device)), None)

    def rank(self, device: str) -> int:
        try:
            return self._rank_of[device]
        except KeyError:
            raise ValueError(f"{device!r} is not in the world") from None

    def ranks(self, g: StageGroup) -> tuple[int, ...]:
        return tuple(map(self.rank, g.devices))

    def slice_ranks(self, g: StageGroup, i: int) -> tuple[int, ...]:
        return tuple(map(self.rank, g.slice(i)))

    def tp_name(self, g: StageGroup, device: str) -> str:
        return tp_group_name(g.replica, g.stage, g.slice_of(device) if g.cp > 1 else None)

    def executor(self, stage: int, mb: int) -> int:
        return self.assignment[stage][mb]

    def layer_partition(self) -> list[tuple[int, int]]:
        return [self._staged[s][0].layers for s in range(self.num_stages)]

    def microbatches_of(self, replica: int, stage: int) -> list[int]:
        return [m for m, r in enumerate(self.assignment[stage]) if r == replica]

    def physical(self) -> "HeteroParallelPlan":
        """The planning view of an interleaved plan: one stage per physical slot, carrying the
        total layer count of its chunks (nominal contiguous ranges) and chunk 0's executors."""
        if self.vpp == 1:
            return self
        P = self.num_physical_stages
        sizes = [sum(self.groups_at(s)[0].num_layers for s in range(p, self.num_stages, P)) for p in range(P)]
        edges = list(itertools.accumulate(sizes, initial=0))
        merged = tuple(replace(g, layers=(edges[g.stage], edges[g.stage + 1]))
                       for g in self.stage_groups if g.stage < P)
        return replace(self, num_stages=P, stage_groups=merged, assignment=self.assignment[:P], vpp=1)

    # ------------------------------------------------------------------ validation
    def _check_groups(self):
        world = set(self.world)
        owner: dict[str, tuple[int, int]] = {}
        slot_devices: dict[tuple[int, int], tuple[str, ...]] = {}
        uniform_cp = {g.cp for g in self.stage_groups}
        for g in self.stage_groups:
            tag = f"r{g.replica}s{g.stage}"
            slot = self.physical_key(g.replica, g.stage)
            if not g.devices:
                yield f"empty group {tag}"
                continue
            if slot_devices.setdefault(slot, g.devices) != g.devices:
                yield f"chunks of physical slot {slot} must use identical devices"
            if len(set(g.devices)) < len(g.devices):
                yield f"group {tag} lists a device twice"
            if g.cp < 1 or len(g.devices) % g.cp:
                yield f"group {tag}: {len(g.devices)} devices do not split into cp={g.cp}"
            if len(uniform_cp) > 1:
                yield "context parallelism must be uniform across groups"
            for d in g.devices:
                if d not in world:
                    yield f"device {d} not in world"
                elif owner.setdefault(d, slot) != slot:
                    yield f"device {d} used twice"
            if d_ranks := [self._rank_of[d] for d in g.devices if d in world]:
                if d_ranks != sorted(d_ranks):
                    yield f"group {tag} devices must be in ascending rank order"
        if world - set(owner):
            yield f"world contains devices outside any group: {sorted(world - set(owner))}"
        if world & set(self.standby):
            yield "standby devices cannot be in the world"

    def _check_layout(self):
        for s in range(self.num_stages):
            here = self._staged.get(s)
            if not here:
                yield f"stage {s} has no group"
                return
            if len({g.layers for g in here}) > 1:
                yield f"stage {s} layer ranges differ across replicas"
        bounds = self.layer_partition()
        contiguous = all(a[1] == b[0] for a, b in zip(bounds, bounds[1:]))
        if not (contiguous and bounds[0][0] == 0 and bounds[-1][1] == self.num_layers):
            yield f"layer partition {bounds} does not tile [0, {self.num_layers})"

    def _check_assignment(self):
        if len(self.assignment) != self.num_stages:
            yield "assignment must have one row per stage"
            return
        for s, row in enumerate(self.assignment):
            if len(row) != self.num_microbatches:
                yield f"assignment row {s} has {len(row)} entries"
            for m, r in enumerate(row):
                if (r, s) not in self._keyed:
                    yield f"micro-batch {m} stage {s} assigned to missing replica {r}"

    def validate(self) -> None:
        """Raise ``ValueError`` with the first rule the plan breaks."""
        if self.vpp < 1 or self.num_stages % self.vpp:
            raise ValueError(f"{self.num_stages} stages cannot be split into {self.vpp} chunks per physical stage")
        for check in (self._check_groups, self._check_layout, self._check_assignment):
            problem = next(check(), None)
            if problem is not None:
                raise ValueError(problem)

    # ------------------------------------------------------------------ process groups
    def tp_slices(self, stage: int) -> list[tuple[str, ...]]:
        """Every TP partition of a stage (one per replica and CP slice).  Each holds a full copy of
        the stage's parameters, so gradients reduce over all of them (DP x CP)."""
        return [g.slice(i) for g in self.groups_at(stage) for i in range(g.cp)]

    def dpshard_holder_sets(self, stage: int, partition_sizes) -> list[tuple[int, ...]]:
        """Reduction groups of shard-aligned DP: each partitioned length ``n`` is split evenly by
        every TP partition's degree, and on the common refinement of those splits every interval
        has exactly one holder per partition -- those holders reduce that interval together."""
        slices = self.tp_slices(stage)
        found: dict[tuple[int, ...], None] = {}
        for n in sorted(set(partition_sizes)):
            splits = [even_split(n, len(sl)) for sl in slices]
            for piece in refine(splits):
                holders = sorted(self.rank(sl[locate(split, piece)]) for sl, split in zip(slices, splits))
                found.setdefault(tuple(holders))
        return list(found)

    def group_specs(self, partition_sizes) -> list[GroupSpec]:
        """Every TP, CP and shard-aligned DP process group the plan needs (size > 1 for TP and
        DP, every CP group), each named as above."""
        specs: dict[str, GroupSpec] = {}

        def add(name, ranks, kind):
            specs.setdefault(name, GroupSpec(name, tuple(ranks), kind))

        for g in self.stage_groups:
            if g.tp > 1:
                for i in range(g.cp):
                    add(tp_group_name(g.replica, g.stage, i if g.cp > 1 else None),
                        sorted(self.slice_ranks(g, i)), "tp")
            if g.cp > 1:
                for j in range(g.tp):
                    add(cp_group_name(g.replica, g.stage, j), sorted(map(self.rank, g.cp_peers(j))), "cp")
        for s in range(self.num_stages):
            for holders in self.dpshard_holder_sets(s, partition_sizes):
                if len(holders) > 1:
                    add(dpshard_group_name(s, holders), holders, "dpshard")
        return list(specs.values())

    # ------------------------------------------------------------------ serialisation
    def to_json(self) -> dict:
        out = {k: getattr(self, k) for k in _scalar_fields()}
        out.update(world=list(self.world), stage_groups=[g.to_json() for g in self.stage_groups],
                   assignment=[list(row) for row in self.assignment], standby=list(self.standby),
                   sequence_parallel=self.sequence_parallel, meta=self.meta)
        ordered = {k: out[k] for k in ("generation", "world", "num_layers", "num_stages", "num_replicas",
                                       "stage_groups", "num_microbatches", "assignment", "standby",
                                       "sequence_parallel", "meta")}
        if self.vpp != 1:
            ordered["vpp"] = self.vpp
        return ordered

    @classmethod
    def from_json(cls, d: dict) -> "HeteroParallelPlan":
        return cls(world=tuple(d["world"]), stage_groups=tuple(map(StageGroup.from_json, d["stage_groups"])),
                   assignment=tuple(map(tuple, d["assignment"])), standby=tuple(d.get("standby", ())),
                   sequence_parallel=d.get("sequence_parallel", False), meta=d.get("meta", {}),
                   vpp=d.get("vpp", 1), **{k: d[k] for k in _scalar_fields()})


def interleave(plan: HeteroParallelPlan, vpp: int) -> HeteroParallelPlan:
    """Split every physical stage's layers evenly into ``vpp`` chunks; chunk ``c`` of physical
    stage ``p`` becomes virtual stage ``c * P + p`` (Megatron's interleaved layout)."""
    if vpp == 1:
        return plan
    P = plan.num_stages
    sizes = [0] * (P * vpp)
    for p in range(P):
        for c, (lo, hi) in enumerate(even_split(plan.groups_at(p)[0].num_layers, vpp)):
            sizes[c * P + p] = hi - lo
    if min(sizes) < 1:
        raise ValueError(f"stage layer counts cannot be split into {vpp} chunks")
    edges = list(itertools.accumulate(sizes, initial=0))

    def chunk(g: StageGroup, c: int) -> StageGroup:
        v = c * P + g.stage
        return StageGroup(g.replica, v, g.devices, (edges[v], edges[v + 1]), g.cp)

    groups = tuple(chunk(g, c) for c in range(vpp) for g in plan.stage_groups)
    rows = tuple(plan.assignment[v % P] for v in range(P * vpp))
    return replace(plan, num_stages=P * vpp, stage_groups=groups, assignment=rows, vpp=vpp)
