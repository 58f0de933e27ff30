"""``resihp-run``: start a coordinator, a node agent, or a whole job on one host.

    resihp-run coordinator --port 29400 --expected-workers 16
    resihp-run agent --node-id n0 --coordinator c0:29400,c1:29400 --nproc 8 -- python train.py ...
    resihp-run local --nnodes 2 --nproc-per-node 4 -- python examples/gpt_dp_demo.py

The subcommands and flags are the reference's (``resihp/control/launcher.py:50-126``), so job
scripts carry over.  The planner is given as ``module:function``; the KV backend is ``memory``
or ``etcd://host:port``.
"""

from __future__ import annotations

import argparse
import importlib
import signal
import threading
import time

from .agent import NodeAgent
from .coordinator import Coordinator
from .health import CompositeProbe, IBPortProbe, NVMLProbe
from .kvstore import InMemoryKV
from ..utils.rpc import parse_addr

# (flag, argparse keyword arguments) per subcommand
_FLAGS = {
    "coordinator": [("--host", dict(default="0.0.0.0")), ("--port", dict(type=int, default=29400)),
                    ("--store-port", dict(type=int, default=29401)), ("--expected-workers", dict(type=int)),
                    ("--min-workers", dict(type=int, default=1)), ("--lease-timeout", dict(type=float, default=3.0)),
                    ("--hang-timeout", dict(type=float, default=300.0)), ("--kv", dict(default="memory")),
                    ("--planner", dict(help="module:function implementing PlannerFn")),
                    ("--id", dict(default="coord-0")),
                    ("--leader-ttl", dict(type=float, help="enable HA election through the KV store"))],
    "agent": [("--node-id", dict(required=True)),
              ("--coordinator", dict(required=True, help="comma-separated host:port list (HA replicas)")),
              ("--nproc", dict(type=int, default=8)),
              ("--devices", dict(default="", help="comma-separated device list, default cuda:0..nproc-1")),
              ("--host", dict(default="127.0.0.1")), ("cmd", dict(nargs=argparse.REMAINDER))],
    "local": [("--nnodes", dict(type=int, default=2)), ("--nproc-per-node", dict(type=int, default=2)),
              ("--planner", {}), ("--hang-timeout", dict(type=float, default=60.0)),
              ("cmd", dict(nargs=argparse.REMAINDER))],
}


def load_planner(spec: str | None):
    """``"package.module:function"`` -> the function (None for an empty spec)."""
    if not spec:
        return None
    module_name, _, attr = spec.partition(":")
    return getattr(importlib.import_module(module_name), attr)


def make_kv(spec: str):
    if spec == "memory":
        return InMemoryKV()
    scheme = "etcd://"
    if not spec.startswith(scheme):
        raise ValueError(f"unknown kv backend {spec!r}")
    from .kvstore import EtcdKV

    return EtcdKV(*parse_addr(spec[len(scheme):]))


def build_parser() -> argparse.ArgumentParser:
    parser = argparse.ArgumentParser(prog="resihp-run")
    roles = parser.add_subparsers(dest="role", required=True)
    for role, flags in _FLAGS.items():
        sub = roles.add_parser(role)
        for name, kw in flags:
            sub.add_argument(name, **kw)
    return parser


def _command(args) -> list[str]:
    cmd = list(args.cmd or [])
    return cmd[1:] if cmd[:1] == ["--"] else cmd


def _serve_until_signalled() -> None:
    done = threading.Event()
    signal.signal(signal.SIGTERM, lambda *_: done.set())
    try:
        while not done.wait(0.5):
            pass
    except KeyboardInterrupt:
        pass


def _run_coordinator(args) -> int:
    coord = Coordinator(host=args.host, port=args.port, store_port=args.store_port, kv=make_kv(args.kv),
                        planner=load_planner(args.planner), expected_workers=args.expected_workers,
                        min_workers=args.min_workers, lease_timeout=args.lease_timeout, hang_timeout=args.hang_timeout,
                        coordinator_id=args.id, leader_ttl=args.leader_ttl).start()
    _serve_until_signalled()
    coord.stop()
    return 0


def _run_agent(args) -> int:
    replicas = list(map(parse_addr, args.coordinator.split(",")))
    devices = args.devices.split(",") if args.devices else [f"cuda:{i}" for i in range(args.nproc)]
    agent = NodeAgent(args.node_id, replicas, host=args.host,
                      health_probe=CompositeProbe(NVMLProbe(), IBPortProbe())).start()
    cmd = _command(args)
    if cmd:
        agent.spawn(cmd, args.nproc, devices=devices)
    _serve_until_signalled()
    agent.stop()
    return 0


def _run_local(args) -> int:
    """Coordinator plus ``nnodes`` simulated nodes on this host (CPU devices); returns the worst
    exit code among the final world's workers."""
    cmd = _command(args)
    coord = Coordinator(planner=load_planner(args.planner), expected_workers=args.nnodes * args.nproc_per_node,
                        hang_timeout=args.hang_timeout).start()
    agents = [NodeAgent(f"n{n}", [coord.address]).start() for n in range(args.nnodes)]
    for agent in agents:
        agent.spawn(cmd, args.nproc_per_node, devices=["cpu"] * args.nproc_per_node)
    procs = [(w.worker_id, w.proc) for agent in agents for w in agent.workers.values() if w.proc is not None]
    while any(proc.poll() is None for _, proc in procs):
        time.sleep(0.5)
    codes = [proc.returncode or 0 for wid, proc in procs if wid in coord.world]
    for agent in agents:
        agent.stop()
    coord.stop()
    return max(codes, default=1)


def main(argv: list[str] | None = None) -> int:
    args = build_parser().parse_args(argv)
    return {"coordinator": _run_coordinator, "agent": _run_agent, "local": _run_local}[args.role](args)


if __name__ == "__main__":
    raise SystemExit(main())
