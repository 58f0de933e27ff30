"""Chaos tests of the control plane with real worker processes (no GPU involved).

Faults are made on the host: SIGKILL, SIGSTOP (a hang without heartbeats), a whole node
vanishing (only the lease reveals it), a main-thread hang with a live heartbeat thread
(progress-based culprit detection), and a worker dying while a PREPARE is outstanding (the
transaction restarts at the next generation).  Every fault must be detected, fenced, and
followed by a committed generation that excludes exactly the failed workers."""

import json
import os
import signal
import sys
import time
from pathlib import Path

import pytest

pytestmark = pytest.mark.dist

ROOT = Path(__file__).resolve().parents[2]
HELPER = str(ROOT / "tests" / "helpers" / "control_worker.py")


def _wait(pred, timeout, what):
    deadline = time.monotonic() + timeout
    while time.monotonic() < deadline:
        if pred():
            return
        time.sleep(0.05)
    raise AssertionError(f"timed out waiting for {what}")


def _env(tmp_path):
    events, triggers = tmp_path / "events.jsonl", tmp_path / "triggers"
    triggers.mkdir(exist_ok=True)
    return events, triggers, {"TEST_EVENT_LOG": str(events), "TEST_TRIGGER_DIR": str(triggers),
                              "PYTHONPATH": str(ROOT) + os.pathsep + os.environ.get("PYTHONPATH", "")}


def test_kill_stop_node_loss_and_silent_hang_are_fenced(tmp_path):
    from resihp_megatron_b200.control.agent import NodeAgent
    from resihp_megatron_b200.control.coordinator import Coordinator

    events, triggers, env = _env(tmp_path)
    coord = Coordinator(expected_workers=6, lease_timeout=1.0, hang_timeout=1.5, abort_timeout=5.0,
                        ready_timeout=10.0, host_store=False).start()
    agents = {}
    try:
        for n in range(3):
            ag = NodeAgent(f"n{n}", [coord.address], hb_interval=0.1, worker_timeout=1.0).start()
            ag.spawn([sys.executable, HELPER], 2, env=env)
            agents[f"n{n}"] = ag
        assert coord.wait_for_commit(1, timeout=30)
        assert sorted(coord.world) == ["n0g0", "n0g1", "n1g0", "n1g1", "n2g0", "n2g1"]

        def committed_without(*gone):
            return lambda: (coord.phase == "running" and not set(gone) & set(coord.world)
                            and coord.committed_generation > 1)

        t0 = time.monotonic()
        os.kill(agents["n2"].workers["n2g1"].pid, signal.SIGKILL)
        _wait(committed_without("n2g1"), 15, "commit after SIGKILL")
        kill_latency = time.monotonic() - t0
        assert len(coord.world) == 5

        stopped = agents["n2"].workers["n2g0"]
        os.kill(stopped.pid, signal.SIGSTOP)
        _wait(committed_without("n2g0", "n2g1"), 15, "commit after SIGSTOP")
        _wait(lambda: stopped.proc.poll() is not None, 5, "the fenced process to be killed")

        lost = agents.pop("n1")
        lost.stop()
        for w in lost.workers.values():
            os.kill(w.pid, signal.SIGKILL)
        _wait(committed_without("n1g0", "n1g1"), 15, "commit after node loss")
        assert any("lease" in h.get("reason", "") for h in coord.history if h["event"] == "failure")

        (triggers / "stall_n0g0").touch()
        (triggers / "collective").touch()
        _wait(lambda: coord.world == ["n0g1"] and coord.phase == "running", 20, "commit after silent hang")
        hang = [h for h in coord.history if h["event"] == "failure" and h["workers"] == ["n0g0"]]
        assert hang and "hang" in hang[0]["reason"]

        last = {}
        for line in events.read_text().splitlines():
            r = json.loads(line)
            if "gen" in r:
                last[r["worker"]] = r
        assert last["n0g1"]["world"] == ["n0g1"] and last["n0g1"]["gen"] == coord.committed_generation
        gens = [h["generation"] for h in coord.history if h["event"] == "commit"]
        assert gens == sorted(gens) and len(gens) >= 5
        assert kill_latency < 5.0
    finally:
        for ag in agents.values():
            ag.stop(kill_workers=True)
        coord.stop()


def test_failure_during_prepare_restarts_the_transaction(tmp_path):
    from resihp_megatron_b200.control.agent import NodeAgent
    from resihp_megatron_b200.control.coordinator import Coordinator

    events, triggers, env = _env(tmp_path)
    coord = Coordinator(expected_workers=4, lease_timeout=1.0, hang_timeout=30, abort_timeout=5.0,
                        ready_timeout=10.0, host_store=False).start()
    agents = []
    try:
        for n in range(2):
            ag = NodeAgent(f"n{n}", [coord.address], hb_interval=0.1, worker_timeout=1.0).start()
            ag.spawn([sys.executable, HELPER], 2, env=env)
            agents.append(ag)
        assert coord.wait_for_commit(1, timeout=30)
        # n1g0 dies as soon as it sees the next PREPARE, i.e. inside the transaction for n0g1's loss
        (triggers / "die_on_prepare_n1g0").touch()
        os.kill(agents[0].workers["n0g1"].pid, signal.SIGKILL)
        _wait(lambda: coord.phase == "running" and sorted(coord.world) == ["n0g0", "n1g1"], 30,
              "commit without both failed workers")
        commits = [h for h in coord.history if h["event"] == "commit"]
        assert commits[-1]["generation"] >= 3, "the interrupted generation must not commit"
        committed = {e["gen"] for e in map(json.loads, events.read_text().splitlines()) if "gen" in e}
        assert 2 not in committed or commits[-1]["generation"] > 2
        assert agents[1].workers["n1g0"].proc.wait(timeout=5) == 3
    finally:
        for ag in agents:
            ag.stop(kill_workers=True)
        coord.stop()


def _events(path):
    return [json.loads(l) for l in path.read_text().splitlines()] if path.exists() else []


def test_leader_dies_mid_transaction_and_successor_completes_it(tmp_path):
    """Two coordinator replicas share a KV store.  The leader's planner blocks inside the
    transaction for generation 2; the leader dies; the standby takes the leader key, restores
    the half-finished transaction from KV and commits generation 3 (reason ``failover``).  The
    deposed leader's late writes are fenced off."""
    import threading

    from resihp_megatron_b200.control.agent import NodeAgent
    from resihp_megatron_b200.control.coordinator import Coordinator, keep_all_planner
    from resihp_megatron_b200.control.kvstore import InMemoryKV
    from tests.dist_utils import free_port

    events, triggers, env = _env(tmp_path)
    kv = InMemoryKV()
    release = threading.Event()

    def stuck(view):
        if view.generation >= 2:
            release.wait(30)
        return keep_all_planner(view)

    ports = [free_port(), free_port()]
    common = dict(kv=kv, expected_workers=4, lease_timeout=2.0, hang_timeout=60, abort_timeout=5.0,
                  ready_timeout=10.0, host_store=False, leader_ttl=0.6)
    leader = Coordinator(port=ports[0], planner=stuck, coordinator_id="c0", **common).start()
    standby = Coordinator(port=ports[1], planner=keep_all_planner, coordinator_id="c1",
                          **common).start(block_until_leader=False)
    addrs = [("127.0.0.1", p) for p in ports]
    agents = []
    try:
        for n in range(2):
            ag = NodeAgent(f"n{n}", addrs, hb_interval=0.1, worker_timeout=10.0, self_fence_after=10.0).start()
            ag.spawn([sys.executable, HELPER], 2, env=env)
            agents.append(ag)
        assert leader.wait_for_commit(1, timeout=30)
        leader.request_replan("planned")
        _wait(lambda: leader.generation >= 2, 10, "the leader to open generation 2")
        time.sleep(0.3)  # the open transaction is persisted
        leader.stop()
        _wait(lambda: standby.is_leader, 10, "the standby to take over")
        _wait(lambda: standby.committed_generation >= 3 and standby.phase == "running", 30, "the successor commit")
        release.set()
        time.sleep(0.5)
        history = standby.history
        assert history[-1]["event"] == "commit" and history[-1]["reason"] == "failover"
        evs = [e for e in _events(events) if "gen" in e]
        assert {e["worker"] for e in evs if e["gen"] == standby.committed_generation} == {
            "n0g0", "n0g1", "n1g0", "n1g1"}
        assert not any(e["gen"] == 2 for e in evs), "the interrupted generation never commits"
        state = json.loads(kv.get("resihp/state"))
        assert state["committed_generation"] == standby.committed_generation
        assert kv.get("resihp/leader") == "c1"
    finally:
        release.set()
        for ag in agents:
            ag.stop(kill_workers=True)
        standby.stop()
        leader.stop()


def test_agent_self_fences_workers_after_losing_the_coordinator(tmp_path):
    from resihp_megatron_b200.control.agent import NodeAgent
    from resihp_megatron_b200.control.coordinator import Coordinator

    events, triggers, env = _env(tmp_path)
    coord = Coordinator(expected_workers=2, lease_timeout=5.0, hang_timeout=60, host_store=False).start()
    ag = NodeAgent("n0", [coord.address], hb_interval=0.1, worker_timeout=10.0, self_fence_after=0.8).start()
    try:
        ag.spawn([sys.executable, HELPER], 2, env=env)
        assert coord.wait_for_commit(1, timeout=30)
        t0 = time.time()
        coord.stop()
        _wait(lambda: {e["worker"] for e in _events(events) if e.get("abort")} == {"n0g0", "n0g1"}, 10,
              "both workers to run their abort callbacks")
        first = min(e["t"] for e in _events(events) if e.get("abort"))
        assert first - t0 >= 0.7, "no self-fence before the grace period"
    finally:
        ag.stop(kill_workers=True)
        coord.stop()
