"""Control-plane message vocabulary (worker <-> NodeAgent <-> Coordinator).

The names are part of the public contract and match the reference
(``resihp/control/protocol.py:8-37``).  Every message that belongs to a reconfiguration
carries ``gen``; a receiver drops anything older than the generation it has moved to,
which fences stale actors.
"""

# worker -> agent
REGISTER = "REGISTER"
HEARTBEAT = "HEARTBEAT"
ABORTED = "ABORTED"        # gen, committed_iteration, has_reduced_grads, inflight_iteration
READY = "READY"            # gen
REPORT = "REPORT"          # kind (timing | build_failed | done | fatal | replan | ...), detail

# agent -> coordinator
AGENT_REGISTER = "AGENT_REGISTER"
WORKER_REGISTER = "WORKER_REGISTER"
NODE_HEARTBEAT = "NODE_HEARTBEAT"
WORKER_FAILED = "WORKER_FAILED"
WORKER_MSG = "WORKER_MSG"

# coordinator -> agent
KILL = "KILL"
TO_WORKER = "TO_WORKER"
COORDINATOR_HELLO = "COORDINATOR_HELLO"

# coordinator -> worker (relayed by the agent)
RECONFIG_NOTICE = "RECONFIG_NOTICE"  # gen, failed, immediate, reason
PREPARE = "PREPARE"                  # gen, world, payload, store_addr, store_prefix, recovery
COMMIT = "COMMIT"                    # gen
SELF_FENCE = "SELF_FENCE"            # the agent lost every coordinator for longer than the lease
SHUTDOWN = "SHUTDOWN"                # the whole world reported done

ALL = (REGISTER, HEARTBEAT, ABORTED, READY, REPORT, AGENT_REGISTER, WORKER_REGISTER, NODE_HEARTBEAT,
       WORKER_FAILED, WORKER_MSG, KILL, TO_WORKER, COORDINATOR_HELLO, RECONFIG_NOTICE, PREPARE, COMMIT,
       SELF_FENCE, SHUTDOWN)


def msg(msg_type: str, /, **fields) -> dict:
    out = dict(fields)
    out["type"] = msg_type
    return out
