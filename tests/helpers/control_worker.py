"""Stand-in worker for control-plane tests, steered by files in ``$TEST_TRIGGER_DIR``:

* ``stall_<id>``            the main loop sleeps forever (heartbeat thread stays alive);
* ``collective``            every worker reports being inside a collective at op 10**6 and waits
                            for the next notice (so only the stalled one is behind);
* ``die_on_prepare_<id>``   the worker exits as soon as it sees a PREPARE.

Each committed generation (and each abort callback) is appended to ``$TEST_EVENT_LOG`` as one JSON line."""

import json
import os
import sys
import time
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parents[2]))

from resihp_megatron_b200.control.worker_client import JobFinished, ReconfigInterrupted, WorkerClient  # noqa: E402


def main() -> None:
    log = open(os.environ["TEST_EVENT_LOG"], "a")
    triggers = Path(os.environ["TEST_TRIGGER_DIR"])
    client = WorkerClient(hb_interval=0.1).connect()
    me = client.worker_id

    def on_abort():
        log.write(json.dumps({"worker": me, "abort": True, "t": time.time()}) + "\n")
        log.flush()

    client.add_abort_callback(on_abort)
    it = 0
    parked = False
    while True:
        try:
            prep = client.wait_prepare(timeout=60)
        except (TimeoutError, JobFinished):
            return
        gen = prep["gen"]
        if (triggers / f"die_on_prepare_{me}").exists():
            os._exit(3)
        if me in prep["world"]:
            client.send_ready(gen)
        try:
            client.wait_commit(gen, timeout=60)
        except ReconfigInterrupted:
            continue
        log.write(json.dumps({"worker": me, "gen": gen, "world": prep["world"], "t": time.time()}) + "\n")
        log.flush()
        if me not in prep["world"]:
            continue
        while not client.reconfig_pending():
            if (triggers / f"stall_{me}").exists():
                time.sleep(3600)
            if not parked and (triggers / "collective").exists():
                parked = True
                client.set_progress(iteration=it, in_collective=True, op_seq=10 ** 6)
                while not client.reconfig_pending():
                    time.sleep(0.02)
                break
            client.set_progress(iteration=it, in_collective=False, op_seq=it)
            client.set_recovery_info(committed_iteration=it)
            it += 1
            time.sleep(0.02)


if __name__ == "__main__":
    main()
