"""A stand-in worker for the control-plane tests, steered by files in ``$TEST_TRIGGER_DIR``:

* ``stall_<id>`` -- the main loop sleeps for good (its heartbeat thread stays alive);
* ``collective`` -- every worker reports sitting inside a collective at op 10**6 and waits for
  the next notice, so only a stalled worker is behind;
* ``die_on_prepare_<id>`` -- the worker exits as soon as it sees a PREPARE.

Every committed generation, and every abort callback, is appended to ``$TEST_EVENT_LOG`` as one
JSON line."""

import json
import os
import sys
import time
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parents[2]))

from resihp_megatron_b200.control.worker_client import JobFinished, ReconfigInterrupted, WorkerClient  # noqa: E402


class _StandIn:
    def __init__(self):
        self.log = open(os.environ["TEST_EVENT_LOG"], "a")
        self.triggers = Path(os.environ["TEST_TRIGGER_DIR"])
        self.client = WorkerClient(hb_interval=0.1).connect()
        self.me = self.client.worker_id
        self.iteration = 0
        self.parked = False
        self.client.add_abort_callback(lambda: self.record(abort=True))

    def record(self, **fields) -> None:
        self.log.write(json.dumps({"worker": self.me, "t": time.time(), **fields}) + "\n")
        self.log.flush()

    def triggered(self, name: str) -> bool:
        return (self.triggers / name).exists()

    def join(self) -> dict | None:
        """One generation: PREPARE, READY (members only), COMMIT.  None when the job ended."""
        while True:
            try:
                prepare = self.client.wait_prepare(timeout=60)
            except (TimeoutError, JobFinished):
                return None
            if self.triggered(f"die_on_prepare_{self.me}"):
                os._exit(3)
            if self.me in prepare["world"]:
                self.client.send_ready(prepare["gen"])
            try:
                self.client.wait_commit(prepare["gen"], timeout=60)
            except ReconfigInterrupted:
                continue
            self.record(gen=prepare["gen"], world=prepare["world"])
            return prepare

    def work(self) -> None:
        """Make progress until the next notice (or stall / park as the triggers say)."""
        while not self.client.reconfig_pending():
            if self.triggered(f"stall_{self.me}"):
                time.sleep(3600)
            if not self.parked and self.triggered("collective"):
                self.parked = True
                self.client.set_progress(iteration=self.iteration, in_collective=True, op_seq=10 ** 6)
                while not self.client.reconfig_pending():
                    time.sleep(0.02)
                return
            self.client.set_progress(iteration=self.iteration, in_collective=False, op_seq=self.iteration)
            self.client.set_recovery_info(committed_iteration=self.iteration)
            self.iteration += 1
            time.sleep(0.02)


def main() -> None:
    worker = _StandIn()
    while (prepare := worker.join()) is not None:
        if worker.me in prepare["world"]:
            worker.work()


if __name__ == "__main__":
    main()
