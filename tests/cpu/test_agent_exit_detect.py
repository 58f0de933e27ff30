"""The node agent sees a worker that has started to exit (``/proc/<pid>/stat``: the exiting task
flag, or a zombie) before its control connection closes -- for a killed GPU process the socket
closes only after the driver has unmapped its device memory."""

import signal
import subprocess
import sys
import time

from resihp_megatron_b200.control.agent import LocalWorker, parse_stat_exiting, pid_exiting


def test_parse_stat_fields_after_the_command_name():
    running = "4242 (python) S 1 4242 4242 0 -1 4194560 100 0 0 0 5 3 0 0 20 0 4 0 100 0 0"
    exiting = "4242 (python) R 1 4242 4242 0 -1 4194564 100 0 0 0 5 3 0 0 20 0 4 0 100 0 0"
    zombie = "4242 (python) Z 1 4242 4242 0 -1 4194560 100 0 0 0 5 3 0 0 20 0 4 0 100 0 0"
    odd_name = "4242 (a) (b c) S 1 4242 4242 0 -1 4194564 1 0 0 0 0 0 0 0 20 0 1 0 1 0 0"
    assert not parse_stat_exiting(running)
    assert parse_stat_exiting(exiting)  # flags 0x400004: the exiting bit
    assert parse_stat_exiting(zombie)
    assert parse_stat_exiting(odd_name)  # fields taken after the last ')'
    assert not parse_stat_exiting("garbage")


def test_killed_child_is_reported_before_it_is_reaped():
    proc = subprocess.Popen([sys.executable, "-c", "import time; time.sleep(60)"])
    try:
        w = LocalWorker("w0", 0, pid=proc.pid)  # a worker the agent adopted by pid (no Popen handle)
        assert not pid_exiting(proc.pid) and w.death_reason(time.monotonic(), 60.0) is None
        proc.send_signal(signal.SIGKILL)
        deadline = time.monotonic() + 5.0
        while not pid_exiting(proc.pid) and time.monotonic() < deadline:
            time.sleep(0.01)
        assert pid_exiting(proc.pid)  # not reaped yet: exiting or a zombie
        assert w.death_reason(time.monotonic(), 60.0) in ("process exiting", "process gone")
    finally:
        proc.kill()
        proc.wait()
