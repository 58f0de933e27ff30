"""``resihp-inject``: print or run a fault schedule against a cluster.

    resihp-inject "hang@time=5:target=n0g1:pid=1234:duration=10" [--execute] [--allow-device-settings]
Dry run by default (commands are printed, nothing changes).  (Reference: ``resihp/inject/cli.py``.)
"""

from __future__ import annotations

import argparse
import json
import shlex

from .faults import ExternalInjector, parse_faults, run_schedule


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="resihp-inject")
    ap.add_argument("spec", help="fault spec, e.g. kill@time=3:target=n0g1:pid=123")
    ap.add_argument("--execute", action="store_true", help="run the commands (default: dry run)")
    ap.add_argument("--allow-device-settings", action="store_true",
                    help="permit clock-lock / power-cap / XID commands (never on shared GPUs)")
    ap.add_argument("--list", action="store_true", help="only print the apply/revert commands")
    a = ap.parse_args(argv)
    faults = parse_faults(a.spec)
    inj = ExternalInjector(dry_run=not a.execute, allow_device_settings=a.allow_device_settings)
    if a.list:
        for f in faults:
            c = inj.commands(f)
            print(json.dumps({"fault": f.to_spec(), "apply": shlex.join(c.apply),
                              "revert": shlex.join(c.revert) if c.revert else None}))
        return 0
    for at, f, action in run_schedule(faults, inj):
        print(f"{at:8.2f}s {action:6s} {f.to_spec()}")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
