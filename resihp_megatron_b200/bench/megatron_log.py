"""Parse Megatron-LM training logs into per-iteration records, for comparing a Megatron-Core
run of the same model/config on the same box (``resihp-bench megatron-log <file>``).
(Reference: ``resihp/bench/megatron_log.py:1-70``; the log line format is Megatron's.)
"""

from __future__ import annotations

import json
import re
import statistics
import sys
from dataclasses import asdict, dataclass

_ITER = re.compile(r"iteration\s+(\d+)/\s*(\d+)")
_FIELD = re.compile(r"\|\s*([^|:]+?):\s*([-+0-9.eE]+)")


@dataclass
class IterRecord:
    iteration: int
    iter_time_ms: float | None
    tflops_per_gpu: float | None
    lm_loss: float | None
    global_batch_size: int | None


def parse_line(line: str) -> IterRecord | None:
    m = _ITER.search(line)
    if m is None or "elapsed time per iteration" not in line:
        return None
    fields = {k.strip(): float(v) for k, v in _FIELD.findall(line)}
    gbs = fields.get("global batch size")
    return IterRecord(int(m.group(1)), fields.get("elapsed time per iteration (ms)"),
                      fields.get("throughput per GPU (TFLOP/s/GPU)"), fields.get("lm loss"),
                      int(gbs) if gbs is not None else None)


def parse_log(text: str) -> list[IterRecord]:
    return [r for r in map(parse_line, text.splitlines()) if r is not None]


def summarize(records: list[IterRecord], skip_first: int = 2, seq_len: int | None = None) -> dict:
    steady = [r for r in records[skip_first:] if r.iter_time_ms is not None] or records
    times = [r.iter_time_ms for r in steady if r.iter_time_ms is not None]
    tflops = [r.tflops_per_gpu for r in steady if r.tflops_per_gpu is not None]
    losses = [(r.iteration, r.lm_loss) for r in records if r.lm_loss is not None]
    out = {"iterations": len(records), "median_iter_time_ms": statistics.median(times) if times else None,
           "median_tflops_per_gpu": statistics.median(tflops) if tflops else None,
           "final_loss": losses[-1][1] if losses else None, "loss_curve": losses}
    gbs = next((r.global_batch_size for r in steady if r.global_batch_size), None)
    if seq_len and gbs and out["median_iter_time_ms"]:
        out["tokens_per_s"] = gbs * seq_len / (out["median_iter_time_ms"] / 1000.0)
    return out


def main(argv: list[str] | None = None) -> int:
    argv = sys.argv[1:] if argv is None else argv
    text = open(argv[0]).read() if argv else sys.stdin.read()
    seq = int(argv[1]) if len(argv) > 1 else None
    recs = parse_log(text)
    print(json.dumps({"summary": summarize(recs, seq_len=seq), "records": [asdict(r) for r in recs]}, indent=2))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
