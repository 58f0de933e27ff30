"""Parses Megatron-LM training logs into per-iteration records, to compare a Megatron-Core run
of the same model and config on the same box (``resihp-bench megatron-log <file> [seq_len]``).
Parity: ``resihp/bench/megatron_log.py:1-70`` (the log line format is Megatron's).
"""

from __future__ import annotations

import json
import re
import statistics
import sys
from dataclasses import asdict, dataclass

_ITERATION = re.compile(r"iteration\s+(\d+)/\s*(\d+)")
_PAIR = re.compile(r"\|\s*([^|:]+?):\s*([-+0-9.eE]+)")
# record field -> the label Megatron prints before the value
_LABELS = {"iter_time_ms": "elapsed time per iteration (ms)", "tflops_per_gpu": "throughput per GPU (TFLOP/s/GPU)",
           "lm_loss": "lm loss", "global_batch_size": "global batch size"}


@dataclass
class IterRecord:
    iteration: int
    iter_time_ms: float | None
    tflops_per_gpu: float | None
    lm_loss: float | None
    global_batch_size: int | None


def parse_line(line: str) -> IterRecord | None:
    """One training-iteration line, or None for any other line."""
    found = _ITERATION.search(line)
    if found is None or _LABELS["iter_time_ms"] not in line:
        return None
    values = {label.strip(): float(number) for label, number in _PAIR.findall(line)}
    fields = {name: values.get(label) for name, label in _LABELS.items()}
    if fields["global_batch_size"] is not None:
        fields["global_batch_size"] = int(fields["global_batch_size"])
    return IterRecord(iteration=int(found.group(1)), **fields)


def parse_log(text: str) -> list[IterRecord]:
    return [rec for rec in (parse_line(line) for line in text.splitlines()) if rec is not None]


def _median(values) -> float | None:
    values = [v for v in values if v is not None]
    return statistics.median(values) if values else None


def summarize(records: list[IterRecord], skip_first: int = 2, seq_len: int | None = None) -> dict:
    """Medians over the steady iterations (after ``skip_first``), the loss curve, and tokens/s
    when the sequence length is given."""
    steady = [r for r in records[skip_first:] if r.iter_time_ms is not None] or records
    curve = [(r.iteration, r.lm_loss) for r in records if r.lm_loss is not None]
    summary = {"iterations": len(records), "median_iter_time_ms": _median(r.iter_time_ms for r in steady),
               "median_tflops_per_gpu": _median(r.tflops_per_gpu for r in steady),
               "final_loss": curve[-1][1] if curve else None, "loss_curve": curve}
    batch = next((r.global_batch_size for r in steady if r.global_batch_size), None)
    if seq_len and batch and summary["median_iter_time_ms"]:
        summary["tokens_per_s"] = batch * seq_len * 1000.0 / summary["median_iter_time_ms"]
    return summary


def main(argv: list[str] | None = None) -> int:
    args = sys.argv[1:] if argv is None else argv
    text = open(args[0]).read() if args else sys.stdin.read()
    records = parse_log(text)
    seq_len = int(args[1]) if len(args) > 1 else None
    print(json.dumps({"summary": summarize(records, seq_len=seq_len), "records": list(map(asdict, records))},
                     indent=2))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
