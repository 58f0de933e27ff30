"""GPU calibration of the planner's cost model from this package's own kernels.

    python -m resihp_megatron_b200.bench.profile_gpu --model llama3-8b --out profile.json \\
        [--tp-sample 2,32257,19295]

Times the forward and the backward of a few decoder layers of ``--model`` (no embedding, no LM
head) on one GPU at several micro-batch shapes -- token counts and squared document lengths that
differ, so the two terms of ``t = alpha * tokens + beta * sum(doc_len^2)`` separate -- with CUDA
events after warm-up, and fits ``ModelProfile`` by least squares (``ModelProfile.fit``).
``bwd_ratio`` is the measured backward / forward time.  ``--tp-sample k,tps_k,tps_1`` adds a
measured tokens/s at TP degree ``k`` and at TP 1 for the same model (e.g. from ``bench.py``),
which fixes ``tp_overhead``.  The JSON written to ``--out`` holds the samples and the profile;
``ModelProfile.calibrated`` finds it under ``plan/profiles/`` by layer shape, so the planner's
predictions rest on measured kernel times instead of nominal rates.
(Reference: ``resihp/plan/model_spec.py:52-83`` defines the same two-term model; its profiles are
analytic.)
"""

from __future__ import annotations

import argparse
import json
import statistics

# (micro-batch sequences, sequence length): tokens and sum of squared document lengths vary apart
SHAPES = ((1, 1024), (1, 2048), (1, 4096), (2, 2048), (4, 1024), (2, 4096))


def tp_samples_from_throughput(entries: list[tuple[int, float, float]]) -> list[tuple[int, float, float]]:
    """``(k, tokens/s at TP k, tokens/s at TP 1)`` -> ``ModelProfile.fit``'s ``(k, t_k, t_1)``: the
    time of one token's work on the k-GPU group and on one GPU."""
    return [(k, 1.0 / tps_k, 1.0 / tps_1) for k, tps_k, tps_1 in entries]


def fit_profile(samples: list[dict], tp_entries: list[tuple[int, float, float]] = ()):
    """``samples``: ``{"tokens", "sum_sq", "fwd_s", "bwd_s"}`` per layer -> ``ModelProfile``."""
    from ..plan.model_spec import ModelProfile

    ratios = [s["bwd_s"] / s["fwd_s"] for s in samples if s.get("bwd_s") and s["fwd_s"] > 0]
    fields = {"bwd_ratio": statistics.median(ratios)} if ratios else {}
    return ModelProfile.fit([(s["tokens"], s["sum_sq"], s["fwd_s"]) for s in samples],
                            tp_samples=tp_samples_from_throughput(list(tp_entries)), **fields)


def measure(model_name: str, layers: int = 2, warmup: int = 3, iters: int = 10, shapes=SHAPES) -> list[dict]:
    """Per-layer forward / backward seconds of ``layers`` middle decoder layers at each shape."""
    import torch

    from ..models.config import get_config
    from ..models.gpt import LlamaModel

    cfg = get_config(model_name)
    out = []
    for mb, seq in shapes:
        model = LlamaModel(cfg.with_(layers=layers, seq_len=seq), "cuda", micro_batch=mb, seq_len=seq,
                           layers=range(layers), first=False, last=False)
        x = (torch.randn(mb * seq, cfg.hidden, device="cuda") * 0.5).bfloat16()
        dy = (torch.randn(mb * seq, cfg.hidden, device="cuda") * 1e-3).bfloat16()
        fwd, both = [], []
        for i in range(warmup + iters):
            s, m, e = (torch.cuda.Event(enable_timing=True) for _ in range(3))
            torch.cuda.synchronize()
            s.record()
            model.forward(x_in=x)
            m.record()
            model.backward(dx_top=dy)
            e.record()
            torch.cuda.synchronize()
            if i >= warmup:
                fwd.append(s.elapsed_time(m) / 1e3)
                both.append(m.elapsed_time(e) / 1e3)
        out.append({"micro_batch": mb, "seq": seq, "tokens": mb * seq, "sum_sq": mb * seq * seq,
                    "fwd_s": statistics.median(fwd) / layers, "bwd_s": statistics.median(both) / layers})
        del model
        torch.cuda.empty_cache()
    return out


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--model", default="llama3-8b")
    ap.add_argument("--layers", type=int, default=2)
    ap.add_argument("--tp-sample", action="append", default=[],
                    help="k,tokens_per_s_at_k,tokens_per_s_at_1 (repeatable)")
    ap.add_argument("--out", default=None)
    args = ap.parse_args(argv)
    tp_entries = [tuple(float(x) for x in t.split(",")) for t in args.tp_sample]
    tp_entries = [(int(k), a, b) for k, a, b in tp_entries]
    samples = measure(args.model, args.layers)
    profile = fit_profile(samples, tp_entries)
    from ..models.config import get_config

    cfg = get_config(args.model)
    doc = {"model": args.model, "shape": {"hidden": cfg.hidden, "ffn": cfg.ffn, "heads": cfg.heads,
                                          "kv_heads": cfg.kv_heads},
           "samples": samples, "tp_samples": tp_entries, "profile": profile.to_json()}
    text = json.dumps(doc, indent=1)
    if args.out:
        with open(args.out, "w") as fh:
            fh.write(text + "\n")
    print(text, flush=True)


if __name__ == "__main__":
    main()
