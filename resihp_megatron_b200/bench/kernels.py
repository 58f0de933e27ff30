"""Kernel microbenchmarks with roofline fractions (``resihp-bench kernels``).

    python -m resihp_megatron_b200.bench.kernels gemm --m 8192 --n 8192 --k 8192
    python -m resihp_megatron_b200.bench.kernels fp8 --m 8192 --n 8192 --k 8192
    python -m resihp_megatron_b200.bench.kernels attention --batch 2 --seq 4096 --heads 32 --kv-heads 8
    python -m resihp_megatron_b200.bench.kernels adam --numel 1000000000
    python -m resihp_megatron_b200.bench.kernels all

Timing: ``--warmup`` untimed launches, then ``--iters`` launches each bracketed by CUDA events
on the launching stream with a synchronize on both sides; the median is reported.  Inputs of
the memory-bound kernels are larger than the 126 MB L2; for GEMMs an L2-sized buffer is
rewritten between timed launches (``--flush``).  Fractions are of the measured copy bandwidth
and cuBLAS bf16 throughput in ``MEASURED_PEAKS.json`` at the repository root when present,
otherwise of the fallback figures 6.65 TB/s and 1.59 PFLOP/s.  One JSON line per case.

The reference has no kernels of its own; its only compute probe is a cuBLAS matmul
(``resihp/detect/validation.py:17-31``), reported here as ``cublas`` beside our GEMM.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def peaks() -> dict:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


class Timer:
    def __init__(self, warmup: int, iters: int, flush: bool):
        self.warmup, self.iters = warmup, iters
        self.scratch = torch.empty(256 << 20, dtype=torch.uint8, device="cuda") if flush else None

    def __call__(self, fn) -> float:
        for _ in range(self.warmup):
            fn()
        torch.cuda.synchronize()
        times = []
        for _ in range(self.iters):
            if self.scratch is not None:
                self.scratch.fill_(1)  # evict L2 between launches
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            s.record()
            fn()
            e.record()
            torch.cuda.synchronize()
            times.append(s.elapsed_time(e))
        return statistics.median(times)


def emit(kind: str, ms: float, *, flops: float = 0.0, bytes_: float = 0.0, **extra) -> dict:
    pk = peaks()
    row = {"kernel": kind, "ms": round(ms, 4)}
    if flops:
        tf = flops / ms / 1e9
        row.update(tflops=round(tf, 1), frac_of_bf16_peak=round(tf / pk["bf16_tflops"], 3))
    if bytes_:
        gbs = bytes_ / ms / 1e6
        row.update(gbs=round(gbs, 1), frac_of_hbm=round(gbs / pk["hbm_gbs"], 3))
    row["peaks"] = pk["source"]
    row.update(extra)
    print(json.dumps(row), flush=True)
    return row


# (name, N, K) of the Llama-3-8B projections; M is the token count of a micro-batch
LLAMA3_8B_PROJ = (("qkv", 6144, 4096), ("o", 4096, 4096), ("gate_up", 28672, 4096), ("down", 4096, 14336),
                  ("head", 128256, 4096))


def bench_gemm_llama(a, t: Timer) -> None:
    """Every GEMM of a Llama-3-8B training step at ``--tokens`` tokens per micro-batch in the three
    layouts of a linear layer (forward NT, dgrad with B MN-major, wgrad with both MN-major and
    fp32 accumulation), beside cuBLAS on the same operands (``torch.matmul``; its wgrad writes
    bf16, so it does slightly less work); the forward also without split-K."""
    from .. import ops

    M = a.tokens
    for name, N, K in LLAMA3_8B_PROJ:
        fl = 2.0 * M * N * K
        x = torch.randn(M, K, device="cuda").bfloat16()
        w = torch.randn(N, K, device="cuda").bfloat16()
        dy = torch.randn(M, N, device="cuda").bfloat16()
        y = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        dx = torch.empty(M, K, device="cuda", dtype=torch.bfloat16)
        dw = torch.zeros(N, K, device="cuda")
        dwb = torch.empty(N, K, device="cuda", dtype=torch.bfloat16)
        rows = [("fwd", lambda: ops.gemm(x, w, out=y), lambda: torch.matmul(x, w.t(), out=y), [M, N, K]),
                ("dgrad", lambda: ops.gemm(dy, w, b_t=True, out=dx), lambda: torch.matmul(dy, w, out=dx), [M, K, N]),
                ("wgrad", lambda: ops.gemm(dy, x, a_t=True, b_t=True, out=dw, accumulate=True),
                 lambda: torch.matmul(dy.t(), x, out=dwb), [N, K, M]),
                ("fwd_nosplit", lambda: ops.gemm(x, w, out=y, variant=2), None, [M, N, K])]
        for layout, ours, cublas, shape in rows:
            r1 = emit(f"gemm_llama_{name}_{layout}", t(ours), flops=fl, shape=shape)
            if cublas is None:
                continue
            r2 = emit(f"cublas_llama_{name}_{layout}", t(cublas), flops=fl, shape=shape)
            print(json.dumps({"kernel": f"ratio_llama_{name}_{layout}", "ours_over_cublas":
                              round(r1["tflops"] / r2["tflops"], 3)}), flush=True)
        del x, w, dy, y, dx, dw, dwb
    assert int(ops.error_state()[0]) == 0


def bench_gemm(a, t: Timer) -> None:
    from .. import ops

    M, N, K = a.m, a.n, a.k
    x = torch.randn(M, K, device="cuda").bfloat16()
    w = torch.randn(N, K, device="cuda").bfloat16()
    out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    fl = 2.0 * M * N * K
    emit("gemm_tcgen05_nt", t(lambda: ops.gemm(x, w, out=out)), flops=fl, shape=[M, N, K])
    emit("gemm_tcgen05_nt_pair_nosplit", t(lambda: ops.gemm(x, w, out=out, variant=2)), flops=fl, shape=[M, N, K])
    emit("gemm_tcgen05_nt_pair_split2", t(lambda: ops.gemm(x, w, out=out, variant=3)), flops=fl, shape=[M, N, K])
    emit("gemm_tcgen05_nt_pair_7stages", t(lambda: ops.gemm(x, w, out=out, variant=4)), flops=fl, shape=[M, N, K])
    xt = x.t().contiguous()
    emit("gemm_tcgen05_tn", t(lambda: ops.gemm(xt, w, a_t=True, out=out)), flops=fl, shape=[M, N, K])
    emit("cublas", t(lambda: torch.matmul(x, w.t(), out=out)), flops=fl, shape=[M, N, K])
    assert int(ops.error_state()[0]) == 0


def bench_fp8(a, t: Timer) -> None:
    """Block-scaled fp8: the GEMM in its forward layout (1 x 128 row scales x 128 x 128 weight
    tiles) and its weight-gradient layout (per-column scales), the quantiser and the fused
    RMSNorm -> fp8, beside cuBLAS fp8 with one scale per tensor (``torch._scaled_mm``) when the
    installed PyTorch offers it.  GEMM fractions are of twice the measured bf16 peak (the dense
    fp8 rate is twice the bf16 rate)."""
    from .. import ops
    from ..ops import fp8

    M, N, K = a.m, a.n, a.k
    fl = 2.0 * M * N * K
    pk = peaks()
    x = torch.randn(M, K, device="cuda").bfloat16()
    w = (torch.randn(N, K, device="cuda") * 0.05).bfloat16()
    xq = fp8.quantize(x, fp8.E4M3, rowwise=True, colwise=True)
    wq = fp8.quantize(w, fp8.E4M3, two_d=True, rowwise=True, colwise=True)
    out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)

    def frac(row):
        if "tflops" in row:
            row["frac_of_2x_bf16_peak"] = round(row["tflops"] / (2 * pk["bf16_tflops"]), 3)
            print(json.dumps({"kernel": row["kernel"], "frac_of_2x_bf16_peak": row["frac_of_2x_bf16_peak"]}),
                  flush=True)

    frac(emit("gemm_fp8_fwd_blockscaled", t(lambda: fp8.gemm(xq.rowwise(), wq.rowwise(), out=out)), flops=fl,
              shape=[M, N, K]))
    frac(emit("gemm_fp8_fwd_register_promotion", t(lambda: fp8.gemm(xq.rowwise(), wq.rowwise(), out=out, variant=1)),
              flops=fl, shape=[M, N, K]))
    # weight-gradient layout: both operands scaled per row along K (per-column scales of B)
    dy = torch.randn(K, M, device="cuda").bfloat16()
    dyq = fp8.quantize(dy, fp8.E5M2, rowwise=True)
    g = torch.zeros(K, N, device="cuda")
    xq2 = fp8.quantize(torch.randn(N, M, device="cuda").bfloat16(), fp8.E4M3, rowwise=True)
    frac(emit("gemm_fp8_wgrad_blockscaled", t(lambda: fp8.gemm(dyq.rowwise(), xq2.rowwise(), out=g, accumulate=True)),
              flops=fl, shape=[K, N, M]))
    frac(emit("gemm_fp8_wgrad_register_promotion",
              t(lambda: fp8.gemm(dyq.rowwise(), xq2.rowwise(), out=g, accumulate=True, variant=1)),
              flops=fl, shape=[K, N, M]))
    try:
        a8, b8 = x.to(torch.float8_e4m3fn), w.to(torch.float8_e4m3fn)
        one = torch.ones((), device="cuda")
        frac(emit("cublas_fp8_tensorwise", t(lambda: torch._scaled_mm(a8, b8.t(), scale_a=one, scale_b=one,
                                                                         out_dtype=torch.bfloat16)),
                  flops=fl, shape=[M, N, K]))
    except Exception as e:  # noqa: BLE001
        print(json.dumps({"kernel": "cublas_fp8_tensorwise", "unavailable": str(e)[:200]}), flush=True)
    # bandwidth-bound producers (bf16 in, fp8 + scales out)
    T, H = a.tokens, a.hidden
    xt = torch.randn(T, H, device="cuda").bfloat16()
    buf = fp8.Fp8Tensor.empty(T, H, fp8.E4M3, rowwise=True, colwise=True, device="cuda")
    emit("fp8_quantize_row_col", t(lambda: fp8.quantize(xt, fp8.E4M3, rowwise=True, colwise=True, out=buf)),
         bytes_=T * H * (2 + 1 + 1), shape=[T, H])
    nw = torch.ones(H, device="cuda").bfloat16()
    rbuf = fp8.Fp8Tensor.empty(T, H, fp8.E4M3, device="cuda")
    rstd = torch.empty(T, device="cuda")
    emit("rmsnorm_fp8", t(lambda: fp8.rmsnorm_quantize(xt, nw, 1e-5, fp8.E4M3, out=rbuf, rstd=rstd)),
         bytes_=T * H * (2 + 1), shape=[T, H])
    assert int(ops.error_state()[0]) == 0


def bench_attention(a, t: Timer) -> None:
    from .. import ops

    B, S, Hq, Hkv, D = a.batch, a.seq, a.heads, a.kv_heads, 128
    qkv = torch.randn(B * S, (Hq + 2 * Hkv) * D, device="cuda").bfloat16()
    q, k, v = qkv[:, : Hq * D], qkv[:, Hq * D:(Hq + Hkv) * D], qkv[:, (Hq + Hkv) * D:]
    kw = dict(batch=B, seq=S, heads=Hq, kv_heads=Hkv, head_dim=D)
    fwd_flops = 4.0 * B * Hq * S * S * D / 2  # causal
    impls = [("tcgen05", ops.ATTN_TCGEN05), ("mma", ops.ATTN_MMA)] if a.with_mma else [("tcgen05", ops.ATTN_TCGEN05)]
    o, lse = ops.attention_fwd(q, k, v, **kw)
    dout = torch.randn_like(o)
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    if a.fwd_variants:  # share of the softmax exponentials on the FMA pipe, 0..3 of every 8
        ref = ops.attention_fwd(q, k, v, impl=ops.ATTN_TCGEN05, variant=0, **kw)[0].float()
        for var in range(4):
            o_var = ops.attention_fwd(q, k, v, impl=ops.ATTN_TCGEN05, variant=var, **kw)[0]
            emit(f"attention_fwd_tcgen05_fma{var}of8",
                 t(lambda: ops.attention_fwd(q, k, v, out=o, lse=lse, impl=ops.ATTN_TCGEN05, variant=var, **kw)),
                 flops=fwd_flops, shape=[B, S, Hq, Hkv, D],
                 max_abs_diff_vs_mufu=float((o_var.float() - ref).abs().max()))
            emit(f"attention_bwd_tcgen05_fma{var}of8",
                 t(lambda: ops.attention_bwd(q, k, v, o, dout, lse, dq, dk, dv, impl=ops.ATTN_TCGEN05, variant=var,
                                             **kw)),
                 flops=2.5 * fwd_flops, shape=[B, S, Hq, Hkv, D])
    for name, impl in impls:
        emit(f"attention_fwd_{name}", t(lambda: ops.attention_fwd(q, k, v, out=o, lse=lse, impl=impl, **kw)),
             flops=fwd_flops, shape=[B, S, Hq, Hkv, D])
        emit(f"attention_bwd_{name}",
             t(lambda: ops.attention_bwd(q, k, v, o, dout, lse, dq, dk, dv, impl=impl, **kw)),
             flops=2.5 * fwd_flops, shape=[B, S, Hq, Hkv, D])
    assert int(ops.error_state()[0]) == 0


def bench_adam(a, t: Timer) -> None:
    from .. import ops

    n = a.numel
    p = torch.randn(n, device="cuda")
    g = torch.randn(n, device="cuda")
    m = torch.zeros(n, device="cuda")
    v = torch.zeros(n, device="cuda")
    pb = torch.empty(n, device="cuda", dtype=torch.bfloat16)
    step = [0]

    def run():
        step[0] += 1
        ops.adam_step(p, g, m, v, pb, lr=1e-4, step=step[0], zero_grad=False)

    # reads p, g, m, v (16 B) and writes p, m, v, bf16 copy (14 B) per element
    emit("adam_fused", t(run), bytes_=30.0 * n, numel=n)


def bench_norm(a, t: Timer) -> None:
    from .. import ops

    T, H = a.tokens, a.hidden
    x = torch.randn(T, H, device="cuda").bfloat16()
    w = torch.ones(H, device="cuda").bfloat16()
    y, rstd = ops.rmsnorm_fwd(x, w)
    emit("rmsnorm_fwd", t(lambda: ops.rmsnorm_fwd(x, w, out=y)), bytes_=4.0 * T * H, shape=[T, H])
    dy = torch.randn_like(x)
    dw = torch.zeros(H, device="cuda")
    emit("rmsnorm_bwd", t(lambda: ops.rmsnorm_bwd(x, w, rstd, dy, dw)), bytes_=6.0 * T * H, shape=[T, H])
    gu = torch.randn(T, 2 * a.ffn, device="cuda").bfloat16()
    act = torch.empty(T, a.ffn, device="cuda", dtype=torch.bfloat16)
    emit("swiglu_fwd", t(lambda: ops.swiglu_fwd(gu, out=act)), bytes_=6.0 * T * a.ffn, shape=[T, a.ffn])


def bench_ce(a, t: Timer) -> None:
    from .. import ops

    T, V = a.tokens, a.vocab
    logits = torch.randn(T, V, device="cuda").bfloat16()
    labels = torch.randint(0, V, (T,), device="cuda")
    emit("cross_entropy_fwd_bwd", t(lambda: ops.cross_entropy_(logits, labels, grad_scale=1.0 / T)),
         bytes_=4.0 * T * V, shape=[T, V])


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(prog="resihp-bench kernels")
    ap.add_argument("which", choices=["gemm", "gemm-llama", "fp8", "attention", "adam", "norm", "ce", "all"])
    ap.add_argument("--m", type=int, default=8192)
    ap.add_argument("--n", type=int, default=8192)
    ap.add_argument("--k", type=int, default=8192)
    ap.add_argument("--batch", type=int, default=2)
    ap.add_argument("--seq", type=int, default=4096)
    ap.add_argument("--heads", type=int, default=32)
    ap.add_argument("--kv-heads", type=int, default=8)
    ap.add_argument("--with-mma", action="store_true", help="also time the mma.sync attention kernels")
    ap.add_argument("--fwd-variants", action="store_true",
                    help="attention: also time 0-3 of every 8 softmax exponentials on the FMA pipe")
    ap.add_argument("--numel", type=int, default=1 << 28)
    ap.add_argument("--tokens", type=int, default=16384)
    ap.add_argument("--hidden", type=int, default=4096)
    ap.add_argument("--ffn", type=int, default=14336)
    ap.add_argument("--vocab", type=int, default=128256)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--no-flush", action="store_true")
    a = ap.parse_args(argv)
    if not torch.cuda.is_available():
        raise SystemExit("kernel benchmarks need a GPU")
    t = Timer(a.warmup, a.iters, not a.no_flush)
    table = {"gemm": bench_gemm, "gemm-llama": bench_gemm_llama, "fp8": bench_fp8, "attention": bench_attention, "adam": bench_adam,
             "norm": bench_norm, "ce": bench_ce}
    for name in (table if a.which == "all" else [a.which]):
        table[name](a, t)


if __name__ == "__main__":
    main()
