"""One pipeline stage of the Llama decoder on one tensor-parallel rank, with sequence parallelism.

Layout (Megatron's, on this package's kernels): q/k/v and gate/up projections are column
parallel (this rank holds ``heads / tp`` query heads, ``kv_heads / tp`` key/value heads and
``ffn / tp`` FFN columns), ``wo`` and ``w2`` are row parallel; the residual stream between the
projections is sharded by token rows (sequence parallel).  Per layer, ``T`` tokens of a
micro-batch, ``T / tp`` of them on this rank:

    h   = rmsnorm(x)                         (this rank's rows, written into the gather chunk)
    qkv = AllGather(h) Wqkv_r^T              (all-gather -> GEMM)        rope(q, k)
    o   = attention(q, k, v)                 (this rank's heads, full sequences)
    x2  = x + ReduceScatter(o Wo_r^T)        (GEMM -> reduce-scatter, residual fused)
    h2  = rmsnorm(x2);  gu = AllGather(h2) W13_r^T;  a = silu(gate) * up
    x'  = x2 + ReduceScatter(a W2_r^T)

The backward mirrors it: the gradient of a reduce-scatter is an all-gather feeding the dgrad GEMM
of ``wo`` / ``w2`` (whose gathered input also feeds the weight gradient), the gradient of an
all-gather is a reduce-scatter after the dgrad GEMM of ``wqkv`` / ``w13``, and the normalised
inputs of the column-parallel weight gradients are recomputed and re-gathered.

With the GPT MLP (``cfg.mlp == "gelu"``) the input projection is ``w1`` alone and
``a = gelu(AllGather(h2) W1_r^T)``.  With an ``Fp8Recipe`` (``fp8=``) the four projections run as
block-scaled fp8 GEMMs (``models.fp8_linear``): for the column-parallel ones each rank's RMSNorm
writes its rows as fp8 and the gather moves fp8 rows with their scales (half the bytes of bf16), the
row-parallel ones store their partial products straight
into the owners' receive slots from the fp8 GEMM's epilogue (``tp.gemm_rs_with``), and every
rank records the amax of its operands for the per-layer history.

Parameters live in two flat sets: ``shd`` (tensor-parallel shards: wq, wk, wv, wo, w1, w3, w2)
and ``rep`` (replicated on every TP rank: the norms, the embedding on the first stage, the final
norm and LM head on the last).  With sequence parallelism every TP rank computes the replicated
parameters' gradients from its own token rows, so ``rep`` is reduced over TP x DP and ``shd``
over DP only.  Initialisation is layout invariant (each logical tensor is drawn from its own
``(seed, name)`` stream and sliced), so every TP/PP/DP layout starts from the same model.

Activations of every in-flight micro-batch live in a slot (allocated on first use, reused after
the micro-batch's backward), so pipeline schedules with several micro-batches in flight do not
allocate in steady state.  (Reference: the TP/SP stage of the CPU model,
``resihp/runtime/reference_model.py:134-260``; the GPU model of the reference is Megatron-Core,
``resihp/runtime/megatron_runtime.py:162``.)
"""

from __future__ import annotations

import torch

from .. import ops
from ..ops import fp8 as fp8_ops
from ..utils.intervals import even_split
from .config import GPTConfig
from .gpt import mlp_act_bwd, mlp_act_fwd
from .params import FlatParams, ParamSpec

SHARDED = ("wq", "wk", "wv", "wo", "w1", "w3", "w2")


def stage_param_specs(cfg: GPTConfig, layers, first: bool, last: bool, tp_rank: int,
                      tp_size: int) -> tuple[list[ParamSpec], list[ParamSpec]]:
    """``(replicated, sharded)`` parameter specs of a stage on TP rank ``tp_rank``."""
    H, D, F = cfg.hidden, cfg.head_dim, cfg.ffn
    if cfg.heads % tp_size or cfg.kv_heads % tp_size or F % tp_size:
        raise ValueError(f"tp={tp_size} must divide heads ({cfg.heads}), kv heads ({cfg.kv_heads}) and ffn ({F})")
    qh = even_split(cfg.heads, tp_size)[tp_rank]
    kh = even_split(cfg.kv_heads, tp_size)[tp_rank]
    fr = even_split(F, tp_size)[tp_rank]
    nq, nk, nf = qh[1] - qh[0], kh[1] - kh[0], fr[1] - fr[0]
    rep: list[ParamSpec] = []
    shd: list[ParamSpec] = []
    if first:
        rep.append(ParamSpec("embed", (cfg.vocab_size, H)))
    for l in layers:
        p = f"layers.{l}."
        rep.append(ParamSpec(p + "attn_norm", (H,), init="ones"))
        rep.append(ParamSpec(p + "mlp_norm", (H,), init="ones"))
        shd += [
            ParamSpec(p + "wq", (nq * D, H), (cfg.heads * D, H), 0, (qh[0] * D, qh[1] * D)),
            ParamSpec(p + "wk", (nk * D, H), (cfg.kv_heads * D, H), 0, (kh[0] * D, kh[1] * D)),
            ParamSpec(p + "wv", (nk * D, H), (cfg.kv_heads * D, H), 0, (kh[0] * D, kh[1] * D)),
            ParamSpec(p + "wo", (H, nq * D), (H, cfg.heads * D), 1, (qh[0] * D, qh[1] * D)),
            ParamSpec(p + "w1", (nf, H), (F, H), 0, fr),
        ] + ([ParamSpec(p + "w3", (nf, H), (F, H), 0, fr)] if cfg.gated else []) + [
            ParamSpec(p + "w2", (H, nf), (H, F), 1, fr),
        ]
    if last:
        rep.append(ParamSpec("final_norm", (H,), init="ones"))
        rep.append(ParamSpec("lm_head", (cfg.vocab_size, H)))
    return rep, shd


class _Slot:
    """Saved activations of one in-flight micro-batch."""

    def __init__(self, stage: "TPStage"):
        c, dev = stage.cfg, stage.device
        T, Tl, H, L = stage.T, stage.Tl, c.hidden, len(stage.layer_ids)
        bf = dict(dtype=torch.bfloat16, device=dev)
        f32 = dict(dtype=torch.float32, device=dev)
        self.x = [torch.empty(Tl, H, **bf) for _ in range(L + 1)]
        self.x2 = [torch.empty(Tl, H, **bf) for _ in range(L)]
        self.rstd1 = [torch.empty(Tl, **f32) for _ in range(L)]
        self.rstd2 = [torch.empty(Tl, **f32) for _ in range(L)]
        self.qkv = [torch.empty(T, stage.qkv_cols, **bf) for _ in range(L)]
        self.o = [torch.empty(T, stage.nq * c.head_dim, **bf) for _ in range(L)]
        self.lse = [torch.empty(stage.mb, stage.nq, stage.S, **f32) for _ in range(L)]
        self.gu = [torch.empty(T, stage.mlp_in, **bf) for _ in range(L)]
        # bf16 stages keep what the weight gradients read instead of recomputing it in the backward:
        # the gathered normalised inputs of the QKV and MLP-input projections and the MLP activation
        keep = stage.keep_inputs
        self.h1 = [torch.empty(T, H, **bf) for _ in range(L)] if keep else None
        self.h2 = [torch.empty(T, H, **bf) for _ in range(L)] if keep else None
        self.act = [torch.empty(T, stage.nf, **bf) for _ in range(L)] if keep else None
        self.ids: torch.Tensor | None = None
        if stage.last:
            self.hf = torch.empty(Tl, H, **bf)
            self.rstd_f = torch.empty(Tl, **f32)
            self.logits = torch.empty(Tl, c.vocab_size, **bf)


class TPStage:
    def __init__(self, cfg: GPTConfig, device, *, layers, first: bool, last: bool, tp, micro_batch: int = 1,
                 seq_len: int | None = None, seed: int = 0, rep_shard: tuple[int, int] = (0, 1),
                 shd_shard: tuple[int, int] = (0, 1), rep_factories=(None, None), shd_factories=(None, None),
                 init: bool = True, fp8=None, sp: bool = True, recompute: bool = False):
        """``tp``: the tensor-parallel backend (``parallel.tp_backend``); ``*_shard`` the
        (rank, count) of the ZeRO-1 optimizer shard of each parameter set over its
        data-parallel group; ``*_factories`` the (buffer, optimizer) factories of ``FlatParams``
        (the fused data-parallel step's peer heap); ``init`` draws the initial weights;
        ``fp8`` an ``Fp8Recipe`` for block-scaled fp8 projections; ``sp=False``: plain tensor
        parallelism (every TP rank holds every token row; the backend all-reduces instead of
        reduce-scattering).  ``recompute=True`` (bf16 only) re-derives the weight gradients'
        inputs in the backward (RMSNorm + all-gather of the QKV / MLP inputs, the MLP activation)
        instead of keeping them per in-flight micro-batch: less memory, two more all-gathers per
        layer."""
        self.cfg, self.device = cfg, torch.device(device)
        self.tp = tp
        self.tp_rank, self.tp_size = tp.rank, tp.world
        self.layer_ids = list(layers)
        self.first, self.last = first, last
        self.mb = micro_batch
        self.S = seq_len or cfg.seq_len
        self.T = self.mb * self.S
        if self.T % self.tp_size:
            raise ValueError(f"{self.T} tokens per micro-batch do not split over tp={self.tp_size}")
        self.sp = sp
        if getattr(tp, "sp", True) != sp:
            raise ValueError("the stage and its TP backend disagree on sequence parallelism")
        self.Tl = self.T // self.tp_size if sp else self.T
        self.nq, self.nk = cfg.heads // self.tp_size, cfg.kv_heads // self.tp_size
        self.nf = cfg.ffn // self.tp_size
        self.mlp_in = (2 if cfg.gated else 1) * self.nf
        self.qkv_cols = (self.nq + 2 * self.nk) * cfg.head_dim
        rep_specs, shd_specs = stage_param_specs(cfg, self.layer_ids, first, last, self.tp_rank, self.tp_size)
        self.rep = FlatParams(rep_specs, self.device, shard_rank=rep_shard[0], shard_count=rep_shard[1],
                              buffer_factory=rep_factories[0], opt_factory=rep_factories[1])
        self.shd = FlatParams(shd_specs, self.device, shard_rank=shd_shard[0], shard_count=shd_shard[1],
                              buffer_factory=shd_factories[0], opt_factory=shd_factories[1])
        if init:  # else a migrated state is loaded next
            self.rep.initialize(seed, cfg.init_std)
            self.shd.initialize(seed, cfg.init_std)
        self.cos, self.sin = ops.rope_tables(self.S, cfg.head_dim, cfg.rope_theta, self.device)
        for l in self.layer_ids:  # fused projection weights are views over consecutive tensors
            self._check_adjacent(f"layers.{l}.", ("wq", "wk", "wv"))
            if cfg.gated:
                self._check_adjacent(f"layers.{l}.", ("w1", "w3"))
        bf = dict(dtype=torch.bfloat16, device=self.device)
        T, Tl, H = self.T, self.Tl, cfg.hidden
        self.ws_a = torch.empty(T, self.nf, **bf)
        self.ws_da = torch.empty(T, self.nf, **bf)
        self.ws_do = torch.empty(T, self.nq * cfg.head_dim, **bf)
        self.ws_dqkv = torch.empty(T, self.qkv_cols, **bf)
        self.ws_dh = torch.empty(Tl, H, **bf)
        self.ws_dx = torch.empty(Tl, H, **bf)
        self.ws_dx2 = torch.empty(Tl, H, **bf)
        self.ws_rstd = torch.empty(Tl, dtype=torch.float32, device=self.device)
        self.loss_acc = torch.zeros((), dtype=torch.float32, device=self.device)
        self.slots: dict[object, _Slot] = {}
        self.free: list[_Slot] = []
        self.deferred: dict[object, list] = {}
        self.f8 = None
        self.keep_inputs = not recompute and fp8 is None
        if fp8 is not None:
            from .fp8_linear import Fp8Linears, check_shapes

            check_shapes(cfg, self.T, self.tp_size)
            self.f8 = Fp8Linears(self.layer_ids, self.device, fp8)

    # ------------------------------------------------------------------ parameter views
    def _check_adjacent(self, p: str, names) -> None:
        P = self.shd
        off = P.offsets[p + names[0]]
        for n in names:
            if P.offsets[p + n] != off:
                raise ValueError(f"{p + n} does not follow {p + names[0]} in the flat buffer")
            off += P.specs[p + n].numel

    def _fused(self, buf: torch.Tensor, p: str, names, rows: int) -> torch.Tensor:
        o = self.shd.offsets[p + names[0]]
        return buf[o:o + rows * self.cfg.hidden].view(rows, self.cfg.hidden)

    def wqkv(self, p: str, grad: bool = False) -> torch.Tensor:
        return self._fused(self.shd.grad if grad else self.shd.bf16, p, ("wq", "wk", "wv"), self.qkv_cols)

    def w13(self, p: str, grad: bool = False) -> torch.Tensor:
        """The MLP input projection's rows on this rank: ``[w1; w3]`` (gated) or ``w1``."""
        names = ("w1", "w3") if self.cfg.gated else ("w1",)
        return self._fused(self.shd.grad if grad else self.shd.bf16, p, names, self.mlp_in)

    def refresh_fp8_weights(self) -> None:
        """Quantise this rank's projection shards once per optimizer step."""
        ws = {}
        for l in self.layer_ids:
            p = f"layers.{l}."
            ws[(l, "qkv")], ws[(l, "o")] = self.wqkv(p), self.shd.w(p + "wo")
            ws[(l, "fc1")], ws[(l, "fc2")] = self.w13(p), self.shd.w(p + "w2")
        self.f8.refresh_weights(ws, self.shd.step)

    # ------------------------------------------------------------------ projections (bf16 or fp8)
    def _norm_col_fwd(self, l: int, lin: str, x: torch.Tensor, norm_w: torch.Tensor, rstd: torch.Tensor,
                      w: torch.Tensor, out: torch.Tensor, keep: torch.Tensor | None = None) -> None:
        """``AllGather(rmsnorm(x)) @ w^T`` for this rank's rows ``x``: bf16 -- the norm writes the
        gather buffer's chunk and the fused all-gather -> GEMM runs; fp8 -- the norm writes this
        rank's rows as fp8 (row-major 1 x 128 scales) straight into the gather buffer, the gather
        moves fp8 rows and their scales, the fp8 GEMM reads them."""
        T, H = self.T, self.cfg.hidden
        if self.f8 is None:
            self._rms(x, norm_w, self.tp.chunk(T, H), rstd)
            _, gathered = self.tp.ag_gemm(T, w, out=out)
            if keep is not None:
                keep.copy_(gathered)
            return
        fmt = self.f8.recipe.fwd_fmt
        dt = fp8_ops.DTYPES[fmt]
        q, sc = self.tp.fp8_local(T, H)
        local = fp8_ops.Fp8Tensor(self.Tl, H, fmt, False, q.view(dt), sc, None, None, True)
        self.f8.norm_quant_x(l, lin, x, norm_w, float(self.cfg.norm_eps), rstd, out=local)
        qf, sf = self.tp.all_gather_fp8(T, H)
        xq = fp8_ops.Fp8Operand(qf.view(dt), sf, 1, H // fp8_ops.BLOCK, 0, fmt)
        fp8_ops.gemm(xq, self.f8.weight(l, lin).rowwise(), out=out)

    def _row_fwd(self, l: int, lin: str, x: torch.Tensor | None, w: torch.Tensor, out: torch.Tensor,
                 residual: torch.Tensor, xq=None) -> None:
        """Row-parallel projection, reduce-scattered to the row shards, plus the residual (fp8:
        ``xq`` is the already quantised input when given)."""
        if self.f8 is None:
            self.tp.gemm_rs(x, w, out=out, residual=residual)
            return
        if xq is None:
            xq = self.f8.quant_x(l, lin, x)
        wq = self.f8.weight(l, lin)
        self.tp.gemm_rs_with(xq.R, w.shape[0], lambda **kw: fp8_ops.gemm(xq.rowwise(), wq.rowwise(), **kw),
                             out=out, residual=residual)

    def _row_bwd(self, w_list, l: int, lin: str, w: torch.Tensor, x: torch.Tensor | None, dx_out: torch.Tensor,
                 grad: torch.Tensor, xq_cols=None) -> None:
        """Backward of a row-parallel projection: the output gradient rows (written into this
        rank's chunk by the caller) are gathered; dgrad into ``dx_out`` and wgrad (``x`` is the
        saved / recomputed full-width input; fp8 without deferral: ``xq_cols()`` may give it
        already quantised along tokens) into ``grad``."""
        T, H = self.T, self.cfg.hidden
        if self.f8 is None:
            _, dy = self.tp.ag_gemm(T, w, out=dx_out, w_t=True)
            self._wgrad(w_list, dy, x, grad, copy_a=True, copy_b=x is self.ws_a)
            return
        dy = self.tp.all_gather(T, H)
        dyq = self.f8.quant_dy(l, lin, dy)
        fp8_ops.gemm(dyq.rowwise(), self.f8.weight(l, lin).colwise(), out=dx_out)
        if xq_cols is not None and w_list is None:
            fp8_ops.gemm(dyq.colwise(), xq_cols().colwise(), out=grad, accumulate=True)
            return
        self._wgrad_f8(w_list, dyq, dy, x, grad, copy_x=x is self.ws_a)

    def _col_bwd(self, w_list, l: int, lin: str, dy: torch.Tensor, w: torch.Tensor, dx_out: torch.Tensor,
                 grad: torch.Tensor, x_full_fn) -> None:
        """Backward of a column-parallel projection: dgrad reduce-scattered into ``dx_out`` (this
        rank's rows); ``x_full_fn()`` recomputes and gathers the input for the wgrad."""
        if self.f8 is None:
            # the dgrad's reduce-scatter runs while the weight-gradient GEMM computes
            finish = self.tp.gemm_rs_async(dy, w, out=dx_out, w_t=True)
            # a kept input lives in the micro-batch's slot until its W pass; a re-gathered one does not
            self._wgrad(w_list, dy, x_full_fn(), grad, copy_a=dy is self.ws_dqkv, copy_b=not self.keep_inputs)
            finish()
            return
        dyq = self.f8.quant_dy(l, lin, dy)
        wq = self.f8.weight(l, lin)
        self.tp.gemm_rs_with(dy.shape[0], self.cfg.hidden,
                             lambda **kw: fp8_ops.gemm(dyq.rowwise(), wq.colwise(), **kw), out=dx_out)
        self._wgrad_f8(w_list, dyq, dy, x_full_fn(), grad, copy_x=True)

    def _wgrad_f8(self, deferred, dyq, dy: torch.Tensor, x: torch.Tensor, out: torch.Tensor, *,
                  copy_x: bool) -> None:
        """fp8 weight gradient ``out += dy^T x``: now (with ``dy``'s transposed layout already
        quantised), or -- deferred -- from bf16 copies, re-quantised in the W pass."""
        if deferred is None:
            fp8_ops.gemm(dyq.colwise(), self.f8.quant_x_cols(x).colwise(), out=out, accumulate=True)
            return
        deferred.append(("f8", dy.clone(), x.clone() if copy_x else x, out))

    def param_sets(self) -> tuple[FlatParams, FlatParams]:
        return self.rep, self.shd

    # ------------------------------------------------------------------ slots
    def _take(self, key) -> _Slot:
        s = self.free.pop() if self.free else _Slot(self)
        self.slots[key] = s
        return s

    def _release(self, key) -> None:
        self.free.append(self.slots.pop(key))

    def inflight(self) -> int:
        return len(self.slots)

    # ------------------------------------------------------------------ forward
    def _rms(self, x, w, out, rstd):
        return ops.rmsnorm_fwd(x, w, float(self.cfg.norm_eps), out=out, rstd=rstd)[0]

    def _qkv_views(self, qkv: torch.Tensor):
        D = self.cfg.head_dim
        return (qkv[:, : self.nq * D], qkv[:, self.nq * D:(self.nq + self.nk) * D],
                qkv[:, (self.nq + self.nk) * D:])

    def forward(self, key, ids_local: torch.Tensor | None = None, x_in: torch.Tensor | None = None,
                labels_local: torch.Tensor | None = None, grad_scale: float = 1.0) -> torch.Tensor | None:
        """Forward of micro-batch ``key``: token ids of this rank's rows (first stage) or the
        received ``[T / tp, H]`` activation; returns the stage output rows (kept until the
        micro-batch's backward) or, on the last stage, None after adding the summed token loss
        into ``loss_acc`` and leaving the logits' gradient in place."""
        cfg, R, P = self.cfg, self.rep, self.shd
        T, H, D = self.T, cfg.hidden, cfg.head_dim
        slot = self._take(key)
        if self.first:
            slot.ids = ids_local
            ops.embedding_fwd(ids_local, R.w("embed"), out=slot.x[0])
        else:
            slot.x[0] = x_in
        if self.f8 is not None:
            self.refresh_fp8_weights()
        for i, l in enumerate(self.layer_ids):
            p = f"layers.{l}."
            x = slot.x[i]
            self._norm_col_fwd(l, "qkv", x, R.w(p + "attn_norm"), slot.rstd1[i], self.wqkv(p), slot.qkv[i],
                               keep=slot.h1[i] if slot.h1 is not None else None)
            q, k, v = self._qkv_views(slot.qkv[i])
            ops.rope_(q, self.nq, D, self.cos, self.sin, self.S)
            ops.rope_(k, self.nk, D, self.cos, self.sin, self.S)
            ops.attention_fwd(q, k, v, batch=self.mb, seq=self.S, heads=self.nq, kv_heads=self.nk, head_dim=D,
                              out=slot.o[i], lse=slot.lse[i])
            self._row_fwd(l, "o", slot.o[i], P.w(p + "wo"), slot.x2[i], x)
            self._norm_col_fwd(l, "fc1", slot.x2[i], R.w(p + "mlp_norm"), slot.rstd2[i], self.w13(p), slot.gu[i],
                               keep=slot.h2[i] if slot.h2 is not None else None)
            if self.f8 is not None:  # the activation is written as the fp8 operand directly
                aq = self.f8.act_quant_x(l, "fc2", slot.gu[i], cfg.gated)
                self._row_fwd(l, "fc2", None, P.w(p + "w2"), slot.x[i + 1], slot.x2[i], xq=aq)
            else:
                a = slot.act[i] if slot.act is not None else self.ws_a
                mlp_act_fwd(cfg, slot.gu[i], a)
                self._row_fwd(l, "fc2", a, P.w(p + "w2"), slot.x[i + 1], slot.x2[i])
        if not self.last:
            return slot.x[-1]
        self._rms(slot.x[-1], R.w("final_norm"), slot.hf, slot.rstd_f)
        ops.gemm(slot.hf, R.w("lm_head"), out=slot.logits)
        loss = ops.cross_entropy_(slot.logits, labels_local, grad_scale=grad_scale)
        self.loss_acc += loss.sum()
        return None

    # ------------------------------------------------------------------ backward
    def _wgrad(self, deferred, a, b, out, *, copy_a: bool = False, copy_b: bool = False) -> None:
        """``out += a^T b`` (fp32 accumulate): now, or -- for a zero-bubble schedule -- in the
        micro-batch's W pass; operands that live in reused buffers (gathered inputs, workspaces)
        are copied when deferred."""
        if deferred is None:
            ops.gemm(a, b, a_t=True, b_t=True, out=out, accumulate=True)
            return
        deferred.append((a.clone() if copy_a else a, b.clone() if copy_b else b, out))

    def backward(self, key, dx_top: torch.Tensor | None = None, defer_w: bool = False) -> torch.Tensor | None:
        """Backward of micro-batch ``key`` (after its forward); accumulates both parameter
        sets' gradients and returns the gradient of the stage input rows (None on the first
        stage).  ``defer_w`` (zero-bubble B/W split): only the input-gradient chain runs now;
        the weight-gradient GEMMs wait for ``weight_backward(key)``."""
        cfg, R, P = self.cfg, self.rep, self.shd
        T, H, D = self.T, cfg.hidden, cfg.head_dim
        slot = self.slots[key]
        dx = self.ws_dx
        w = [] if defer_w else None
        if self.last:
            ops.gemm(slot.logits, R.w("lm_head"), b_t=True, out=self.ws_dh)
            self._wgrad(w, slot.logits, slot.hf, R.g("lm_head"))
            ops.rmsnorm_bwd(slot.x[-1], R.w("final_norm"), slot.rstd_f, self.ws_dh, R.g("final_norm"), out=dx)
        else:
            dx.copy_(dx_top)
        for i in reversed(range(len(self.layer_ids))):
            l = self.layer_ids[i]
            p = f"layers.{l}."
            # MLP: the reduce-scatter's gradient is an all-gather feeding w2's dgrad and wgrad
            self.tp.chunk(T, H).copy_(dx)
            if self.f8 is not None and w is None:
                # wgrad input: the activation recomputed and quantised in one pass (gu still holds
                # the pre-activation: its gradient overwrites it only below)
                self._row_bwd(w, l, "fc2", P.w(p + "w2"), None, self.ws_da, P.g(p + "w2"),
                              xq_cols=lambda i=i: self.f8.act_quant_cols(slot.gu[i], cfg.gated))
            elif slot.act is not None:  # the activation kept from the forward
                self._row_bwd(w, l, "fc2", P.w(p + "w2"), slot.act[i], self.ws_da, P.g(p + "w2"))
            else:
                mlp_act_fwd(cfg, slot.gu[i], self.ws_a)
                self._row_bwd(w, l, "fc2", P.w(p + "w2"), self.ws_a, self.ws_da, P.g(p + "w2"))
            dgu = mlp_act_bwd(cfg, slot.gu[i], self.ws_da, slot.gu[i])

            def h2_full(i=i, p=p):
                if slot.h2 is not None:
                    return slot.h2[i]
                self._rms(slot.x2[i], R.w(p + "mlp_norm"), self.tp.chunk(T, H), self.ws_rstd)
                return self.tp.all_gather(T, H)

            self._col_bwd(w, l, "fc1", dgu, self.w13(p), self.ws_dh, self.w13(p, grad=True), h2_full)
            ops.rmsnorm_bwd(slot.x2[i], R.w(p + "mlp_norm"), slot.rstd2[i], self.ws_dh, R.g(p + "mlp_norm"), dres=dx,
                            out=self.ws_dx2)
            dx2 = self.ws_dx2
            # attention
            self.tp.chunk(T, H).copy_(dx2)
            self._row_bwd(w, l, "o", P.w(p + "wo"), slot.o[i], self.ws_do, P.g(p + "wo"))
            q, k, v = self._qkv_views(slot.qkv[i])
            dq, dk, dv = self._qkv_views(self.ws_dqkv)
            ops.attention_bwd(q, k, v, slot.o[i], self.ws_do, slot.lse[i], dq, dk, dv, batch=self.mb, seq=self.S,
                              heads=self.nq, kv_heads=self.nk, head_dim=D)
            ops.rope_(dq, self.nq, D, self.cos, self.sin, self.S, inverse=True)
            ops.rope_(dk, self.nk, D, self.cos, self.sin, self.S, inverse=True)

            def h_full(i=i, p=p):
                if slot.h1 is not None:
                    return slot.h1[i]
                self._rms(slot.x[i], R.w(p + "attn_norm"), self.tp.chunk(T, H), self.ws_rstd)
                return self.tp.all_gather(T, H)

            self._col_bwd(w, l, "qkv", self.ws_dqkv, self.wqkv(p), self.ws_dh, self.wqkv(p, grad=True), h_full)
            ops.rmsnorm_bwd(slot.x[i], R.w(p + "attn_norm"), slot.rstd1[i], self.ws_dh, R.g(p + "attn_norm"),
                            dres=dx2, out=dx)
        if self.first:
            ops.embedding_bwd(slot.ids, dx, R.g("embed"))
        if w is None:
            self._release(key)
        else:
            self.deferred[key] = w
        return None if self.first else dx

    def weight_backward(self, key) -> None:
        """The deferred weight-gradient GEMMs of micro-batch ``key`` (zero-bubble W pass)."""
        for item in self.deferred.pop(key):
            if item[0] == "f8":
                _, dy, x, out = item
                dyq = fp8_ops.quantize(dy, self.f8.recipe.bwd_fmt, rowwise=False, colwise=True)
                fp8_ops.gemm(dyq.colwise(), self.f8.quant_x_cols(x).colwise(), out=out, accumulate=True)
            else:
                a, b, out = item
                ops.gemm(a, b, a_t=True, b_t=True, out=out, accumulate=True)
        self._release(key)
