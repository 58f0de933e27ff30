"""Block-scaled fp8 linear layers of the decoder, with per-layer amax history.

Every linear layer (``qkv``, ``o``, ``fc1``, ``fc2``) runs its three GEMMs in fp8 on the tcgen05
tensor cores (``ops.fp8``):

* forward: the input ``x`` quantised E4M3 with 1 x 128 row scales, the weight E4M3 with
  128 x 128 tile scales (quantised once per optimizer step, both layouts);
* dgrad: the output gradient ``dy`` quantised E5M2 (1 x 128, both layouts) against the weight's
  transposed layout;
* wgrad: ``dy``'s transposed layout against ``x`` re-quantised along the token dimension
  (1 x 128 blocks of tokens), accumulated into the fp32 gradient.

Block scales are computed from the data they scale (current scaling); the quantiser also folds
each operand's magnitude into a per-layer ``pending`` amax slot (``x``, ``w`` and ``dy`` of every
linear: 12 slots).  At the end of an iteration the pending amaxes are reduced with MAX over every
rank (one all-reduce for all layers) and pushed into a per-layer history of ``history`` steps --
the delayed-scaling state of the reference (``resihp/runtime/reference_model.py:204-227``,
reduced in ``resihp/runtime/hetero_runtime.py:122-134``), which migrates with its layer
(``layers.<l>.amax_history``, ``[12, history]``) and rolls back with an aborted iteration.  A
non-finite reduced amax marks the iteration's gradients as unusable (``has_nonfinite``); with
``Fp8Recipe.skip_nonfinite`` the trainers then drop the iteration instead of applying it.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from ..ops import fp8

LINEARS = ("qkv", "o", "fc1", "fc2")
ROLES = ("x", "w", "dy")
SLOTS = {(lin, role): i for i, (lin, role) in enumerate((l, r) for l in LINEARS for r in ROLES)}
NSLOTS = len(SLOTS)


@dataclass(frozen=True)
class Fp8Recipe:
    fwd: str = "e4m3"  # forward operands (activations, weights)
    bwd: str = "e5m2"  # output gradients
    history: int = 16  # amax history length per recorded tensor
    skip_nonfinite: bool = False  # drop an iteration whose reduced amax is inf / NaN (one host read per step)

    @property
    def fwd_fmt(self) -> int:
        return fp8.fmt_of(self.fwd)

    @property
    def bwd_fmt(self) -> int:
        return fp8.fmt_of(self.bwd)


def history_key(layer: int) -> str:
    return f"layers.{layer}.amax_history"


def check_shapes(cfg, tokens: int, tp: int = 1) -> None:
    """Every fp8 GEMM dimension must be a multiple of the 128-wide blocks: the tokens of a
    micro-batch, the hidden size and each rank's share of the heads and of the FFN."""
    D = cfg.head_dim
    dims = {"tokens per micro-batch": tokens, "hidden": cfg.hidden,
            "query heads x head dim per rank": cfg.heads * D // tp,
            "q / k / v rows per rank": (cfg.heads + 2 * cfg.kv_heads) * D // tp, "ffn per rank": cfg.ffn // tp}
    bad = {k: v for k, v in dims.items() if v % 128}
    if bad:
        raise ValueError(f"fp8 needs multiples of 128: {bad}")


class Fp8Linears:
    """fp8 state of a contiguous set of decoder layers on one rank."""

    def __init__(self, layer_ids, device, recipe: Fp8Recipe):
        self.recipe = recipe
        self.device = torch.device(device)
        self.layer_ids = list(layer_ids)
        self.index = {l: i for i, l in enumerate(self.layer_ids)}
        n = len(self.layer_ids)
        self.pending = torch.zeros(n, NSLOTS, dtype=torch.float32, device=self.device)
        self.history = torch.zeros(n, NSLOTS, recipe.history, dtype=torch.float32, device=self.device)
        self.weights: dict[tuple[int, str], fp8.Fp8Tensor] = {}
        self._ws: dict[tuple, fp8.Fp8Tensor] = {}
        self.version = None

    # ------------------------------------------------------------------ amax bookkeeping
    def amax(self, layer: int, lin: str, role: str) -> torch.Tensor:
        i = self.index[layer]
        j = SLOTS[(lin, role)]
        return self.pending[i, j:j + 1]

    def finish_iteration(self, reduce_max=None) -> None:
        """``reduce_max(t)``: in-place MAX all-reduce over every rank (None: one rank), given the
        int32 view of the pending amaxes -- their bit patterns order like the magnitudes and a
        NaN stays the largest, which a floating-point MAX would not guarantee."""
        if reduce_max is not None:
            reduce_max(self.pending.view(torch.int32))
        fp8.amax_history_push(self.history, self.pending)

    def has_nonfinite(self) -> bool:
        """Whether the latest pushed amaxes contain inf / NaN (reads one value to the host)."""
        return not bool(torch.isfinite(self.history[..., 0]).all())

    def state(self) -> dict[str, torch.Tensor]:
        """Per-layer histories under their logical keys (views)."""
        return {history_key(l): self.history[i] for l, i in self.index.items()}

    def load_state(self, state: dict[str, torch.Tensor]) -> None:
        for l, i in self.index.items():
            key = history_key(l)
            if key in state:
                self.history[i].copy_(state[key])

    # ------------------------------------------------------------------ operands
    def _buf(self, R: int, C: int, fmt: int, two_d: bool, rowwise: bool, colwise: bool,
             tag: str = "") -> fp8.Fp8Tensor:
        key = (R, C, fmt, two_d, rowwise, colwise, tag)
        t = self._ws.get(key)
        if t is None:
            t = self._ws[key] = fp8.Fp8Tensor.empty(R, C, fmt, two_d=two_d, rowwise=rowwise, colwise=colwise,
                                                    device=self.device)
        return t

    def refresh_weights(self, weights: dict[tuple[int, str], torch.Tensor], version) -> None:
        """Quantise every weight (both layouts, 128 x 128 tiles) once per ``version`` (the
        optimizer step count); records the weights' amax."""
        if version == self.version:
            return
        for (layer, lin), w in weights.items():
            out = self.weights.get((layer, lin))
            if out is None:
                out = self.weights[(layer, lin)] = fp8.Fp8Tensor.empty(
                    w.shape[0], w.shape[1], self.recipe.fwd_fmt, two_d=True, rowwise=True, colwise=True,
                    device=self.device)
            fp8.quantize(w, self.recipe.fwd_fmt, two_d=True, rowwise=True, colwise=True,
                         amax=self.amax(layer, lin, "w"), out=out)
        self.version = version

    def weight(self, layer: int, lin: str) -> fp8.Fp8Tensor:
        return self.weights[(layer, lin)]

    def quant_x(self, layer: int, lin: str, x: torch.Tensor) -> fp8.Fp8Tensor:
        """Forward input, rowwise (its amax recorded)."""
        R, C = x.shape
        out = self._buf(R, C, self.recipe.fwd_fmt, False, True, False, "x")
        return fp8.quantize(x, self.recipe.fwd_fmt, rowwise=True, amax=self.amax(layer, lin, "x"), out=out)

    def norm_quant_x(self, layer: int, lin: str, x: torch.Tensor, norm_w: torch.Tensor, eps: float,
                     rstd: torch.Tensor, out: fp8.Fp8Tensor | None = None) -> fp8.Fp8Tensor:
        """Forward input that is an RMSNorm output: normalised and quantised in one kernel
        (``rstd`` saved for the backward; amax recorded)."""
        R, C = x.shape
        if out is None:
            out = self._buf(R, C, self.recipe.fwd_fmt, False, True, False, "x")
        return fp8.rmsnorm_quantize(x, norm_w, eps, self.recipe.fwd_fmt, out=out, rstd=rstd,
                                    amax=self.amax(layer, lin, "x"))

    def act_quant_x(self, layer: int, lin: str, gu: torch.Tensor, gated: bool) -> fp8.Fp8Tensor:
        """Forward input that is the MLP activation of ``gu``: activation and quantisation in one
        kernel (amax recorded)."""
        T = gu.shape[0]
        F = gu.shape[1] // (2 if gated else 1)
        out = self._buf(T, F, self.recipe.fwd_fmt, False, True, False, "x")
        return fp8.act_quantize(gu, gated, self.recipe.fwd_fmt, out=out, amax=self.amax(layer, lin, "x"))

    def act_quant_cols(self, gu: torch.Tensor, gated: bool) -> fp8.Fp8Tensor:
        """Weight-gradient input that is the MLP activation of ``gu``: recomputed and quantised
        along tokens in one kernel (the bf16 activation is never written)."""
        T = gu.shape[0]
        F = gu.shape[1] // (2 if gated else 1)
        out = self._buf(T, F, self.recipe.fwd_fmt, False, False, True, "xc")
        return fp8.quantize(gu, self.recipe.fwd_fmt, rowwise=False, colwise=True, out=out,
                            act="swiglu" if gated else "gelu")

    def quant_x_cols(self, x: torch.Tensor) -> fp8.Fp8Tensor:
        """Weight-gradient input: blocks along the token dimension (transposed layout)."""
        R, C = x.shape
        out = self._buf(R, C, self.recipe.fwd_fmt, False, False, True, "xc")
        return fp8.quantize(x, self.recipe.fwd_fmt, rowwise=False, colwise=True, out=out)

    def quant_dy(self, layer: int, lin: str, dy: torch.Tensor) -> fp8.Fp8Tensor:
        """Output gradient, both layouts (its amax recorded)."""
        R, C = dy.shape
        out = self._buf(R, C, self.recipe.bwd_fmt, False, True, True, "dy")
        return fp8.quantize(dy, self.recipe.bwd_fmt, rowwise=True, colwise=True, amax=self.amax(layer, lin, "dy"),
                            out=out)

    # ------------------------------------------------------------------ GEMMs
    def forward(self, layer: int, lin: str, x: torch.Tensor, out: torch.Tensor,
                residual: torch.Tensor | None = None) -> torch.Tensor:
        xq = self.quant_x(layer, lin, x)
        return fp8.gemm(xq.rowwise(), self.weight(layer, lin).rowwise(), out=out, residual=residual)

    def backward(self, layer: int, lin: str, dy: torch.Tensor, x: torch.Tensor, dx_out: torch.Tensor,
                 grad: torch.Tensor) -> torch.Tensor:
        """dgrad into ``dx_out`` (bf16) and wgrad accumulated into ``grad`` (fp32)."""
        dyq = self.quant_dy(layer, lin, dy)
        fp8.gemm(dyq.rowwise(), self.weight(layer, lin).colwise(), out=dx_out)
        fp8.gemm(dyq.colwise(), self.quant_x_cols(x).colwise(), out=grad, accumulate=True)
        return dx_out
