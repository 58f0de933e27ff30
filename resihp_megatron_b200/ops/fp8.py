"""Block-scaled fp8 (E4M3 forward / E5M2 backward) on tcgen05 tensor cores (``csrc/fp8_sm100.cu``).

``quantize(x)`` turns a bf16 ``[R, C]`` tensor into fp8 with power-of-two block scales:

* 1 x 128 blocks (activations and gradients): one scale per row segment of 128 columns
  (``rowwise``) and/or per column segment of 128 rows (``colwise``, stored transposed as
  ``[C, R]`` so it is K-major for the GEMMs that contract over R);
* 128 x 128 blocks (``two_d``, weights): one scale per tile, shared by both layouts.

Every scale is ``2^e`` with ``e`` the smallest exponent for which the block's amax fits the
format's largest finite value, so ``x / s`` is exact and the only rounding is the cast to fp8
(nearest even).  ``quantize_reference`` is the same computation in PyTorch: it reproduces the
kernel's bytes and scales bit for bit (for finite inputs), which is what the GPU tests check and
what the CPU tests run on.

``gemm(a, b)`` takes two ``Fp8Operand`` (K-major ``[rows, K]`` data plus scale addressing) and
computes ``alpha * sum_kb sa * sb * (a_kb . b_kb)`` -- the three GEMMs of a linear layer are

* forward ``y = x W^T``:   ``gemm(xq.rowwise(), wq.rowwise())``
* dgrad   ``dx = dy W``:   ``gemm(dyq.rowwise(), wq.colwise())``
* wgrad   ``dW = dy^T x``: ``gemm(dyq.colwise(), xq.colwise(), out=grad, accumulate=True)``

The reference framework's fp8 is Transformer Engine inside Megatron-Core; its semantics oracle
emulates delayed scaling with an amax history (``resihp/runtime/reference_model.py:44-46,
204-227``) whose global amax is reduced with MAX over every rank
(``resihp/runtime/hetero_runtime.py:122-134``).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from ._build import ext
from .counter import count

E4M3, E5M2 = 0, 1
DTYPES = {E4M3: torch.float8_e4m3fn, E5M2: torch.float8_e5m2}
MAX_EXP = {E4M3: 8, E5M2: 15}  # largest finite value = 1.75 * 2^MAX_EXP
BLOCK = 128
EPI_BF16, EPI_F32, EPI_F32_ACC, EPI_BF16_RES, EPI_SCATTER = 0, 1, 2, 3, 4


def fmt_of(name: str | int) -> int:
    if isinstance(name, int):
        return name
    return {"e4m3": E4M3, "e5m2": E5M2}[name.lower()]


@dataclass
class Fp8Operand:
    """K-major fp8 matrix ``[rows, K]``; the scale of row ``r`` in K-block ``kb`` is
    ``scale[kb * kb_stride + (r >> shift) * row_stride]``."""

    data: torch.Tensor
    scale: torch.Tensor
    kb_stride: int
    row_stride: int
    shift: int
    fmt: int

    @property
    def rows(self) -> int:
        return self.data.shape[0]

    @property
    def K(self) -> int:
        return self.data.shape[1]

    def scale_matrix(self) -> torch.Tensor:
        """``[rows, K / 128]`` scales (the addressing made explicit)."""
        r = torch.arange(self.rows, device=self.scale.device)[:, None] >> self.shift
        kb = torch.arange(self.K // BLOCK, device=self.scale.device)[None, :]
        return self.scale.reshape(-1)[kb * self.kb_stride + r * self.row_stride]

    def dequantize(self) -> torch.Tensor:
        s = self.scale_matrix().repeat_interleave(BLOCK, dim=1)
        return self.data.float() * s


@dataclass
class Fp8Tensor:
    """A quantised bf16 ``[R, C]`` tensor: rowwise data ``[R, C]`` and/or colwise data ``[C, R]``.
    Scales: 1 x 128 rowwise ``s_row`` ``[C/128, R]`` (``row_major``: ``[R, C/128]``, a row's
    scales contiguous -- they travel with the row in a gather), colwise ``s_col`` ``[R/128, C]``;
    with ``two_d`` one ``s_row`` ``[C/128, R/128]`` serves both layouts."""

    R: int
    C: int
    fmt: int
    two_d: bool
    q_row: torch.Tensor | None
    s_row: torch.Tensor | None
    q_col: torch.Tensor | None
    s_col: torch.Tensor | None
    row_major: bool = False

    @classmethod
    def empty(cls, R: int, C: int, fmt: int = E4M3, *, two_d: bool = False, rowwise: bool = True,
              colwise: bool = False, device=None, row_major: bool = False) -> "Fp8Tensor":
        if C % BLOCK or (R % BLOCK and (two_d or colwise)):
            raise ValueError(f"fp8 tensors need dims multiples of {BLOCK} (rows too unless rowwise-only), "
                             f"got [{R}, {C}]")
        dt = DTYPES[fmt]
        f32 = dict(dtype=torch.float32, device=device)
        q_row = torch.empty(R, C, dtype=dt, device=device) if rowwise else None
        q_col = torch.empty(C, R, dtype=dt, device=device) if colwise else None
        if two_d:
            s_row, s_col = torch.empty(C // BLOCK, R // BLOCK, **f32), None
        else:
            s_row = (torch.empty(R, C // BLOCK, **f32) if row_major else torch.empty(C // BLOCK, R, **f32)) \
                if rowwise else None
            s_col = torch.empty(R // BLOCK, C, **f32) if colwise else None
        return cls(R, C, fmt, two_d, q_row, s_row, q_col, s_col, row_major and not two_d)

    def rowwise(self) -> Fp8Operand:
        """Operand ``[R, K = C]`` (forward input, weight for the forward, dgrad's gradient)."""
        assert self.q_row is not None, "quantised without the rowwise layout"
        if self.two_d:
            return Fp8Operand(self.q_row, self.s_row, self.R // BLOCK, 1, 7, self.fmt)
        if self.row_major:
            return Fp8Operand(self.q_row, self.s_row, 1, self.C // BLOCK, 0, self.fmt)
        return Fp8Operand(self.q_row, self.s_row, self.R, 1, 0, self.fmt)

    def colwise(self) -> Fp8Operand:
        """Operand ``[C, K = R]`` (the transpose: weight for dgrad, wgrad's two operands)."""
        assert self.q_col is not None, "quantised without the colwise layout"
        if self.two_d:
            return Fp8Operand(self.q_col, self.s_row, 1, self.R // BLOCK, 7, self.fmt)
        return Fp8Operand(self.q_col, self.s_col, self.C, 1, 0, self.fmt)


ACTS = {None: 0, "gelu": 1, "swiglu": 2}


def quantize(x: torch.Tensor, fmt: int | str = E4M3, *, two_d: bool = False, rowwise: bool = True,
             colwise: bool = False, amax: torch.Tensor | None = None, out: Fp8Tensor | None = None,
             row_major: bool = False, act: str | None = None) -> Fp8Tensor:
    """Quantise bf16 ``x [R, C]`` (C a multiple of 128; R too unless rowwise-only).  ``amax`` (fp32,
    >= 1 element) receives ``max(amax[0], max |x|)`` -- NaN and inf propagate.  ``row_major``:
    rowwise scales stored ``[R, C/128]`` (taken from ``out`` when given).  ``act``: quantise the
    MLP activation of ``x`` instead -- ``"gelu"`` (``x`` is ``[R, C]``) or ``"swiglu"`` (``x`` is
    ``[R, 2C]``: gate | up) -- computed and rounded to bf16 exactly as the activation kernels do."""
    fmt = fmt_of(fmt)
    R, C = x.shape
    if act == "swiglu":
        C //= 2
    if out is None:
        out = Fp8Tensor.empty(R, C, fmt, two_d=two_d, rowwise=rowwise, colwise=colwise, device=x.device,
                              row_major=row_major)
    ext().fp8_quantize(x, fmt, two_d, _u8(out.q_row), out.s_row, _u8(out.q_col), out.s_col, amax, out.row_major,
                       ACTS[act])
    count(1)
    return out


def rmsnorm_quantize(x: torch.Tensor, w: torch.Tensor, eps: float, fmt: int | str = E4M3, *, out: Fp8Tensor,
                     rstd: torch.Tensor | None = None, amax: torch.Tensor | None = None) -> Fp8Tensor:
    """``quantize(rmsnorm(x) * w)`` in one pass (rowwise 1 x 128 blocks into ``out``, whose scale
    layout -- K-block or row major -- is kept); ``rstd`` receives the per-row ``1 / rms``.
    Bit-identical to ``ops.rmsnorm_fwd`` followed by ``quantize``."""
    fmt = fmt_of(fmt)
    op = out.rowwise()
    ext().rmsnorm_fp8(x, w, rstd, float(eps), fmt, out.q_row.view(torch.uint8), out.s_row, op.kb_stride,
                      op.row_stride, amax)
    count(1)
    return out


def act_quantize(x: torch.Tensor, gated: bool, fmt: int | str = E4M3, *, out: Fp8Tensor,
                 amax: torch.Tensor | None = None) -> Fp8Tensor:
    """The MLP activation -- ``gelu(x)`` of ``[T, F]`` or ``silu(gate) * up`` of ``[T, 2F]``
    (``gated``) -- quantised rowwise into ``out`` (``[T, F]``) in one pass; bit-identical to
    ``ops.gelu_fwd`` / ``ops.swiglu_fwd`` followed by ``quantize``."""
    fmt = fmt_of(fmt)
    op = out.rowwise()
    ext().act_fp8(x, bool(gated), fmt, out.q_row.view(torch.uint8), out.s_row, op.kb_stride, op.row_stride, amax)
    count(1)
    return out


def amax_history_push(history: torch.Tensor, pending: torch.Tensor) -> None:
    """``history [..., len]`` (fp32): shift by one, ``pending`` (same leading shape) into slot 0,
    then zero ``pending`` -- the delayed-scaling update after the amax reduction."""
    ext().amax_history_push(history, pending)
    count(1)


def amax_history_push_reference(history: torch.Tensor, pending: torch.Tensor) -> None:
    history[..., 1:] = history[..., :-1].clone()
    history[..., 0] = pending
    pending.zero_()


def _u8(t):
    return None if t is None else t.view(torch.uint8)


class Fp8ShapeError(ValueError, RuntimeError):
    """A block-scaled GEMM was given operands the kernel cannot take (raised in Python, before
    any native call)."""


def _check_operand(op: Fp8Operand, name: str) -> None:
    d = op.data
    if d.dim() != 2 or d.element_size() != 1 or not d.is_contiguous():
        raise Fp8ShapeError(f"{name}: data must be a contiguous 2-D tensor of 1-byte elements, got "
                            f"{tuple(d.shape)} {d.dtype}")
    rows, K = d.shape
    if rows <= 0 or K <= 0 or rows % BLOCK or K % BLOCK:
        raise Fp8ShapeError(f"{name}: rows and K must be positive multiples of {BLOCK}, got [{rows}, {K}]")
    if op.shift not in (0, 7) or op.kb_stride < 0 or op.row_stride < 0:
        raise Fp8ShapeError(f"{name}: bad scale addressing (kb_stride={op.kb_stride}, "
                            f"row_stride={op.row_stride}, shift={op.shift})")
    s = op.scale
    if s.dtype != torch.float32 or not s.is_contiguous():
        raise Fp8ShapeError(f"{name}: scales must be contiguous fp32")
    last = (K // BLOCK - 1) * op.kb_stride + ((rows - 1) >> op.shift) * op.row_stride
    if last >= s.numel():
        raise Fp8ShapeError(f"{name}: {s.numel()} scales cannot cover index {last}")
    if op.fmt not in DTYPES:
        raise Fp8ShapeError(f"{name}: unknown fp8 format {op.fmt}")


def _check_operands(a: Fp8Operand, b: Fp8Operand) -> None:
    _check_operand(a, "a")
    _check_operand(b, "b")
    if a.K != b.K:
        raise Fp8ShapeError(f"contraction sizes differ: a has K={a.K}, b has K={b.K}")
    if a.data.device != b.data.device:
        raise Fp8ShapeError("a and b live on different devices")


def gemm(a: Fp8Operand, b: Fp8Operand, *, out: torch.Tensor | None = None, out_dtype: torch.dtype = torch.bfloat16,
         accumulate: bool = False, alpha: float = 1.0, residual: torch.Tensor | None = None,
         scatter: tuple[list[int], int] | None = None, variant: int = 0) -> torch.Tensor | None:
    """``out [a.rows, b.rows] (+)= alpha * block-scaled a @ b^T`` (all dims multiples of 128).
    ``residual``: bf16 ``out = product + residual``.  ``scatter = (recv_ptrs, slot)``: no local
    output; row ``m`` is stored (bf16) into rank ``m // (rows / world)``'s receive buffer
    ``[world][rows / world][N]`` at ``slot`` -- the partial products of a reduce-scatter.
    Shapes and scale addressing are validated here, before the extension is called.
    ``variant``: 2 applies the scales in the tensor core (block-scaled MMA, E8M0 scale per 32
    K-elements; exact for these power-of-two scales) on single CTAs, 0 (default) likewise except
    for products under ``SMALL_FLOPS`` (register promotion: no scale-packing launches), 3 on CTA pairs
    (``a.rows`` a multiple of 256; measured slower at 8192^3), 1 promotes per 128-deep K-block in
    registers (the earlier kernel, kept for comparison)."""
    _check_operands(a, b)
    if variant not in (0, 1, 2, 3):
        raise ValueError("variant is 0 (default), 1 (register promotion), 2 (single CTA) or 3 (CTA pair)")
    if variant == 3 and a.rows % 256:
        raise Fp8ShapeError(f"the CTA-pair kernel needs a.rows a multiple of 256, got {a.rows}")
    if scatter is not None:
        ptrs, slot = scatter
        ext().gemm_fp8(a.data.view(torch.uint8), a.fmt, a.scale, a.kb_stride, a.row_stride, a.shift,
                       b.data.view(torch.uint8), b.fmt, b.scale, b.kb_stride, b.row_stride, b.shift, None, EPI_SCATTER,
                       float(alpha), None, [int(p) for p in ptrs], int(slot), variant=variant)
        count(_launches(a, b, variant))
        return None
    if residual is not None:
        if out is None:
            out = torch.empty(a.rows, b.rows, dtype=torch.bfloat16, device=a.data.device)
        ext().gemm_fp8(a.data.view(torch.uint8), a.fmt, a.scale, a.kb_stride, a.row_stride, a.shift,
                       b.data.view(torch.uint8), b.fmt, b.scale, b.kb_stride, b.row_stride, b.shift, out, EPI_BF16_RES,
                       float(alpha), residual, variant=variant)
        count(_launches(a, b, variant))
        return out
    if accumulate:
        if out is None or out.dtype != torch.float32:
            raise ValueError("accumulate=True needs an fp32 `out`")
        epi = EPI_F32_ACC
    else:
        dt = out.dtype if out is not None else out_dtype
        epi = EPI_F32 if dt == torch.float32 else EPI_BF16
    if out is None:
        out = torch.empty(a.rows, b.rows, dtype=torch.float32 if epi != EPI_BF16 else torch.bfloat16,
                          device=a.data.device)
    ext().gemm_fp8(a.data.view(torch.uint8), a.fmt, a.scale, a.kb_stride, a.row_stride, a.shift,
                   b.data.view(torch.uint8), b.fmt, b.scale, b.kb_stride, b.row_stride, b.shift, out, epi, float(alpha),
                   variant=variant)
    count(_launches(a, b, variant))
    return out


SMALL_FLOPS = 3.0e10  # variant 0 below this product size: the register-promotion kernel


def _promotes(a: Fp8Operand, b: Fp8Operand, variant: int) -> bool:
    """Whether ``gemm`` runs the register-promotion kernel (the rule of the native dispatch)."""
    if variant == 1:
        return True
    if variant != 0 or 2.0 * a.rows * b.rows * a.K >= SMALL_FLOPS:
        return False
    return b.shift != 0 or (b.row_stride == 1 and b.kb_stride % 4 == 0 and b.scale.data_ptr() % 16 == 0)


def _launches(a: Fp8Operand, b: Fp8Operand, variant: int) -> int:
    """Kernels one ``gemm`` call launches: the block-scaled path packs A's and B's scales first."""
    return 1 if _promotes(a, b, variant) else 3


# ---------------------------------------------------------------------------- PyTorch emulation
def scale_exponent(amax: torch.Tensor, fmt: int) -> torch.Tensor:
    """Exponent ``e`` of the power-of-two scale: the smallest with ``amax * 2^-e <= 1.75 * 2^F``,
    clamped to [-126, 126]; 0 for zero, inf and NaN (integer arithmetic on the fp32 bits, as the
    kernel does)."""
    bits = amax.float().contiguous().view(torch.int32).to(torch.int64) & 0x7FFFFFFF
    E = bits >> 23
    mant = bits & 0x7FFFFF
    e = (E - 127) - MAX_EXP[fmt] + (mant > 0x600000).to(torch.int64)
    e = e.clamp(-126, 126)
    return torch.where((bits == 0) | (E == 255), torch.zeros_like(e), e)


def pow2(e: torch.Tensor) -> torch.Tensor:
    return ((e + 127).to(torch.int32) << 23).view(torch.float32)


def quantize_reference(x: torch.Tensor, fmt: int | str = E4M3, *, two_d: bool = False, rowwise: bool = True,
                       colwise: bool = False, amax: torch.Tensor | None = None, row_major: bool = False) -> Fp8Tensor:
    """``quantize`` in PyTorch (any device): same bytes and scales for finite inputs."""
    fmt = fmt_of(fmt)
    R, C = x.shape
    if C % BLOCK or (R % BLOCK and (two_d or colwise)):
        raise ValueError(f"fp8 tensors need dims multiples of {BLOCK} (rows too unless rowwise-only), got [{R}, {C}]")
    xf = x.float()
    dt = DTYPES[fmt]
    nr, nc = R // BLOCK, C // BLOCK
    out = Fp8Tensor(R, C, fmt, two_d, None, None, None, None, row_major and not two_d)
    if amax is not None:
        amax[0] = torch.maximum(amax[0], xf.abs().max())
    if two_d:
        tmax = xf.abs().reshape(nr, BLOCK, nc, BLOCK).amax(dim=(1, 3))  # [nr, nc]
        e = scale_exponent(tmax, fmt)
        inv = pow2(-e).repeat_interleave(BLOCK, 0).repeat_interleave(BLOCK, 1)
        q = (xf * inv).to(dt)
        out.s_row = pow2(e).t().contiguous()
        if rowwise:
            out.q_row = q
        if colwise:
            out.q_col = q.t().contiguous()
        return out
    if rowwise:
        bmax = xf.abs().reshape(R, nc, BLOCK).amax(-1)  # [R, nc]
        e = scale_exponent(bmax, fmt)
        out.q_row = (xf * pow2(-e).repeat_interleave(BLOCK, 1)).to(dt)
        out.s_row = pow2(e).contiguous() if out.row_major else pow2(e).t().contiguous()
    if colwise:
        bmax = xf.abs().reshape(nr, BLOCK, C).amax(1)  # [nr, C]
        e = scale_exponent(bmax, fmt)
        out.q_col = (xf * pow2(-e).repeat_interleave(BLOCK, 0)).to(dt).t().contiguous()
        out.s_col = pow2(e).contiguous()
    return out


def gemm_reference(a: Fp8Operand, b: Fp8Operand, *, out: torch.Tensor | None = None,
                   out_dtype: torch.dtype = torch.bfloat16, accumulate: bool = False, alpha: float = 1.0,
                   residual: torch.Tensor | None = None):
    """``gemm`` in PyTorch: block products summed in fp32 (the kernel's order of K-blocks)."""
    nk = a.K // BLOCK
    sa, sb = a.scale_matrix(), b.scale_matrix()
    acc = torch.zeros(a.rows, b.rows, dtype=torch.float32, device=a.data.device)
    af, bf = a.data.float(), b.data.float()
    for kb in range(nk):
        sl = slice(kb * BLOCK, (kb + 1) * BLOCK)
        acc += (af[:, sl] @ bf[:, sl].t()) * (sa[:, kb:kb + 1] * sb[:, kb][None, :])
    acc = acc * alpha
    if residual is not None:
        acc = acc + residual.float()
    if accumulate:
        out += acc
        return out
    if out is None:
        return acc.to(out_dtype)
    out.copy_(acc)
    return out
