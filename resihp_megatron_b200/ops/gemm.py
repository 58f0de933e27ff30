"""bf16 GEMM on tcgen05 tensor cores (``csrc/gemm_sm100.cu``).

``gemm(a, b)`` computes ``op(a) @ op(b).T`` where ``op(a)`` is ``[M, K]`` and ``op(b)`` is
``[N, K]``.  ``a_t=True`` means ``a`` is stored as ``[K, M]`` (so ``op(a) = a.T``) and
``b_t=True`` means ``b`` is stored as ``[K, N]``.  The kernel reads either layout directly
(K-major or MN-major shared-memory operands), so the three GEMMs of a linear layer need no
transpose:

* forward ``y = x @ w.T``      -> ``gemm(x, w)``
* dgrad   ``dx = dy @ w``      -> ``gemm(dy, w, b_t=True)``
* wgrad   ``dw = dy.T @ x``    -> ``gemm(dy, x, a_t=True, b_t=True)`` (fp32, accumulating)

``variant``: 0 picks the kernel (the 2-CTA ``cta_group::2`` kernel for M >= 512 and N >= 256,
with split-K in two k shares when the tile count would leave the last wave of SM pairs mostly
idle), 1 the single-CTA kernel, 2 the CTA pair without split, 3 the CTA pair with split forced,
4 the CTA pair with a 7-stage operand ring, 5 the CTA pair with 256 x 128 tiles, 6 the CTA pair
with only the partial last wave's tiles split (tuning).

The reference framework has no GEMM of its own; its compute path is Megatron/TE
(``resihp/runtime/megatron_runtime.py``) and its GEMM probe is ``torch.matmul``
(``resihp/detect/validation.py:17-31``).
"""

from __future__ import annotations

import torch

from ._build import ext
from .counter import count

EPI_BF16 = 0
EPI_F32 = 1
EPI_F32_ACC = 2
EPI_BF16_RES = 3


def gemm(
    a: torch.Tensor,
    b: torch.Tensor,
    *,
    a_t: bool = False,
    b_t: bool = False,
    out: torch.Tensor | None = None,
    out_dtype: torch.dtype = torch.bfloat16,
    accumulate: bool = False,
    residual: torch.Tensor | None = None,
    alpha: float = 1.0,
    variant: int = 0,
) -> torch.Tensor:
    M = a.shape[1] if a_t else a.shape[0]
    N = b.shape[1] if b_t else b.shape[0]
    if accumulate:
        if out is None or out.dtype != torch.float32:
            raise ValueError("accumulate=True needs an fp32 `out`")
        epi = EPI_F32_ACC
    elif residual is not None:
        epi = EPI_BF16_RES
    else:
        epi = EPI_F32 if (out.dtype if out is not None else out_dtype) == torch.float32 else EPI_BF16
    if out is None:
        out = torch.empty((M, N), dtype=torch.float32 if epi in (EPI_F32, EPI_F32_ACC) else torch.bfloat16,
                          device=a.device)
    ext().gemm(a, a_t, b, b_t, out, epi, float(alpha), residual, int(variant))
    count(1)
    return out


def error_state(device: int | None = None) -> torch.Tensor:
    """Per-device error words written by kernels whose bounded waits ran out (0 = clean)."""
    if device is None:
        device = torch.cuda.current_device()
    return ext().error_state(device)
