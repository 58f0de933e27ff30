"""Adam(W) with explicit, name-keyed state (CPU semantic path and migration tests).

The update is bit-for-bit that of ``torch.optim.Adam(foreach=False)``: the same tensor ops in
the same order (lerp for the first moment, mul + addcmul for the second, bias-corrected denom,
addcdiv).  State lives in plain tensors keyed by parameter name so the migration engine can
slice, ship and reshard it (``state_tensors`` / ``load_state_tensors`` use the ``param/``,
``exp_avg/`` and ``exp_avg_sq/`` prefixes).  The GPU path runs the same formula in one fused
kernel over flat fp32 buffers (``ops.adam_step``).  (Reference: ``resihp/runtime/optim.py``.)
"""

from __future__ import annotations

import math

import torch


@torch.no_grad()
def adam_update_(p: torch.Tensor, g: torch.Tensor, m: torch.Tensor, v: torch.Tensor, step: int, lr: float,
                 betas=(0.9, 0.999), eps: float = 1e-8, weight_decay: float = 0.0) -> None:
    b1, b2 = betas
    bc1 = 1 - b1 ** step
    bc2_sqrt = math.sqrt(1 - b2 ** step)
    if weight_decay:
        g = g.add(p, alpha=weight_decay)
    m.lerp_(g, 1 - b1)
    v.mul_(b2).addcmul_(g, g.conj(), value=1 - b2)
    denom = (v.sqrt() / bc2_sqrt).add_(eps)
    p.addcdiv_(m, denom, value=-lr / bc1)


class Adam:
    def __init__(self, params: dict[str, torch.Tensor], lr: float = 1e-3, betas=(0.9, 0.999), eps: float = 1e-8,
                 weight_decay: float = 0.0):
        self.params = dict(params)
        self.lr, self.betas, self.eps, self.weight_decay = lr, betas, eps, weight_decay
        self.step_count = 0
        self.state = {n: {"exp_avg": torch.zeros_like(p), "exp_avg_sq": torch.zeros_like(p)}
                      for n, p in self.params.items()}

    def zero_grad(self) -> None:
        for p in self.params.values():
            p.grad = None

    @torch.no_grad()
    def step(self) -> None:
        self.step_count += 1
        for n, p in self.params.items():
            g = p.grad if p.grad is not None else torch.zeros_like(p)
            s = self.state[n]
            adam_update_(p, g, s["exp_avg"], s["exp_avg_sq"], self.step_count, self.lr, self.betas, self.eps,
                         self.weight_decay)

    def state_tensors(self) -> dict[str, torch.Tensor]:
        out: dict[str, torch.Tensor] = {}
        for n, p in self.params.items():
            out[f"param/{n}"] = p.data
            out[f"exp_avg/{n}"] = self.state[n]["exp_avg"]
            out[f"exp_avg_sq/{n}"] = self.state[n]["exp_avg_sq"]
        return out

    def load_state_tensors(self, tensors: dict[str, torch.Tensor], step_count: int) -> None:
        with torch.no_grad():
            for n, p in self.params.items():
                p.data.copy_(tensors[f"param/{n}"])
                self.state[n]["exp_avg"].copy_(tensors[f"exp_avg/{n}"])
                self.state[n]["exp_avg_sq"].copy_(tensors[f"exp_avg_sq/{n}"])
        self.step_count = step_count
