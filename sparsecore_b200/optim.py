"""AdamW that updates only the live slots of SparseLinear weights.

The reference trains SparseLinear with a stock torch optimizer over the
aliased padded ``values`` tensor (``sparselab/nn.py:183-184``): every slot,
padding included, is read and written each step.  ``LiveAdamW`` keeps
torch's AdamW semantics (decoupled weight decay, per-slot state that stays
with the slot across topology rewrites) but runs one fused kernel per sparse
weight (``sl_adamw_live``) that skips padding slots -- their value stays
exactly 0 and their moments are never touched -- and a stock
``torch.optim.AdamW`` for every other parameter.

Values agree with ``torch.optim.AdamW`` to float rounding (rel 1e-6), not
bit for bit: torch's foreach kernels round some steps differently.  The step
counter lives on the host, so the optimizer is not CUDA-graph capturable;
use ``torch.optim.AdamW(capturable=True)`` inside a captured step.
"""
from __future__ import annotations

import torch

from . import _native as N

__all__ = ["LiveAdamW"]


class LiveAdamW(torch.optim.Optimizer):
    def __init__(self, model: torch.nn.Module, lr: float = 1e-3, betas=(0.9, 0.999),
                 eps: float = 1e-8, weight_decay: float = 1e-2):
        from .nn import SparseLinear

        if lr < 0.0 or eps < 0.0 or not (0.0 <= betas[0] < 1.0) or not (0.0 <= betas[1] < 1.0):
            raise ValueError(f"LiveAdamW: invalid hyper-parameters lr={lr}, betas={betas}, eps={eps}")
        self.sparse = [m for m in model.modules() if isinstance(m, SparseLinear)]
        sparse_ids = {id(m._values) for m in self.sparse}
        dense = [p for p in model.parameters() if p.requires_grad and id(p) not in sparse_ids]
        defaults = dict(lr=lr, betas=tuple(betas), eps=eps, weight_decay=weight_decay)
        super().__init__([m._values for m in self.sparse] or [torch.zeros(0)], defaults)
        self.dense_opt = (torch.optim.AdamW(dense, lr=lr, betas=betas, eps=eps,
                                            weight_decay=weight_decay) if dense else None)

    @torch.no_grad()
    def step(self, closure=None):
        loss = closure() if closure is not None else None
        group = self.param_groups[0]
        b1, b2 = group["betas"]
        for m in self.sparse:
            p = m._values
            if p.grad is None:
                continue
            st = self.state[p]
            if not st:
                st["step"] = 0
                st["exp_avg"] = torch.zeros_like(p)
                st["exp_avg_sq"] = torch.zeros_like(p)
            st["step"] += 1
            csr = m._csr
            N.call("sl_adamw_live", csr._abi_ref(), N.ptr(p.grad), N.ptr(st["exp_avg"]),
                   N.ptr(st["exp_avg_sq"]), float(group["lr"]), float(b1), float(b2),
                   float(group["eps"]), float(group["weight_decay"]), int(st["step"]),
                   csr._stream())
        if self.dense_opt is not None:
            for g in self.dense_opt.param_groups:
                g["lr"] = group["lr"]
            self.dense_opt.step()
        return loss

    def zero_grad(self, set_to_none: bool = True):
        super().zero_grad(set_to_none=set_to_none)
        if self.dense_opt is not None:
            self.dense_opt.zero_grad(set_to_none=set_to_none)
