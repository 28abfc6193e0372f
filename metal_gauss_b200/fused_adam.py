"""Adam in one device pass (metal_gauss/fused_adam.py:26-54; adam.metal:25-42).

torch.optim.Adam's arithmetic, including where eps enters (after dividing by
sqrt(bias_correction2)), and torch's state layout ('step', 'exp_avg',
'exp_avg_sq' per parameter), which MCMC relocation edits in place
(mcmc.py:107-121).
"""

from __future__ import annotations

import torch

from . import ext


class FusedAdam(torch.optim.Optimizer):
    def __init__(self, params, lr=1e-3, betas=(0.9, 0.999), eps=1e-15):
        super().__init__(params, dict(lr=lr, betas=betas, eps=eps))

    @torch.no_grad()
    def step(self, closure=None):
        loss = closure() if closure is not None else None
        for group in self.param_groups:
            b1, b2 = group["betas"]
            lr, eps = group["lr"], group["eps"]
            for p in group["params"]:
                if p.grad is None:
                    continue
                g = p.grad
                if g.is_sparse:
                    raise RuntimeError("FusedAdam does not support sparse gradients")
                st = self.state[p]
                if not st:
                    st["step"] = 0
                    st["exp_avg"] = torch.zeros_like(p)
                    st["exp_avg_sq"] = torch.zeros_like(p)
                st["step"] += 1
                ext.adam_step(p.view(-1), g.contiguous().view(-1), st["exp_avg"].view(-1),
                              st["exp_avg_sq"].view(-1), lr, b1, b2, eps, st["step"])
        return loss
