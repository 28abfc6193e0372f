"""Adam that updates only the visible Gaussians' rows, on the device.

Same interface and state as metal_gauss/selective_adam.py:22-206: rowwise
groups (the default) take the visibility mask passed to step() and keep one
step count per Gaussian ('steps', float) for the bias corrections, with
    p -= lr * sqrt(1 - b2^k) / (1 - b1^k) * m / (sqrt(v) + eps);
groups marked rowwise=False (e.g. per-image appearance) get ordinary Adam
('step' int). A mask shorter than the parameter's row count treats the extra
(preallocated capacity) rows as invisible. Each rowwise parameter is one
kernel pass over its rows plus a tiny step-count update, instead of the
reference's gathers and scatters.
"""

from __future__ import annotations

import torch

from . import ext


class SelectiveAdam(torch.optim.Optimizer):
    def __init__(self, groups: list[dict], eps: float = 1e-15,
                 betas: tuple[float, float] = (0.9, 0.999)):
        defaults = {"lr": 1e-3, "eps": eps, "betas": betas, "rowwise": True}
        super().__init__(groups, defaults)
        self.groups = self.param_groups

    def _state_for(self, p: torch.Tensor, rowwise: bool) -> dict:
        st = self.state[p]
        if "exp_avg" not in st:
            st["exp_avg"] = torch.zeros_like(p)
            st["exp_avg_sq"] = torch.zeros_like(p)
            if rowwise:
                st["steps"] = torch.zeros(p.shape[0], device=p.device)
            else:
                st["step"] = 0
        return st

    @staticmethod
    def _check_gradient(p: torch.Tensor) -> torch.Tensor:
        grad = p.grad
        if grad.is_sparse:
            raise RuntimeError("SelectiveAdam does not support sparse gradients")
        if grad.shape != p.shape:
            raise ValueError(f"gradient shape {tuple(grad.shape)} does not match parameter "
                             f"shape {tuple(p.shape)}")
        if not p.is_cuda:
            raise RuntimeError("SelectiveAdam (cuda) requires CUDA tensors, got device "
                               f"'{p.device}'; refusing to fall back")
        if not p.is_contiguous():
            raise RuntimeError("SelectiveAdam updates parameters in place and needs them "
                               "contiguous")
        return grad.contiguous()

    @torch.no_grad()
    def step(self, visible: torch.Tensor, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        if visible.ndim != 1 or visible.dtype is not torch.bool:
            raise TypeError("visible must be a one-dimensional boolean tensor")
        vis_u8 = None
        for group in self.param_groups:
            lr, eps = group["lr"], group["eps"]
            b1, b2 = group["betas"]
            for p in group["params"]:
                if p.grad is None:
                    continue
                grad = self._check_gradient(p)
                if not group["rowwise"]:
                    st = self._state_for(p, rowwise=False)
                    st["step"] += 1
                    ext.adam_step(p.view(-1), grad.view(-1), st["exp_avg"].view(-1),
                                  st["exp_avg_sq"].view(-1), lr, b1, b2, eps, st["step"])
                    continue
                if p.dim() == 0 or p.shape[0] < visible.numel():
                    raise ValueError("rowwise SelectiveAdam parameters must have at least one "
                                     "row per visibility-mask entry")
                if vis_u8 is None or vis_u8.device != p.device:
                    vis_u8 = visible.to(device=p.device, dtype=torch.uint8).contiguous()
                st = self._state_for(p, rowwise=True)
                ext.selective_adam_step(p, grad, st["exp_avg"], st["exp_avg_sq"], st["steps"],
                                        vis_u8, lr, b1, b2, eps)
        return loss
