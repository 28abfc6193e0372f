"""SSIM and the training loss on the device (train.py:38-105, ssim.py).

`gaussian_kernel`, `ssim` and `_SSIMFused` keep the reference trainer's
interface and the five-kernel structure of its fused SSIM (stack + blur,
blur, tail; tail adjoint, two blurs, chain). `l1_ssim_loss` is the training
path: 0.8 L1 + 0.2 (1 - SSIM) forward and backward in two tiled kernels; its
backward only scales the gradient computed in the forward.
"""

from __future__ import annotations

import torch

from . import ext


def gaussian_kernel(size: int = 11, sigma: float = 1.5, device="cuda", groups: int = 15):
    """1D window shaped (groups,1,1,size), as train._gaussian_kernel."""
    x = torch.arange(size, dtype=torch.float32, device=device) - size // 2
    g = torch.exp(-x ** 2 / (2 * sigma ** 2))
    return (g / g.sum()).view(1, 1, 1, size).expand(groups, 1, 1, size).contiguous()


_gaussian_kernel = gaussian_kernel


class _SSIMFused(torch.autograd.Function):
    """Whole SSIM on the device (train.py:67-105): returns the (1,3,H,W) map."""

    @staticmethod
    def forward(ctx, a, b, w):
        H, W = a.shape[0], a.shape[1]
        inter = ext.ssim_stack_blur_h(a, b, w, H, W)
        blurred = ext.ssim_blur15(inter, w, 1, H, W)
        ctx.save_for_backward(a, b, w, blurred)
        return ext.ssim_tail_forward(blurred, H, W)

    @staticmethod
    def backward(ctx, grad_out):
        a, b, w, blurred = ctx.saved_tensors
        H, W = a.shape[0], a.shape[1]
        d_blur = ext.ssim_tail_backward(blurred, grad_out.contiguous(), H, W)
        d_inter = ext.ssim_blur15(d_blur, w, 1, H, W)   # vertical adjoint
        d_stack = ext.ssim_blur15(d_inter, w, 0, H, W)  # horizontal adjoint
        return ext.ssim_chain_backward(a, b, d_stack, H, W), None, None


def ssim(a: torch.Tensor, b: torch.Tensor, kernel: torch.Tensor) -> torch.Tensor:
    """a, b: (H,W,3) in [0,1]; 11-tap sigma 1.5 SSIM (train.py:52-64)."""
    return _SSIMFused.apply(a.contiguous(), b.contiguous(),
                            kernel[0, 0, 0].contiguous()).mean()


class _L1SSIMLoss(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, y, w, w_l1, w_ssim):
        loss, grad = ext.l1_ssim_loss(x.contiguous(), y.contiguous(), w, w_l1, w_ssim)
        ctx.save_for_backward(grad)
        return loss[0]

    @staticmethod
    def backward(ctx, g):
        (grad,) = ctx.saved_tensors
        return grad * g, None, None, None, None


def l1_ssim_loss(x: torch.Tensor, y: torch.Tensor, kernel: torch.Tensor | None = None,
                 w_l1: float = 0.8, w_ssim: float = 0.2) -> torch.Tensor:
    """w_l1 * mean|x - y| + w_ssim * (1 - SSIM(x, y)) for (H,W,3) images,
    differentiable in x (train.py:389-393)."""
    if kernel is None:
        kernel = gaussian_kernel(device=x.device)
    w = kernel[0, 0, 0].contiguous() if kernel.dim() == 4 else kernel.contiguous()
    return _L1SSIMLoss.apply(x, y, w, w_l1, w_ssim)
