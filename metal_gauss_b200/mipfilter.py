"""Mip-Splatting's 3D smoothing filter, on the GPU (drop-in for
metal_gauss/mipfilter.py).

    filter_3d = min over the cameras that see it of depth / max focal * sqrt(0.2)
    scales'   = sqrt(scales^2 + filter_3d^2)
    opacity'  = opacity * sqrt(prod(scales^2) / prod(scales'^2))

`compute_3d_filter` (mipfilter.py:30-76) runs as one pass over the Gaussians
that visits every camera (`mg_compute_3d_filter`); `apply_3d_filter`
(mipfilter.py:79-93) is an autograd function over `mg_apply_3d_filter` and its
adjoint, differentiable in scales and opacities with the filter constant, as
in the reference. The training engine applies the filter itself
(`Trainer.compute_filter_3d`) and carries its gradient inside the projection
adjoint.
"""

from __future__ import annotations

import torch

from . import _lib
from ._lib import ptr


def _view_size(v) -> tuple[int, int]:
    if hasattr(v, "width") and hasattr(v, "height"):
        return int(v.width), int(v.height)
    H, W = v.image.shape[:2]           # the reference's training views
    return int(W), int(H)


def _camera(v) -> _lib.Camera:
    W, H = _view_size(v)
    vm = torch.as_tensor(v.viewmat).detach().to("cpu", torch.float32)
    K = torch.as_tensor(v.K).detach().to("cpu", torch.float32)
    return _lib.make_camera(vm, float(K[0, 0]), float(K[1, 1]), float(K[0, 2]), float(K[1, 2]),
                            W, H, 0.01, 100.0, 0.3, float(max(W, H)), torch.zeros(3))


@torch.no_grad()
def compute_3d_filter(means: torch.Tensor, views, near: float = 0.2,
                      margin: float = 0.15) -> torch.Tensor:
    """Per-Gaussian low-pass scale (N,), from the cameras `views` (with .K,
    .viewmat and either .width/.height or an .image of the frame size). A
    Gaussian no camera sees gets the largest distance any Gaussian got."""
    if means.device.type != "cuda":
        raise RuntimeError("compute_3d_filter: the CUDA backend needs CUDA tensors")
    views = list(views)
    m = means.detach().to(torch.float32).contiguous()
    n = m.shape[0]
    out = torch.empty(n, dtype=torch.float32, device=m.device)
    cams = (_lib.Camera * max(1, len(views)))(*[_camera(v) for v in views])
    scratch = torch.empty(_lib.load().mg_compute_3d_filter_scratch_bytes(), dtype=torch.uint8,
                          device=m.device)
    _lib.call("mg_compute_3d_filter", ptr(m), n, _lib.C.cast(cams, _lib.C.c_void_p), len(views),
              float(near), float(margin), ptr(out), ptr(scratch), scratch.numel(), _lib.stream())
    return out


class _Apply3dFilter(torch.autograd.Function):
    @staticmethod
    def forward(ctx, scales, opacities, filter_3d):
        s = scales.detach().to(torch.float32).contiguous()
        o = opacities.detach().to(torch.float32).contiguous()
        f = filter_3d.detach().to(torch.float32).contiguous()
        out_s, out_o = torch.empty_like(s), torch.empty_like(o)
        _lib.call("mg_apply_3d_filter", ptr(s), ptr(o), ptr(f), s.shape[0], ptr(out_s),
                  ptr(out_o), _lib.stream())
        ctx.save_for_backward(s, o, f)
        return out_s, out_o

    @staticmethod
    def backward(ctx, g_s, g_o):
        s, o, f = ctx.saved_tensors
        g_s = torch.zeros_like(s) if g_s is None else g_s.to(torch.float32).contiguous()
        g_o = torch.zeros_like(o) if g_o is None else g_o.to(torch.float32).contiguous()
        d_s, d_o = torch.empty_like(s), torch.empty_like(o)
        _lib.call("mg_apply_3d_filter_backward", ptr(s), ptr(o), ptr(f), ptr(g_s), ptr(g_o),
                  s.shape[0], ptr(d_s), ptr(d_o), _lib.stream())
        return d_s, d_o, None


def apply_3d_filter(scales: torch.Tensor, opacities: torch.Tensor, filter_3d: torch.Tensor):
    """Widen the Gaussians and dim them to match: (scales (N,3), opacities
    (N,)) -> (new scales, new opacities), differentiable in both inputs."""
    if scales.device.type != "cuda":
        raise RuntimeError("apply_3d_filter: the CUDA backend needs CUDA tensors")
    return _Apply3dFilter.apply(scales, opacities, filter_3d)
