"""CUDA backend: the reference's render() on sm_100a kernels.

Mirrors metal_gauss/metal_backend.py: the same render() keyword surface and
positional order (sh_rest last, metal_backend.py:396-407), the same info keys
(:551-559), the same two autograd functions (preprocess and rasterise), the
split SH layout without concatenation, absgrad through a caller buffer, and
antialias applied to opacity before binning. Differences, all inside the
backend: binning, the radix sort and the per-tile ranges run on the device
(bin_and_sort); the background blend is folded into the rasteriser; the
explicit-colour route uses the same fused preprocess with colour evaluation
switched off instead of the torch projection.

Every tensor must already be on a CUDA device: CPU tensors are refused, never
moved, and nothing falls back to another renderer.
"""

from __future__ import annotations

import math

import torch

from . import _lib, ext
from ._lib import G2D_ABSUV, ptr

SUPPORTED_TILES = (8, 12, 16, 32)


def _check_tile(tile: int) -> None:
    if tile not in SUPPORTED_TILES:
        raise RuntimeError(
            f"tile {tile} needs {tile * tile} threads per threadgroup (one CUDA block per "
            f"tile); the rasteriser supports tiles {SUPPORTED_TILES}, at most 1024 threads")


class _PreprocessCUDA(torch.autograd.Function):
    """Fused projection + SH + activation (metal_backend.py:288-333)."""

    @staticmethod
    def forward(ctx, means, quats, scales, sh, sh_rest, ctx_opac, viewmat, fx, fy, cx, cy, W, H,
                near, far, blur, max_radius, cam_center, sh_degree):
        fused = sh_rest is sh
        args = [t.contiguous() for t in (means, quats, scales)]
        sh_c = None if sh is None else sh.contiguous()
        rest = sh_c if fused else (None if sh_rest is None else sh_rest.contiguous())
        uv, conic, depth, rxy, valid, color = ext.preprocess_forward(
            *args, sh_c, rest, ctx_opac.contiguous(), viewmat, fx, fy, cx, cy, W, H, near, far,
            blur, max_radius, cam_center, sh_degree)
        ctx.save_for_backward(*args, *(t for t in (sh_c, rest) if t is not None), valid)
        ctx.has_sh = sh is not None
        ctx.fused = fused
        ctx.meta = (viewmat, fx, fy, cx, cy, W, H, near, far, blur, max_radius, cam_center,
                    sh_degree)
        ctx.mark_non_differentiable(depth, rxy, valid)
        return uv, conic, depth, rxy, valid, color

    @staticmethod
    def backward(ctx, d_uv, d_conic, d_depth, d_rxy, d_valid, d_color):
        saved = ctx.saved_tensors
        means, quats, scales = saved[:3]
        if ctx.has_sh:
            sh, rest = saved[3], saved[4]
        else:
            sh = rest = None
        valid = saved[-1]
        n = means.shape[0]
        if d_uv is None:
            d_uv = torch.zeros(n, 2, device=means.device)
        if d_conic is None:
            d_conic = torch.zeros(n, 3, device=means.device)
        if d_color is None and ctx.has_sh:
            d_color = torch.zeros(n, 3, device=means.device)
        d_means, d_quats, d_scales, d_sh, d_sh_rest = ext.preprocess_backward(
            means, quats, scales, sh, rest, d_uv, d_conic, d_color if ctx.has_sh else None,
            valid, *ctx.meta)
        # fused layout: d_sh and d_sh_rest alias; return it once (never doubled)
        d_rest = None if (ctx.fused or not ctx.has_sh) else d_sh_rest
        return (d_means, d_quats, d_scales, d_sh, d_rest) + (None,) * 14


class _RasterizeCUDA(torch.autograd.Function):
    """Tile rasterisation, forward and backward (metal_backend.py:336-364).
    absgrad is a statistic, not an adjoint: the caller's buffer is filled by
    the backward."""

    @staticmethod
    def forward(ctx, uv, conic, opacity, color, gauss_ids, tile_offsets, W, H, tile, tiles_x,
                absgrad_out=None, background=None):
        args = [t.contiguous() for t in (uv, conic, opacity, color)]
        state = []
        rgb, alpha, T, ncontrib = ext.rasterize_forward(*args, gauss_ids, tile_offsets, W, H,
                                                        tile, tiles_x, background=background,
                                                        state_out=state)
        # the packed records and checkpoints let the backward split long
        # walks into segments; rgb and alpha are saved so in-place edits of
        # the outputs are caught by autograd's version check
        ctx.save_for_backward(*args, gauss_ids, tile_offsets, T, ncontrib, alpha, rgb)
        ctx.state = state[0]
        ctx.dims = (W, H, tile, tiles_x)
        ctx.absgrad_out = absgrad_out
        ctx.background = background
        return rgb, alpha

    @staticmethod
    def backward(ctx, grad_rgb, grad_alpha):
        (uv, conic, opacity, color, gauss_ids, tile_offsets, T, ncontrib, alpha,
         rgb) = ctx.saved_tensors
        W, H, tile, tiles_x = ctx.dims
        if grad_rgb is None:
            grad_rgb = torch.zeros(H, W, 3, device=uv.device)
        want_abs = ctx.absgrad_out is not None
        g = ext.rasterize_backward_packed(uv, conic, opacity, color, gauss_ids, tile_offsets, T,
                                          ncontrib, grad_rgb, grad_alpha, W, H, tile, tiles_x,
                                          want_abs, background=ctx.background, alpha=alpha,
                                          state=ctx.state, rgb=rgb)
        ctx.state = None
        if want_abs:
            ctx.absgrad_out[:g.shape[0]] += g[:, G2D_ABSUV]
        return (g[:, 0:2], g[:, 4:7], g[:, 2], g[:, 8:11]) + (None,) * 8


class _AntialiasOpacity(torch.autograd.Function):
    """opacity * antialias_scale(conic, blur) (metal_backend.py:506-511) in
    one kernel each way: mg_antialias_opacity and its adjoint, which carries
    the gradient to both the conic and the opacity."""

    @staticmethod
    def forward(ctx, conic, opacities, blur):
        c = conic.detach().to(torch.float32).contiguous()
        o = opacities.detach().to(torch.float32).contiguous()
        out = torch.empty_like(o)
        _lib.call("mg_antialias_opacity", ptr(c), ptr(o), c.shape[0], float(blur), ptr(out),
                  _lib.stream())
        ctx.save_for_backward(c, o)
        ctx.blur = float(blur)
        return out

    @staticmethod
    def backward(ctx, g):
        c, o = ctx.saved_tensors
        d_c, d_o = torch.empty_like(c), torch.empty_like(o)
        _lib.call("mg_antialias_opacity_backward", ptr(c), ptr(o),
                  ptr(g.to(torch.float32).contiguous()), c.shape[0], ctx.blur, ptr(d_c),
                  ptr(d_o), _lib.stream())
        return d_c, d_o, None


def antialias_opacity(conic: torch.Tensor, opacities: torch.Tensor, blur: float) -> torch.Tensor:
    """The compensated opacities the rasteriser draws with antialiasing on,
    differentiable in the conic and the opacities."""
    return _AntialiasOpacity.apply(conic, opacities, blur)


def antialias_scale(conic: torch.Tensor, blur: float) -> torch.Tensor:
    """Mip-Splatting opacity compensation sqrt(det_before/det_after),
    recovered from the conic (metal_backend.py:367-393), as a torch
    expression (the reference's own helper; render() uses the fused
    antialias_opacity)."""
    cxx, cxy, cyy = conic[:, 0], conic[:, 1], conic[:, 2]
    det_conic = (cxx * cyy - cxy * cxy).clamp_min(1e-12)
    det_after = 1.0 / det_conic
    a = cyy * det_after
    b = -cxy * det_after
    c = cxx * det_after
    det_before = (a - blur) * (c - blur) - b * b
    return (det_before.clamp_min(0.0) / det_after).clamp(0.0, 1.0).sqrt()


def build_tile_lists_cuda(uv, rxy, depth, valid, conic, opacity, W, H, tile,
                          max_per_tile: int = 0, workspace=None):
    """Device binning with the exact ellipse test: (gauss_ids, tile_offsets,
    tiles_x), gauss_ids sorted by (tile, depth) -- the contract of
    build_tile_lists_metal (metal_backend.py:217-285). `max_per_tile` keeps
    the nearest N per tile (an approximation, off by default, :262-283)."""
    ids, offsets, tx = ext.bin_and_sort(uv.contiguous(), rxy.contiguous(), conic.contiguous(),
                                        opacity.contiguous(), valid.to(torch.int32).contiguous(),
                                        depth.contiguous(), W, H, tile, workspace=workspace)
    if max_per_tile > 0 and ids.numel() > 0:
        n_tiles = offsets.numel() - 1
        counts = (offsets[1:] - offsets[:-1]).to(torch.int64)
        tile_of = torch.repeat_interleave(torch.arange(n_tiles, device=ids.device), counts)
        rank = torch.arange(ids.numel(), device=ids.device) - offsets[:-1].to(torch.int64)[tile_of]
        keep = rank < max_per_tile
        ids = ids[keep].contiguous()
        kept = torch.minimum(counts, torch.tensor(max_per_tile, device=ids.device))
        offsets = torch.cat([torch.zeros(1, dtype=torch.int64, device=ids.device),
                             torch.cumsum(kept, 0)]).to(torch.int32)
    return ids, offsets, tx


def render(means, quats, scales, opacities, sh, K, viewmat, W, H,
           sh_degree: int = 3, tile: int | None = None,
           near: float = 0.01, far: float = 100.0,
           background=(0.0, 0.0, 0.0), colors=None, max_radius_frac: float = 1.0,
           sh_rest=None, antialias: bool = False, absgrad_out=None, **_ignored):
    """Same positional signature as metal_backend.render / torch_ref.render.
    Returns (rgb (H,W,3), alpha (H,W), info)."""
    explicit_colors = colors is not None
    if means.device.type != "cuda":
        raise RuntimeError(
            f"cuda backend requires CUDA tensors, got device '{means.device}'. "
            "Refusing to silently move data or fall back to another backend.")
    if tile is None:
        tile = 16
    _check_tile(tile)
    K_h = K if K.device.type == "cpu" else K.detach().cpu()
    fx, fy, cx, cy = (float(K_h[0, 0]), float(K_h[1, 1]), float(K_h[0, 2]), float(K_h[1, 2]))
    vm_h = viewmat.detach()
    if vm_h.device.type != "cpu":
        vm_h = vm_h.cpu()
    vm_h = vm_h.to(torch.float32).contiguous()
    cam_center = -vm_h[:3, :3].T @ vm_h[:3, 3]

    if explicit_colors:
        sh_in = rest_in = None
        deg = -1
    elif sh_rest is None:
        sh_in = sh
        if sh_in.shape[1] < 16:
            pad = torch.zeros(sh_in.shape[0], 16 - sh_in.shape[1], 3, device=sh_in.device,
                              dtype=sh_in.dtype)
            sh_in = torch.cat([sh_in, pad], dim=1)
        rest_in = sh_in
        deg = sh_degree
    else:
        if sh.shape[1] != 1:
            raise ValueError(
                f"with sh_rest given, sh must be the DC band (N,1,3); got {tuple(sh.shape)}")
        sh_in, rest_in = sh, sh_rest
        if rest_in.shape[1] < 15:
            pad = torch.zeros(rest_in.shape[0], 15 - rest_in.shape[1], 3, device=rest_in.device,
                              dtype=rest_in.dtype)
            rest_in = torch.cat([rest_in, pad], dim=1)
        deg = sh_degree

    uv, conic, depth, rxy, valid_i, pre_color = _PreprocessCUDA.apply(
        means, quats, scales, sh_in, rest_in, opacities.detach(), vm_h, fx, fy, cx, cy, W, H,
        near, far, 0.3, max_radius_frac * max(W, H), cam_center, deg)
    colors = colors if explicit_colors else pre_color
    valid_b = valid_i.bool()
    if antialias:
        # before binning: the SnugBox bound then uses the compensated opacity
        opacities = antialias_opacity(conic, opacities, 0.3)

    gauss_ids, tile_offsets, tiles_x = build_tile_lists_cuda(
        uv.detach(), rxy.detach(), depth.detach(), valid_i, conic.detach(), opacities.detach(),
        W, H, tile)

    bg = None if background is None else tuple(float(x) for x in background)
    rgb, alpha = _RasterizeCUDA.apply(uv, conic, opacities, colors, gauss_ids, tile_offsets,
                                      W, H, tile, tiles_x, absgrad_out, bg)
    if uv.requires_grad:
        uv.retain_grad()
    return rgb, alpha, {
        "uv": uv,
        "tiles": int(tile_offsets.numel() - 1),
        "isect_total": int(gauss_ids.numel()),
        "isect_dropped": 0,
        "isect_dropped_frac": 0.0,
        "valid_mask": valid_b,
        "backend": "cuda",
    }
