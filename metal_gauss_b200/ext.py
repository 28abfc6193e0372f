"""The reference bridge's functions on CUDA tensors.

Same names, argument order and return lists as the pybind11 module that
metal_gauss.metal_backend._load() builds (metal_gauss/csrc/rasterize.mm:
518-533), implemented as thin torch wrappers over the C ABI of
libmg_b200.so: outputs are allocated here from PyTorch's caching allocator,
raw device pointers go down, and every call is enqueued on the current CUDA
stream. Added beyond the reference: sort_pairs, tile_ranges and bin_and_sort
(the device radix sort and range extraction that replace torch.argsort and
torch.searchsorted), selective_adam_step and l1_ssim_loss.
"""

from __future__ import annotations

import math

import torch

from . import _lib
from ._lib import G2D_ABSUV, G2D_COLOR, G2D_CONIC, G2D_OPACITY, G2D_STRIDE, G2D_UV, ptr

F32 = torch.float32


def _check(t: torch.Tensor, what: str, dtype=F32) -> torch.Tensor:
    if not t.is_cuda:
        raise RuntimeError(f"{what} must be a CUDA tensor (the cuda backend requires CUDA "
                           f"tensors), got device '{t.device}'")
    if t.dtype != dtype:
        raise RuntimeError(f"{what} must be {dtype}, got {t.dtype}")
    if not t.is_contiguous():
        raise RuntimeError(f"{what} must be contiguous")
    return t


def init(src: str | None = None) -> None:
    """Kept for the reference's call sequence (_ext.init(metal source)); the
    CUDA library is compiled ahead of time, so this only loads it."""
    _lib.load()


def _empty(shape, like: torch.Tensor, dtype=F32) -> torch.Tensor:
    return torch.empty(shape, dtype=dtype, device=like.device)


def sh_layout(sh: torch.Tensor, sh_rest: torch.Tensor):
    """SH layout check and uniform, as setShLayout (rasterize.mm:211-224)."""
    fused = sh.shape[1] == 16
    if not (fused or (sh.shape[1] == 1 and sh_rest.shape[1] == 15)):
        raise RuntimeError("SH must be either one (N,16,3) tensor or (N,1,3)+(N,15,3); got "
                           f"{tuple(sh.shape)} and {tuple(sh_rest.shape)}")
    return fused, (_lib.SH_FUSED if fused else _lib.SH_SPLIT)


# ------------------------------------------------------------------ preprocess

def preprocess_forward(means, quats, scales, sh, sh_rest, opacities, viewmat, fx, fy, cx, cy,
                       W, H, near, far, blur, max_radius, cam_center, sh_degree):
    """-> [uv (N,2), conic (N,3), depth (N,), rxy (N,2), valid (N,) int32,
    color (N,3)] (rasterize.mm:244-284). sh may be None for explicit colours."""
    for t, w in ((means, "means"), (quats, "quats"), (scales, "scales"),
                 (opacities, "opacities")):
        _check(t, w)
    n = means.shape[0]
    uv, conic, depth = _empty((n, 2), means), _empty((n, 3), means), _empty((n,), means)
    rxy, valid = _empty((n, 2), means), _empty((n,), means, torch.int32)
    color = _empty((n, 3), means)
    if sh is not None:
        _check(sh, "sh"), _check(sh_rest, "sh_rest")
        _, lay = sh_layout(sh, sh_rest)
        deg = int(sh_degree)
    else:
        lay, deg = _lib.SH_FUSED, -1
    cam = _lib.make_camera(viewmat, fx, fy, cx, cy, W, H, near, far, blur, max_radius,
                           cam_center)
    _lib.call("mg_preprocess_forward", ptr(means), ptr(quats), ptr(scales), ptr(sh),
              ptr(sh_rest), lay, ptr(opacities), _lib.C.byref(cam), deg, n, ptr(uv),
              ptr(conic), ptr(depth), ptr(rxy), ptr(valid), ptr(color), _lib.stream())
    return [uv, conic, depth, rxy, valid, color]


def _row_view(t: torch.Tensor, width: int, what: str) -> tuple[torch.Tensor, int]:
    """A (N, width) float view whose rows are contiguous; returns (t, stride)."""
    if t.dim() != 2 or t.shape[1] != width or t.stride(1) != 1 or t.dtype != F32 or not t.is_cuda:
        t = _check(t.contiguous().reshape(-1, width), what)
    return t, t.stride(0)


def preprocess_backward(means, quats, scales, sh, sh_rest, d_uv, d_conic, d_color, valid,
                        viewmat, fx, fy, cx, cy, W, H, near, far, blur, max_radius, cam_center,
                        sh_degree):
    """-> [d_means, d_quats, d_scales, d_sh, d_sh_rest] (rasterize.mm:286-327).
    The incoming gradients may be strided row views (e.g. into the packed
    rasteriser gradient record) and are read in place."""
    n = means.shape[0]
    d_uv, s_uv = _row_view(d_uv, 2, "d_uv")
    d_conic, s_conic = _row_view(d_conic, 3, "d_conic")
    d_means, d_quats, d_scales = _empty((n, 3), means), _empty((n, 4), means), _empty((n, 3), means)
    if sh is not None and d_color is not None:
        d_color, s_color = _row_view(d_color, 3, "d_color")
        fused, lay = sh_layout(sh, sh_rest)
        d_sh = _empty((n, 16 if fused else 1, 3), means)
        d_rest = d_sh if fused else _empty((n, 15, 3), means)
        deg = int(sh_degree)
    else:
        d_color, s_color, lay, d_sh, d_rest, deg = None, 3, _lib.SH_FUSED, None, None, -1
    cam = _lib.make_camera(viewmat, fx, fy, cx, cy, W, H, near, far, blur, max_radius,
                           cam_center)
    _lib.call("mg_preprocess_backward", ptr(means), ptr(quats), ptr(scales), ptr(sh),
              ptr(sh_rest), lay, ptr(d_uv), s_uv, ptr(d_conic), s_conic, ptr(d_color), s_color,
              ptr(valid), _lib.C.byref(cam), deg, n, ptr(d_means), ptr(d_quats), ptr(d_scales),
              ptr(d_sh), ptr(d_rest), _lib.stream())
    return [d_means, d_quats, d_scales, d_sh, d_rest]


# --------------------------------------------------------------------- binning

def bin_count(uv, rxy, conic, opacity, valid, W, H, tile, tiles_x, tiles_y):
    """-> counts (N,) int32 (rasterize.mm:485-497)."""
    n = uv.shape[0]
    counts = _empty((n,), uv, torch.int32)
    _lib.call("mg_bin_count", ptr(uv), ptr(rxy), ptr(conic), ptr(opacity), ptr(valid), n, W, H,
              tile, tiles_x, tiles_y, ptr(counts), _lib.stream())
    return counts


def bin_write(uv, rxy, conic, opacity, valid, depth, offsets, total, W, H, tile, tiles_x,
              tiles_y):
    """-> [keys (M,) int64 = tile<<32 | depth bits, ids (M,) int32]
    (rasterize.mm:499-516)."""
    n = uv.shape[0]
    keys = _empty((total,), uv, torch.int64)
    ids = _empty((total,), uv, torch.int32)
    _lib.call("mg_bin_write", ptr(uv), ptr(rxy), ptr(conic), ptr(opacity), ptr(valid),
              ptr(depth), ptr(offsets), total, n, W, H, tile, tiles_x, tiles_y, ptr(keys),
              ptr(ids), _lib.stream())
    return [keys, ids]


def sort_pairs(keys: torch.Tensor, vals: torch.Tensor, bits: int | None = None):
    """Stable radix sort of (keys, vals) on the low `bits` key bits; returns new
    (keys, vals). keys int32/int64 (read as unsigned), vals int32."""
    n = keys.numel()
    kb = keys.element_size()
    if bits is None:
        bits = 8 * kb
    k, v = keys.clone(), vals.clone()
    if n <= 1:
        return k, v
    k_alt, v_alt = torch.empty_like(k), torch.empty_like(v)
    nbytes = _lib.load().mg_sort_scratch_bytes(n, bits, kb)
    scratch = torch.empty(nbytes, dtype=torch.uint8, device=keys.device)
    fn = "mg_sort_pairs_u64" if kb == 8 else "mg_sort_pairs_u32"
    _lib.call(fn, ptr(k), ptr(v), ptr(k_alt), ptr(v_alt), n, bits, ptr(scratch), nbytes,
              _lib.stream())
    return k, v


def tile_ranges(sorted_keys: torch.Tensor, n_tiles: int) -> torch.Tensor:
    """offsets (T+1,) int32 from sorted 64-bit keys (tile in the high word) or
    sorted int32 tile ids; replaces the searchsorted of metal_backend.py:257."""
    offsets = torch.empty(n_tiles + 1, dtype=torch.int32, device=sorted_keys.device)
    m = sorted_keys.numel()
    if sorted_keys.element_size() == 8:
        _lib.call("mg_tile_ranges", None, ptr(sorted_keys), m, n_tiles, ptr(offsets),
                  _lib.stream())
    else:
        _lib.call("mg_tile_ranges", ptr(sorted_keys), None, m, n_tiles, ptr(offsets),
                  _lib.stream())
    return offsets


class BinWorkspace:
    """Reusable device scratch for bin_and_sort (grown on demand)."""

    def __init__(self):
        self.prep = None
        self.emit = None
        self.total = None

    def get(self, name: str, nbytes: int, device) -> torch.Tensor:
        buf = getattr(self, name)
        if buf is None or buf.numel() < nbytes or buf.device != torch.device(device):
            buf = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=device)
            setattr(self, name, buf)
        return buf


_default_ws: dict[int, BinWorkspace] = {}


def bin_and_sort(uv, rxy, conic, opacity, valid, depth, W, H, tile, workspace=None):
    """The whole binning of one view: -> (gauss_ids (M,) int32 sorted by
    (tile, depth, Gaussian index), tile_offsets (T+1,) int32, tiles_x).
    One device->host read (the pair total), as build_tile_lists_metal."""
    dev = uv.device
    n = uv.shape[0]
    tx, ty = math.ceil(W / tile), math.ceil(H / tile)
    if n == 0:
        return (torch.zeros(0, dtype=torch.int32, device=dev),
                torch.zeros(tx * ty + 1, dtype=torch.int32, device=dev), tx)
    ws = workspace or _default_ws.setdefault(dev.index or 0, BinWorkspace())
    L = _lib.load()
    pbytes = L.mg_bin_prepare_scratch_bytes(n, tx * ty)
    prep = ws.get("prep", pbytes, dev)
    total_dev = ws.get("total", 8, dev)
    s = _lib.stream()
    _lib.call("mg_bin_prepare", ptr(uv), ptr(rxy), ptr(conic), ptr(opacity), ptr(valid),
              ptr(depth), n, W, H, tile, 0, ptr(total_dev), ptr(prep), prep.numel(), s)
    m = int(total_dev[:8].view(torch.int64).item())
    gauss_ids = torch.empty(m, dtype=torch.int32, device=dev)
    offsets = torch.empty(tx * ty + 1, dtype=torch.int32, device=dev)
    ebytes = L.mg_bin_emit_scratch_bytes(n, m, tx * ty)
    emit = ws.get("emit", ebytes, dev)
    _lib.call("mg_bin_emit", ptr(uv), ptr(rxy), ptr(conic), ptr(opacity), n, m, W, H, tile, 0,
              ptr(prep), ptr(gauss_ids), ptr(offsets), ptr(emit), emit.numel(), s)
    return gauss_ids, offsets, tx


# ------------------------------------------------------------------ raster

def tile_order(tile_offsets: torch.Tensor, work: torch.Tensor | None = None) -> torch.Tensor:
    """Tile ids heaviest first: by `work` (e.g. the forward's tile walk
    lengths) when given, else by list length."""
    n_tiles = tile_offsets.numel() - 1
    order = torch.empty(n_tiles, dtype=torch.int32, device=tile_offsets.device)
    _lib.call("mg_tile_order", ptr(tile_offsets), ptr(work), n_tiles, ptr(order), _lib.stream())
    return order


class RasterState:
    """What one view's forward leaves for its backward: the packed splat
    records and the rasteriser scratch (walk lengths, checkpoints)."""

    def __init__(self, splats: torch.Tensor, scratch: torch.Tensor, m: int, W: int, H: int,
                 tile: int):
        self.splats, self.scratch, self.m = splats, scratch, m
        self.W, self.H, self.tile = W, H, tile


def pack_splats(uv, conic, opacity, color) -> torch.Tensor:
    """(N, 12) packed records the rasterisers read (mg_pack_splats)."""
    for t, w in ((uv, "uv"), (conic, "conic"), (opacity, "opacity"), (color, "color")):
        _check(t, w)
    n = uv.shape[0]
    splats = _empty((n, _lib.SPLAT_FLOATS), uv)
    _lib.call("mg_pack_splats", ptr(uv), ptr(conic), ptr(opacity), ptr(color), n, ptr(splats),
              None, _lib.stream())
    return splats


def raster_scratch(W: int, H: int, tile: int, m: int, device) -> torch.Tensor:
    nbytes = _lib.load().mg_raster_scratch_bytes(W, H, tile, m)
    if nbytes == 0:
        raise RuntimeError(f"rasteriser scratch: bad size arguments W={W} H={H} tile={tile} "
                           f"m={m}")
    return torch.empty(nbytes, dtype=torch.uint8, device=device)


def _bg_arg(background):
    if background is None:
        return None, None
    bg = (_lib.C.c_float * 3)(*[float(x) for x in background])
    return bg, _lib.C.cast(bg, _lib.C.c_void_p)


def rasterize_forward(uv, conic, opacity, color, gauss_ids, tile_offsets, W, H, tile, tiles_x,
                      background=None, tile_work_out=None, state_out: list | None = None):
    """-> [rgb (H,W,3), alpha (H,W), T (H,W), n_contrib (H,W) int32 stop index]
    (rasterize.mm:79-113). `background` (3 floats) folds the reference's
    blend (metal_backend.py:539-541) into the kernel. `tile_work_out`
    (n_tiles int32), when given, receives each tile's walk length. When
    `state_out` is a list, the view's RasterState is appended to it for
    rasterize_backward_packed."""
    for t, w in ((uv, "uv"), (conic, "conic"), (opacity, "opacity"), (color, "color")):
        _check(t, w)
    _check(gauss_ids, "gauss_ids", torch.int32)
    _check(tile_offsets, "tile_offsets", torch.int32)
    rgb = _empty((H, W, 3), uv)
    alpha = _empty((H, W), uv)
    T = _empty((H, W), uv)
    stop = _empty((H, W), uv, torch.int32)
    m = gauss_ids.numel()  # the lists index into gauss_ids: no host read needed
    splats = pack_splats(uv, conic, opacity, color)
    scratch = raster_scratch(W, H, tile, m, uv.device)
    _bg, bgp = _bg_arg(background)
    _lib.call("mg_rasterize_forward", ptr(splats), ptr(gauss_ids), ptr(tile_offsets), m, W, H,
              tile, tiles_x, bgp, ptr(rgb), ptr(alpha), ptr(T), ptr(stop), ptr(tile_work_out),
              ptr(scratch), scratch.numel(), _lib.stream())
    if state_out is not None:
        state_out.append(RasterState(splats, scratch, m, W, H, tile))
    return [rgb, alpha, T, stop]


def rasterize_backward_packed(uv, conic, opacity, color, gauss_ids, tile_offsets, final_T,
                              n_contrib, grad_rgb, grad_alpha, W, H, tile, tiles_x,
                              want_absgrad, background=None, alpha=None, grad2d=None,
                              state: RasterState | None = None, rgb=None):
    """Backward into the packed (N, 12) record; accumulates into `grad2d` when
    given, else into a fresh zeroed one. With the forward's `state` (and its
    `rgb`, `alpha`), long walks are split into segments that start from the
    forward's checkpoints; without, every warp block walks its whole list.
    Returns grad2d."""
    n = uv.shape[0]
    if grad2d is None:
        grad2d = torch.zeros((n, G2D_STRIDE), dtype=F32, device=uv.device)
    grad_rgb = grad_rgb.contiguous()
    grad_alpha = None if grad_alpha is None else grad_alpha.contiguous()
    _bg, bgp = _bg_arg(background)
    segmented = state is not None
    if segmented:
        if rgb is None or alpha is None:
            raise RuntimeError("rasterize_backward: the forward state needs its rgb and alpha")
        if (state.W, state.H, state.tile) != (W, H, tile):
            raise RuntimeError("rasterize_backward: forward state is for another view")
        splats, scratch, m = state.splats, state.scratch, state.m
    else:
        m = gauss_ids.numel()
        splats = pack_splats(uv, conic, opacity, color)
        scratch = raster_scratch(W, H, tile, m, uv.device)
    _lib.call("mg_rasterize_backward", ptr(splats), ptr(gauss_ids), ptr(tile_offsets), m,
              ptr(rgb) if segmented else None, ptr(alpha), ptr(final_T), ptr(n_contrib),
              ptr(grad_rgb), ptr(grad_alpha), W, H, tile, tiles_x, bgp, int(bool(want_absgrad)),
              n, ptr(grad2d), int(segmented), ptr(scratch), scratch.numel(), _lib.stream())
    return grad2d


def rasterize_backward(uv, conic, opacity, color, gauss_ids, tile_offsets, final_T, n_contrib,
                       grad_rgb, grad_alpha, W, H, tile, tiles_x, want_absgrad):
    """-> [d_uv (N,2), d_conic (N,3), d_opacity (N,), d_color (N,3), d_absuv]
    (rasterize.mm:147-194). The first four are row views into one packed
    gradient record per Gaussian; d_absuv is (N,) with absgrad, else (1,)."""
    g = rasterize_backward_packed(uv, conic, opacity, color, gauss_ids, tile_offsets, final_T,
                                  n_contrib, grad_rgb, grad_alpha, W, H, tile, tiles_x,
                                  want_absgrad)
    d_abs = g[:, G2D_ABSUV] if want_absgrad else torch.zeros(1, dtype=F32, device=uv.device)
    return [g[:, G2D_UV:G2D_UV + 2], g[:, G2D_CONIC:G2D_CONIC + 3], g[:, G2D_OPACITY],
            g[:, G2D_COLOR:G2D_COLOR + 3], d_abs]


def pack_intersections(uv, conic, opacity, color, gauss_ids):
    """-> [p_xy_opac (M,3), p_conic (M,3), p_rgb (M,3)] (rasterize.mm:115-145)."""
    m = gauss_ids.numel()
    a, b, c = _empty((m, 3), uv), _empty((m, 3), uv), _empty((m, 3), uv)
    _lib.call("mg_pack_intersections", ptr(uv), ptr(conic), ptr(opacity), ptr(color),
              ptr(gauss_ids), m, ptr(a), ptr(b), ptr(c), _lib.stream())
    return [a, b, c]


# ------------------------------------------------------------------ optimisers

def adam_step(p, g, m, v, lr, b1, b2, eps, step):
    """In-place torch.optim.Adam step on flat tensors (rasterize.mm:329-360)."""
    for t, w in ((p, "adam tensor"), (g, "adam tensor"), (m, "adam tensor"), (v, "adam tensor")):
        _check(t, w)
    if not (g.numel() == p.numel() == m.numel() == v.numel()):
        raise RuntimeError("adam_step: parameter/grad/moment numel mismatch")
    bc1 = 1.0 - b1 ** step
    sq = math.sqrt(1.0 - b2 ** step)
    _lib.call("mg_adam_step", ptr(p), ptr(g), ptr(m), ptr(v), p.numel(), lr, b1, b2, eps, bc1, sq,
              _lib.stream())


def selective_adam_step(p, g, m, v, steps, visible_u8, lr, b1, b2, eps):
    """Row-selective Adam on a (rows, ...) parameter; advances steps after."""
    rows = p.shape[0]
    width = p.numel() // rows if rows else 0
    nvis = visible_u8.numel()
    _lib.call("mg_selective_adam_step", ptr(p), ptr(g), ptr(m), ptr(v), ptr(steps),
              ptr(visible_u8), nvis, rows, width, lr, b1, b2, eps, _lib.stream())
    _lib.call("mg_selective_adam_advance_steps", ptr(steps), ptr(visible_u8), nvis, rows,
              _lib.stream())


# ---------------------------------------------------------------------- SSIM

def ssim_tail_forward(b, H, W):
    _check(b, "blurred stack")
    if b.numel() != 15 * H * W:
        raise RuntimeError("ssim_tail_forward: expected 15*H*W")
    out = torch.empty((1, 3, H, W), dtype=F32, device=b.device)
    _lib.call("mg_ssim_tail_forward", ptr(b), H, W, ptr(out), _lib.stream())
    return out


def ssim_tail_backward(b, gout, H, W):
    _check(b, "blurred stack"), _check(gout, "grad")
    gb = torch.empty_like(b)
    _lib.call("mg_ssim_tail_backward", ptr(b), ptr(gout), H, W, ptr(gb), _lib.stream())
    return gb


def ssim_stack_blur_h(x, y, w, H, W):
    _check(x, "x"), _check(y, "y"), _check(w, "weights")
    if x.numel() != 3 * H * W or y.numel() != x.numel():
        raise RuntimeError("expected (H,W,3)")
    out = torch.empty((1, 15, H, W), dtype=F32, device=x.device)
    _lib.call("mg_ssim_stack_blur_h", ptr(x), ptr(y), ptr(w), H, W, ptr(out), _lib.stream())
    return out


def ssim_blur15(src, w, dir, H, W):
    _check(src, "src"), _check(w, "weights")
    out = torch.empty_like(src)
    _lib.call("mg_ssim_blur15", ptr(src), ptr(w), int(dir), H, W, ptr(out), _lib.stream())
    return out


def ssim_chain_backward(x, y, d_stack, H, W):
    _check(x, "x"), _check(y, "y"), _check(d_stack, "d_stack")
    d_x = torch.empty_like(x)
    _lib.call("mg_ssim_chain_backward", ptr(x), ptr(y), ptr(d_stack), H, W, ptr(d_x),
              _lib.stream())
    return d_x


def l1_ssim_loss(x, y, w, w_l1=0.8, w_ssim=0.2, scale=1.0, grad_out=None, loss_out=None):
    """Fused w_l1*L1 + w_ssim*(1-SSIM) forward+backward for one (H,W,3) image.
    Returns (loss_dev (1,) accumulated into loss_out when given, grad_x)."""
    _check(x, "x"), _check(y, "y"), _check(w, "weights")
    H, W = x.shape[0], x.shape[1]
    grad = torch.empty_like(x) if grad_out is None else grad_out
    loss = torch.zeros(1, dtype=F32, device=x.device) if loss_out is None else loss_out
    nbytes = _lib.load().mg_l1_ssim_scratch_bytes(H, W)
    scratch = torch.empty(nbytes, dtype=torch.uint8, device=x.device)
    _lib.call("mg_l1_ssim_loss", ptr(x), ptr(y), ptr(w), H, W, w_l1, w_ssim, scale, ptr(grad),
              ptr(loss), ptr(scratch), nbytes, _lib.stream())
    return loss, grad


def device_error() -> int:
    """Reads and clears the device error word (0 = none); synchronises."""
    return _lib.device_error()
