"""CPU oracle -- TEST INFRASTRUCTURE ONLY.

A plain-C restatement (mg_oracle.c) of nandometzger/metal-gauss's training hot
path as its Metal kernels define it, wrapped for numpy. Only tests/,
__graft_entry__.smoke() and bench.py's CPU-baseline leg import this package,
always as the checker; the product (metal_gauss_b200) never imports, links or
calls it and fails loudly when its CUDA library is missing.

Parity of this restatement with the reference is pinned against fixtures made
by the reference's own code (tests/golden/make_golden.py,
tests/test_oracle_golden.py).
"""

from __future__ import annotations

import ctypes as C
import math
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
SRC = HERE / "mg_oracle.c"
LIB = HERE / "libmg_oracle.so"

CFLAGS = ["-O2", "-fopenmp", "-ffp-contract=off", "-fno-fast-math", "-fPIC", "-shared",
          "-std=c11", "-I", str(ROOT / "include")]

G2D_STRIDE, G2D_UV, G2D_OPACITY, G2D_ABSUV, G2D_CONIC, G2D_COLOR = 12, 0, 2, 3, 4, 8


def _compiler() -> str:
    """A C compiler that can link OpenMP (some images point $CC at a wrapper
    without libgomp's spec file, so each candidate is probed)."""
    import shutil
    import tempfile
    cands = [os.environ.get("MG_ORACLE_CC"), "/usr/bin/gcc", shutil.which("gcc"),
             os.environ.get("CC"), shutil.which("cc")]
    with tempfile.TemporaryDirectory() as td:
        probe = Path(td) / "p.c"
        probe.write_text("int main(void){return 0;}\n")
        for c in cands:
            if not c or not Path(c).exists():
                continue
            r = subprocess.run([c, "-fopenmp", str(probe), "-o", str(Path(td) / "p")],
                               capture_output=True)
            if r.returncode == 0:
                return c
    raise RuntimeError("no C compiler with OpenMP support found for the oracle")


def build(force: bool = False) -> Path:
    """Compile libmg_oracle.so with gcc (no-op when up to date)."""
    hdr = ROOT / "include" / "mg_b200.h"
    if (not force and LIB.exists() and LIB.stat().st_mtime >= SRC.stat().st_mtime
            and LIB.stat().st_mtime >= hdr.stat().st_mtime):
        return LIB
    cc = _compiler()
    tmp = LIB.with_suffix(".so.tmp")
    subprocess.run([cc, *CFLAGS, "-o", str(tmp), str(SRC), "-lm"], check=True)
    os.replace(tmp, LIB)
    return LIB


class Camera(C.Structure):
    _fields_ = [("viewmat", C.c_float * 16), ("fx", C.c_float), ("fy", C.c_float),
                ("cx", C.c_float), ("cy", C.c_float), ("cam_center", C.c_float * 4),
                ("width", C.c_int32), ("height", C.c_int32), ("near_plane", C.c_float),
                ("far_plane", C.c_float), ("blur", C.c_float), ("max_radius", C.c_float)]


class ShLayout(C.Structure):
    _fields_ = [("stride_dc", C.c_int32), ("stride_rest", C.c_int32),
                ("offset_rest", C.c_int32), ("unused", C.c_int32)]


FUSED = (16, 16, 1)
SPLIT = (1, 15, 0)

_lib = None


def lib():
    global _lib
    if _lib is None:
        build()
        L = C.CDLL(str(LIB))
        vp, i64, i32, f32 = C.c_void_p, C.c_int64, C.c_int32, C.c_float
        L.mgo_preprocess_forward.argtypes = [vp, vp, vp, vp, vp, ShLayout, vp, C.POINTER(Camera),
                                             i32, i64, vp, vp, vp, vp, vp, vp]
        L.mgo_preprocess_backward.argtypes = [vp, vp, vp, vp, vp, ShLayout, vp, i64, vp, i64, vp,
                                              i64, vp, C.POINTER(Camera), i32, i64, vp, vp, vp,
                                              vp, vp]
        L.mgo_bin_count.argtypes = [vp, vp, vp, vp, vp, i64, i32, i32, i32, i32, i32, vp]
        L.mgo_bin_write.argtypes = [vp, vp, vp, vp, vp, vp, vp, i64, i32, i32, i32, i32, i32,
                                    vp, vp]
        L.mgo_sort_pairs_u64.argtypes = [vp, vp, i64, i32]
        L.mgo_tile_ranges.argtypes = [vp, i64, i32, vp]
        L.mgo_rasterize_forward.argtypes = [vp, vp, vp, vp, vp, vp, i32, i32, i32, vp, vp, vp,
                                            vp, vp]
        L.mgo_rasterize_backward.argtypes = [vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, i32, i32,
                                             i32, vp, vp, i32, vp]
        L.mgo_adam_step.argtypes = [vp, vp, vp, vp, i64, f32, f32, f32, f32, f32, f32]
        L.mgo_selective_adam_step.argtypes = [vp, vp, vp, vp, vp, vp, i64, i64, i64, f32, f32,
                                              f32, f32]
        L.mgo_l1_ssim_loss.argtypes = [vp, vp, vp, i32, i32, f32, f32, vp]
        L.mgo_l1_ssim_loss.restype = C.c_double
        _lib = L
    return _lib


def _p(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


# ------------------------------------------------------------------ cameras

def camera(viewmat, K, W: int, H: int, near: float = 0.01, far: float = 100.0,
           blur: float = 0.3, max_radius_frac: float = 1.0) -> Camera:
    """The reference's per-view constants (metal_backend.py:447-501):
    cam_center = -R^T t is formed in float32 like the reference's torch op."""
    vm = _f32(viewmat).reshape(4, 4)
    K = np.asarray(K, dtype=np.float64)
    cc = -(vm[:3, :3].T.astype(np.float32) @ vm[:3, 3].astype(np.float32))
    cam = Camera()
    cam.viewmat[:] = [float(x) for x in vm.reshape(-1)]
    cam.fx, cam.fy, cam.cx, cam.cy = float(K[0, 0]), float(K[1, 1]), float(K[0, 2]), float(K[1, 2])
    cam.cam_center[:] = [float(cc[0]), float(cc[1]), float(cc[2]), 0.0]
    cam.width, cam.height = int(W), int(H)
    cam.near_plane, cam.far_plane, cam.blur = near, far, blur
    cam.max_radius = float(np.float32(max_radius_frac * max(W, H)))
    return cam


def sh_layout(sh: np.ndarray, sh_rest: np.ndarray | None):
    if sh_rest is None or sh_rest is sh:
        return ShLayout(*FUSED, 0)
    return ShLayout(*SPLIT, 0)


def pad_sh(sh: np.ndarray | None, sh_rest: np.ndarray | None):
    """Zero-pads to 16 (fused) or 1 + 15 (split) bands (metal_backend.py:482-497)."""
    if sh is None:
        return None, None
    sh = _f32(sh)
    if sh_rest is None:
        if sh.shape[1] < 16:
            sh = np.concatenate([sh, np.zeros((sh.shape[0], 16 - sh.shape[1], 3), np.float32)], 1)
        return sh, sh
    rest = _f32(sh_rest)
    if rest.shape[1] < 15:
        rest = np.concatenate([rest, np.zeros((rest.shape[0], 15 - rest.shape[1], 3),
                                              np.float32)], 1)
    return sh, rest


# --------------------------------------------------------------- preprocess

def preprocess_forward(means, quats, scales, sh, sh_rest, opacities, cam: Camera,
                       sh_degree: int) -> dict:
    means, quats, scales, opac = map(_f32, (means, quats, scales, opacities))
    n = means.shape[0]
    out = dict(uv=np.zeros((n, 2), np.float32), conic=np.zeros((n, 3), np.float32),
               depth=np.zeros(n, np.float32), rxy=np.zeros((n, 2), np.float32),
               valid=np.zeros(n, np.int32), color=np.zeros((n, 3), np.float32))
    sh_p, rest_p = pad_sh(sh, sh_rest)
    lay = sh_layout(sh_p, rest_p) if sh_p is not None else ShLayout(*FUSED, 0)
    lib().mgo_preprocess_forward(_p(means), _p(quats), _p(scales), _p(sh_p), _p(rest_p), lay,
                                 _p(opac), C.byref(cam), sh_degree if sh_p is not None else -1,
                                 n, _p(out["uv"]), _p(out["conic"]), _p(out["depth"]),
                                 _p(out["rxy"]), _p(out["valid"]), _p(out["color"]))
    return out


def preprocess_backward(means, quats, scales, sh, sh_rest, d_uv, d_conic, d_color, valid,
                        cam: Camera, sh_degree: int) -> dict:
    means, quats, scales = map(_f32, (means, quats, scales))
    n = means.shape[0]
    d_uv, d_conic = _f32(d_uv), _f32(d_conic)
    valid = np.ascontiguousarray(valid, dtype=np.int32)
    sh_p, rest_p = pad_sh(sh, sh_rest)
    out = dict(means=np.zeros((n, 3), np.float32), quats=np.zeros((n, 4), np.float32),
               scales=np.zeros((n, 3), np.float32))
    if sh_p is not None and d_color is not None:
        lay = sh_layout(sh_p, rest_p)
        d_sh = np.zeros_like(sh_p)
        d_rest = d_sh if rest_p is sh_p else np.zeros_like(rest_p)
        dcol = _f32(d_color)
        deg = sh_degree
    else:
        lay, d_sh, d_rest, dcol, deg = ShLayout(*FUSED, 0), None, None, None, -1
    lib().mgo_preprocess_backward(_p(means), _p(quats), _p(scales), _p(sh_p), _p(rest_p), lay,
                                  _p(d_uv), d_uv.shape[1], _p(d_conic), d_conic.shape[1],
                                  _p(dcol), 3, _p(valid), C.byref(cam), deg, n,
                                  _p(out["means"]), _p(out["quats"]), _p(out["scales"]),
                                  _p(d_sh), _p(d_rest))
    out["sh"], out["sh_rest"] = d_sh, d_rest
    return out


def antialias_scale(conic: np.ndarray, blur: float) -> np.ndarray:
    """sqrt(det_before/det_after) from the conic (metal_backend.py:367-393), fp32."""
    c = _f32(conic)
    cxx, cxy, cyy = c[:, 0], c[:, 1], c[:, 2]
    det_conic = np.maximum(cxx * cyy - cxy * cxy, np.float32(1e-12))
    det_after = np.float32(1.0) / det_conic
    a, b, cc = cyy * det_after, -cxy * det_after, cxx * det_after
    det_before = (a - np.float32(blur)) * (cc - np.float32(blur)) - b * b
    return np.sqrt(np.clip(np.maximum(det_before, 0) / det_after, 0, 1)).astype(np.float32)


# ---------------------------------------------------------------- 3D filter

def compute_3d_filter(means, views, near=0.2, margin=0.15) -> np.ndarray:
    """Mip-Splatting's 3D filter (metal_gauss/mipfilter.py:30-76) in float32:
    views are (K (3,3), viewmat (4,4), W, H). The smallest camera depth among
    the cameras whose margin-widened frame holds the projected mean in front
    of `near`; unseen Gaussians take the largest such depth (1 when nothing
    is seen); then depth / max focal * sqrt(0.2)."""
    m = _f32(means)
    n = m.shape[0]
    dist = np.full(n, np.inf, np.float32)
    seen = np.zeros(n, bool)
    focal = 0.0
    for K, vm, W, H in views:
        K, vm = _f32(K), _f32(vm)
        pc = (m @ vm[:3, :3].T + vm[:3, 3]).astype(np.float32)
        z = pc[:, 2]
        fx, fy, cx, cy = (np.float32(K[0, 0]), np.float32(K[1, 1]), np.float32(K[0, 2]),
                          np.float32(K[1, 2]))
        zc = np.maximum(z, np.float32(1e-6))
        u = fx * pc[:, 0] / zc + cx
        w = fy * pc[:, 1] / zc + cy
        mW, mH = np.float32(margin * W), np.float32(margin * H)
        inview = ((z > np.float32(near)) & (u > -mW) & (u < np.float32((1.0 + margin) * W))
                  & (w > -mH) & (w < np.float32((1.0 + margin) * H)))
        dist = np.where(inview, np.minimum(dist, z), dist).astype(np.float32)
        seen |= inview
        focal = max(focal, float(K[0, 0]), float(K[1, 1]))
    if seen.any():
        dist[~seen] = dist[seen].max()
    else:
        dist[:] = 1.0
    if focal <= 0.0:
        focal = 1.0
    return ((dist / np.float32(focal)) * np.float32(0.2 ** 0.5)).astype(np.float32)


def apply_3d_filter(scales, opac, filter_3d):
    """(sqrt(s^2 + f^2), op * sqrt(clamp(prod s^2 / prod (s^2 + f^2), 0, 1)))
    (mipfilter.py:79-93), float32."""
    s, o, f = _f32(scales), _f32(opac), _f32(filter_3d)
    s2 = s * s
    s2f = s2 + (f * f)[:, None]
    coef = np.sqrt(np.clip((s2[:, 0] * s2[:, 1] * s2[:, 2]) /
                           (s2f[:, 0] * s2f[:, 1] * s2f[:, 2]), 0, 1))
    return np.sqrt(s2f).astype(np.float32), (o * coef).astype(np.float32)


def apply_3d_filter_backward(scales, opac, filter_3d, d_scales_out, d_opac_out):
    """Gradients of apply_3d_filter's outputs carried to (scales, opacities),
    the filter held constant: d s_i = g_si s_i / s'_i + g_o op coef f^2 /
    (s_i (s_i^2 + f^2)), d op = g_o coef. Computed in float64."""
    s, o, f = (np.asarray(x, np.float64) for x in (scales, opac, filter_3d))
    gs, go = np.asarray(d_scales_out, np.float64), np.asarray(d_opac_out, np.float64)
    s2 = s * s
    s2f = s2 + (f * f)[:, None]
    coef = np.sqrt(np.clip(s2.prod(1) / s2f.prod(1), 0, 1))
    ds = gs * s / np.sqrt(s2f) + (go * o * coef)[:, None] * (f * f)[:, None] / (s * s2f)
    return ds.astype(np.float32), (go * coef).astype(np.float32)


# -------------------------------------------------------------- MCMC (mcmc.py)

def _sigmoid32(x):
    x = _f32(x)
    with np.errstate(over="ignore"):  # exp(-x) = inf gives the exact limit 0
        return (np.float32(1) / (np.float32(1) + np.exp(-x))).astype(np.float32)


def _mcmc_split(o, n):
    """(logit of 1 - (1-o)^(1/n), log of the binomial scale ratio), float32
    (mcmc.py:43-50, :83-86)."""
    o = _f32(o)
    nf = np.asarray(n, np.float32)
    o_new = (np.float32(1) - np.maximum(np.float32(1) - o, np.float32(1e-6)) **
             (np.float32(1) / nf)).astype(np.float32)
    logit = np.log(np.clip(o_new, 1e-6, 1 - 1e-6) / np.maximum(1 - o_new, np.float32(1e-6)))
    denom = np.maximum(np.maximum(nf, 1) * np.maximum(o_new, np.float32(1e-6)), np.float32(1e-6))
    ratio = np.sqrt(np.clip(o_new / denom, 0.05, 1.0))
    return logit.astype(np.float32), np.log(ratio).astype(np.float32)


def mcmc_relocate(params: dict, picks, dead_thresh=0.005, active=None):
    """relocate (mcmc.py:52-104) with its draws given: returns (new params,
    rows whose optimizer state is reset). `picks` are row indices, one per
    dead row in increasing row order."""
    p = {k: np.array(v, dtype=np.float32, copy=True) for k, v in params.items()}
    n_act = p["logit_opac"].shape[0] if active is None else active
    opac = _sigmoid32(p["logit_opac"][:n_act])
    dead = np.nonzero(opac < np.float32(dead_thresh))[0]
    pick = np.asarray(picks, np.int64)
    if dead.size == 0:
        return p, np.zeros(0, np.int64)
    counts = np.clip(np.bincount(pick, minlength=n_act), 1, 51)
    logit_new, log_ratio = _mcmc_split(opac[pick], counts[pick])
    for k in p:
        if k not in ("logit_opac", "log_scales"):
            p[k][dead] = p[k][pick]
    p["log_scales"][dead] = p["log_scales"][pick] + log_ratio[:, None]
    p["logit_opac"][dead] = logit_new
    uniq = np.unique(pick)
    lu, ru = _mcmc_split(opac[uniq], counts[uniq])
    p["logit_opac"][uniq] = lu
    p["log_scales"][uniq] += ru[:, None]
    return p, np.concatenate([dead, uniq])


def mcmc_grow(params: dict, picks, target: int, active: int):
    """grow (mcmc.py:124-163) with its draws given: (new params, reset rows)."""
    p = {k: np.array(v, dtype=np.float32, copy=True) for k, v in params.items()}
    target = min(target, p["logit_opac"].shape[0])
    if target <= active:
        return p, np.zeros(0, np.int64)
    opac = _sigmoid32(p["logit_opac"][:active])
    pick = np.asarray(picks, np.int64)
    dst = np.arange(active, target)
    counts = np.clip(np.bincount(pick, minlength=active), 1, 51) + 1
    logit_new, log_ratio = _mcmc_split(opac[pick], counts[pick])
    for k in p:
        if k not in ("logit_opac", "log_scales"):
            p[k][dst] = p[k][pick]
    p["log_scales"][dst] = p["log_scales"][pick] + log_ratio[:, None]
    p["logit_opac"][dst] = logit_new
    uniq = np.unique(pick)
    lu, ru = _mcmc_split(opac[uniq], counts[uniq])
    p["logit_opac"][uniq] = lu
    p["log_scales"][uniq] += ru[:, None]
    return p, np.concatenate([dst, uniq])


def mcmc_add_noise(params: dict, eps, lr_means, weight=4e4, opacity_gate=0.005, active=None):
    """add_noise (mcmc.py:166-192) with its normal draws `eps` (N,3) given:
    the new means."""
    m = np.array(params["means"], dtype=np.float32, copy=True)
    n = m.shape[0] if active is None else active
    opac = _sigmoid32(params["logit_opac"][:n])
    gate = _sigmoid32(np.float32(-100.0) * (opac - np.float32(opacity_gate)))
    e = _f32(eps)[:n] * np.exp(_f32(params["log_scales"][:n]))
    q = _f32(params["quats"][:n])
    q = q / np.maximum(np.linalg.norm(q, axis=1, keepdims=True), np.float32(1e-12))
    w, u = q[:, 0:1], q[:, 1:4]
    t = np.float32(2.0) * np.cross(u, e)
    world = e + w * t + np.cross(u, t)
    m[:n] += world * gate[:, None] * np.float32(lr_means) * np.float32(weight)
    return m


# ------------------------------------------------------------------ binning

def tiles_of(W: int, H: int, tile: int) -> tuple[int, int]:
    return math.ceil(W / tile), math.ceil(H / tile)


def bin_count(uv, rxy, conic, opacity, valid, W, H, tile) -> np.ndarray:
    tx, ty = tiles_of(W, H, tile)
    uv, rxy, conic, opacity = map(_f32, (uv, rxy, conic, opacity))
    valid = np.ascontiguousarray(valid, dtype=np.int32)
    counts = np.zeros(uv.shape[0], np.int32)
    lib().mgo_bin_count(_p(uv), _p(rxy), _p(conic), _p(opacity), _p(valid), uv.shape[0], W, H,
                        tile, tx, ty, _p(counts))
    return counts


def bin_write(uv, rxy, conic, opacity, valid, depth, offsets, total, W, H, tile):
    tx, ty = tiles_of(W, H, tile)
    uv, rxy, conic, opacity, depth = map(_f32, (uv, rxy, conic, opacity, depth))
    valid = np.ascontiguousarray(valid, dtype=np.int32)
    offs = np.ascontiguousarray(offsets, dtype=np.int64)
    keys = np.zeros(total, np.uint64)
    ids = np.zeros(total, np.int32)
    lib().mgo_bin_write(_p(uv), _p(rxy), _p(conic), _p(opacity), _p(valid), _p(depth), _p(offs),
                        uv.shape[0], W, H, tile, tx, ty, _p(keys), _p(ids))
    return keys, ids


def build_tile_lists(uv, rxy, conic, opacity, valid, depth, W, H, tile):
    """(gauss_ids, tile_offsets, keys) in the order of a stable sort on
    (tile_id << 32 | depth_bits) keys emitted in Gaussian order."""
    tx, ty = tiles_of(W, H, tile)
    counts = bin_count(uv, rxy, conic, opacity, valid, W, H, tile).astype(np.int64)
    offs = np.cumsum(counts) - counts
    total = int(counts.sum())
    keys, ids = bin_write(uv, rxy, conic, opacity, valid, depth, offs, total, W, H, tile)
    bits = max(1, math.ceil(math.log2(max(tx * ty, 2)))) + 32
    lib().mgo_sort_pairs_u64(_p(keys), _p(ids), total, bits)
    offsets = np.zeros(tx * ty + 1, np.int32)
    lib().mgo_tile_ranges(_p(keys), total, tx * ty, _p(offsets))
    return ids, offsets, keys


# ------------------------------------------------------------------- raster

def rasterize_forward(uv, conic, opacity, color, ids, offsets, W, H, tile, background=None):
    uv, conic, opacity, color = map(_f32, (uv, conic, opacity, color))
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    offsets = np.ascontiguousarray(offsets, dtype=np.int32)
    rgb = np.zeros((H, W, 3), np.float32)
    alpha = np.zeros((H, W), np.float32)
    T = np.ones((H, W), np.float32)
    stop = np.zeros((H, W), np.int32)
    bg = None if background is None else _f32(background)
    lib().mgo_rasterize_forward(_p(uv), _p(conic), _p(opacity), _p(color), _p(ids), _p(offsets),
                                W, H, tile, _p(bg), _p(rgb), _p(alpha), _p(T), _p(stop))
    return rgb, alpha, T, stop


def rasterize_backward(uv, conic, opacity, color, ids, offsets, T, stop, grad_rgb, grad_alpha,
                       W, H, tile, background=None, alpha=None, want_absgrad=False):
    uv, conic, opacity, color = map(_f32, (uv, conic, opacity, color))
    n = uv.shape[0]
    g2d = np.zeros((n, G2D_STRIDE), np.float32)
    bg = None if background is None else _f32(background)
    lib().mgo_rasterize_backward(
        _p(uv), _p(conic), _p(opacity), _p(color), _p(np.ascontiguousarray(ids, np.int32)),
        _p(np.ascontiguousarray(offsets, np.int32)), _p(_f32(T)),
        _p(np.ascontiguousarray(stop, np.int32)), _p(_f32(grad_rgb)),
        _p(None if grad_alpha is None else _f32(grad_alpha)), W, H, tile, _p(bg),
        _p(None if alpha is None else _f32(alpha)), int(bool(want_absgrad)), _p(g2d))
    return g2d


# ------------------------------------------------------------ whole render

def render(means, quats, scales, opacities, sh, K, viewmat, W, H, sh_degree=3, tile=16,
           near=0.01, far=100.0, background=(0.0, 0.0, 0.0), colors=None,
           max_radius_frac=1.0, sh_rest=None, antialias=False):
    """The reference's render() (metal_backend.py:396-559) on the CPU: returns
    (rgb, alpha, state) where state holds every intermediate for backward()."""
    cam = camera(viewmat, K, W, H, near, far, 0.3, max_radius_frac)
    explicit = colors is not None
    pre = preprocess_forward(means, quats, scales, None if explicit else sh,
                             None if explicit else sh_rest, opacities, cam, sh_degree)
    color = _f32(colors) if explicit else pre["color"]
    opac = _f32(opacities)
    aa = antialias_scale(pre["conic"], 0.3) if antialias else None
    if aa is not None:
        opac = (opac * aa).astype(np.float32)
    ids, offsets, keys = build_tile_lists(pre["uv"], pre["rxy"], pre["conic"], opac, pre["valid"],
                                          pre["depth"], W, H, tile)
    bg = None if background is None else _f32(background)
    rgb, alpha, T, stop = rasterize_forward(pre["uv"], pre["conic"], opac, color, ids, offsets,
                                            W, H, tile, bg)
    state = dict(cam=cam, pre=pre, color=color, opac=opac, ids=ids, offsets=offsets, keys=keys,
                 T=T, stop=stop, alpha=alpha, bg=bg, W=W, H=H, tile=tile, explicit=explicit,
                 means=means, quats=quats, scales=scales, sh=sh, sh_rest=sh_rest,
                 sh_degree=sh_degree, antialias=antialias)
    return rgb, alpha, state


def render_backward(state: dict, grad_rgb, grad_alpha=None, want_absgrad=False) -> dict:
    """Gradients w.r.t. the render() inputs (means, quats, scales, opacities,
    sh/sh_rest or colors) for the given output gradients. Antialiasing is
    forward-only here."""
    if state["antialias"]:
        raise NotImplementedError("oracle backward through antialias_scale")
    s, pre = state, state["pre"]
    W, H, tile = s["W"], s["H"], s["tile"]
    g2d = rasterize_backward(pre["uv"], pre["conic"], s["opac"], s["color"], s["ids"],
                             s["offsets"], s["T"], s["stop"], grad_rgb, grad_alpha, W, H, tile,
                             s["bg"], s["alpha"], want_absgrad)
    d_uv = np.ascontiguousarray(g2d[:, G2D_UV:G2D_UV + 2])
    d_conic = np.ascontiguousarray(g2d[:, G2D_CONIC:G2D_CONIC + 3])
    d_color = np.ascontiguousarray(g2d[:, G2D_COLOR:G2D_COLOR + 3])
    out = preprocess_backward(s["means"], s["quats"], s["scales"],
                              None if s["explicit"] else s["sh"],
                              None if s["explicit"] else s["sh_rest"], d_uv, d_conic,
                              None if s["explicit"] else d_color, pre["valid"], s["cam"],
                              s["sh_degree"])
    out["opacities"] = np.ascontiguousarray(g2d[:, G2D_OPACITY])
    out["uv"] = d_uv
    out["conic"] = d_conic
    out["absgrad"] = np.ascontiguousarray(g2d[:, G2D_ABSUV])
    if s["explicit"]:
        out["colors"] = d_color
    return out


# -------------------------------------------------------------- optimisers

def adam_step(p, g, m, v, lr, b1, b2, eps, step):
    bc1 = 1.0 - b1 ** step
    sq = math.sqrt(1.0 - b2 ** step)
    lib().mgo_adam_step(_p(p), _p(g), _p(m), _p(v), p.size, lr, b1, b2, eps, bc1, sq)


def selective_adam_step(p, g, m, v, steps, visible, lr, b1=0.9, b2=0.999, eps=1e-15):
    rows = p.shape[0]
    width = p.size // rows if rows else 0
    vis = np.ascontiguousarray(visible, dtype=np.uint8)
    lib().mgo_selective_adam_step(_p(p), _p(g), _p(m), _p(v), _p(steps), _p(vis), vis.size,
                                  rows, width, lr, b1, b2, eps)


# -------------------------------------------------------------------- loss

def gaussian_window(size: int = 11, sigma: float = 1.5) -> np.ndarray:
    """train._gaussian_kernel's 1D window (train.py:38-49), in float32."""
    x = np.arange(size, dtype=np.float32) - np.float32(size // 2)
    g = np.exp(-(x * x) / np.float32(2 * sigma * sigma)).astype(np.float32)
    return (g / g.sum(dtype=np.float32)).astype(np.float32)


def l1_ssim_loss(x, y, w_l1=0.8, w_ssim=0.2, window=None, want_grad=True):
    x, y = _f32(x), _f32(y)
    H, W = x.shape[:2]
    w = gaussian_window() if window is None else _f32(window)
    grad = np.zeros_like(x) if want_grad else None
    loss = lib().mgo_l1_ssim_loss(_p(x), _p(y), _p(w), H, W, w_l1, w_ssim, _p(grad))
    return loss, grad
