"""ctypes binding of libmg_b200.so (the C ABI in include/mg_b200.h).

The library is built in-tree by build_native.py and loaded from
metal_gauss_b200/_native/. There is no fallback: if the library is missing or
fails to load, every entry point raises.
"""

from __future__ import annotations

import ctypes as C
import os
import threading
from pathlib import Path

import torch

from . import build_native

LIB_PATH = build_native.LIB

G2D_STRIDE = 12
G2D_UV, G2D_OPACITY, G2D_ABSUV, G2D_CONIC, G2D_COLOR = 0, 2, 3, 4, 8
SPLAT_FLOATS = 12        # MG_SPLAT_FLOATS: one packed splat record
ADAM_ROW_FACTORS_READY, ADAM_KEEP_STEPS = 1, 2   # mg_adam_multi flags
RASTER_SEGMENT = 256     # MG_RASTER_SEGMENT


class Camera(C.Structure):
    _fields_ = [("viewmat", C.c_float * 16), ("fx", C.c_float), ("fy", C.c_float),
                ("cx", C.c_float), ("cy", C.c_float), ("cam_center", C.c_float * 4),
                ("width", C.c_int32), ("height", C.c_int32), ("near_plane", C.c_float),
                ("far_plane", C.c_float), ("blur", C.c_float), ("max_radius", C.c_float)]


class ShLayout(C.Structure):
    _fields_ = [("stride_dc", C.c_int32), ("stride_rest", C.c_int32),
                ("offset_rest", C.c_int32), ("unused", C.c_int32)]


class AdamSegment(C.Structure):
    _fields_ = [("offset", C.c_int64), ("width", C.c_int32), ("lr", C.c_float),
                ("elem_begin", C.c_int64), ("elem_end", C.c_int64)]


class RowSegment(C.Structure):
    _fields_ = [("ptr", C.c_void_p), ("width", C.c_int32)]


class StepPrologue(C.Structure):
    """mg_step_prologue: the start of a training step folded into the
    multi-view projection (activations, optional 3D filter, gradient rows and
    the loss set to zero, visibility written)."""
    _fields_ = [("log_scales", C.c_void_p), ("logit_opac", C.c_void_p),
                ("filter_3d", C.c_void_p), ("act_scales", C.c_void_p),
                ("act_opac", C.c_void_p), ("out_scales", C.c_void_p),
                ("out_opac", C.c_void_p), ("zero", C.c_void_p * 4),
                ("zero_width", C.c_int32 * 4), ("zero_word", C.c_void_p)]


SH_FUSED = ShLayout(16, 16, 1, 0)
SH_SPLIT = ShLayout(1, 15, 0, 0)

vp, i64, i32, f32, sz = C.c_void_p, C.c_int64, C.c_int32, C.c_float, C.c_size_t
CAM = C.POINTER(Camera)

# name -> (restype, argtypes)
SIGNATURES = {
    "mg_last_error": (C.c_char_p, []),
    "mg_version": (C.c_int, []),
    "mg_launch_count": (C.c_uint64, []),
    "mg_preprocess_forward": (i32, [vp, vp, vp, vp, vp, ShLayout, vp, CAM, i32, i64, vp, vp, vp,
                                    vp, vp, vp, vp]),
    "mg_preprocess_backward": (i32, [vp, vp, vp, vp, vp, ShLayout, vp, i64, vp, i64, vp, i64,
                                     vp, CAM, i32, i64, vp, vp, vp, vp, vp, vp]),
    "mg_preprocess_backward_accumulate": (i32, [vp, vp, vp, vp, vp, vp, vp, vp, CAM, i32, i64,
                                                vp, vp, vp, vp, vp, vp, vp, vp, vp]),
    "mg_sh_backward_views": (i32, [vp, vp, vp, i32, i64, vp, vp, i32, i64, vp, vp, vp, vp]),
    "mg_mcmc_scratch_bytes": (sz, [i64]),
    "mg_mcmc_relocate": (i32, [vp, i32, i32, i32, vp, i32, i64, f32, vp, vp, C.c_uint64, vp, vp,
                               sz, vp]),
    "mg_mcmc_grow": (i32, [vp, i32, i32, i32, vp, i32, i64, i64, i64, vp, vp, C.c_uint64, vp, vp,
                           sz, vp]),
    "mg_mcmc_add_noise": (i32, [vp, vp, vp, vp, i64, f32, f32, f32, C.c_uint64, vp, vp]),
    "mg_compute_3d_filter_scratch_bytes": (sz, []),
    "mg_compute_3d_filter": (i32, [vp, i64, vp, i32, f32, f32, vp, vp, sz, vp]),
    "mg_apply_3d_filter": (i32, [vp, vp, vp, i64, vp, vp, vp]),
    "mg_apply_3d_filter_backward": (i32, [vp, vp, vp, vp, vp, i64, vp, vp, vp]),
    "mg_preprocess_forward_views": (i32, [vp, vp, vp, vp, vp, ShLayout, vp, vp, i32, i32, i64,
                                          i64, vp, vp, vp, vp, vp, vp, vp,
                                          C.POINTER(StepPrologue), vp]),
    "mg_sh_colour_views": (i32, [vp, vp, vp, ShLayout, vp, i32, i32, i64, i64, vp, vp, vp]),
    "mg_preprocess_backward_views": (i32, [vp, vp, vp, vp, vp, vp, vp, vp, i32, i64, i64, vp,
                                           vp, vp, vp, vp, vp, vp]),
    "mg_bin_count": (i32, [vp, vp, vp, vp, vp, i64, i32, i32, i32, i32, i32, vp, vp]),
    "mg_bin_write": (i32, [vp, vp, vp, vp, vp, vp, vp, i64, i64, i32, i32, i32, i32, i32, vp, vp,
                           vp]),
    "mg_sort_scratch_bytes": (sz, [i64, i32, i32]),
    "mg_sort_pairs_u32": (i32, [vp, vp, vp, vp, i64, i32, vp, sz, vp]),
    "mg_sort_pairs_u64": (i32, [vp, vp, vp, vp, i64, i32, vp, sz, vp]),
    "mg_sort_pairs_u32_noalloc": (i32, [vp, vp, i64, i32, vp]),
    "mg_tile_ranges": (i32, [vp, vp, i64, i32, vp, vp]),
    "mg_bin_prepare_scratch_bytes": (sz, [i64, i32]),
    "mg_bin_prepare": (i32, [vp, vp, vp, vp, vp, vp, i64, i32, i32, i32, i32, vp, vp, sz, vp]),
    "mg_regularizer_grad": (i32, [vp, vp, i64, f32, f32, vp, vp, vp, vp, sz, vp]),
    "mg_antialias_opacity_views": (i32, [vp, vp, i64, i32, i64, f32, vp, vp]),
    "mg_antialias_grad2d_views": (i32, [vp, vp, i64, i32, i64, f32, vp, vp]),
    "mg_bin_prepare_views_scratch_bytes": (sz, [i64, i32, i32]),
    "mg_bin_prepare_views": (i32, [vp, vp, vp, vp, vp, vp, i64, i32, i64, i64, i32, i32, i32,
                                   i32, vp, vp, sz, vp]),
    "mg_bin_emit_views_scratch_bytes": (sz, [i64, i32, i64, i32]),
    "mg_bin_emit_views": (i32, [vp, vp, vp, vp, i64, i32, i64, i64, i64, i32, i32, i32, i32,
                                vp, vp, vp, vp, sz, vp]),
    "mg_bin_emit_scratch_bytes": (sz, [i64, i64, i32]),
    "mg_bin_emit": (i32, [vp, vp, vp, vp, i64, i64, i32, i32, i32, i32, vp, vp, vp, vp, sz,
                          vp]),
    "mg_pack_splats": (i32, [vp, vp, vp, vp, i64, vp, vp, vp]),
    "mg_antialias_opacity": (i32, [vp, vp, i64, f32, vp, vp]),
    "mg_antialias_opacity_backward": (i32, [vp, vp, vp, i64, f32, vp, vp, vp]),
    "mg_raster_scratch_bytes": (sz, [i32, i32, i32, i64]),
    "mg_rasterize_forward": (i32, [vp, vp, vp, i64, i32, i32, i32, i32, vp, vp, vp, vp, vp, vp,
                                   vp, sz, vp]),
    "mg_rasterize_backward": (i32, [vp, vp, vp, i64, vp, vp, vp, vp, vp, vp, i32, i32, i32, i32,
                                    vp, i32, i64, vp, i32, vp, sz, vp]),
    "mg_tile_order": (i32, [vp, vp, i32, vp, vp]),
    "mg_pack_intersections": (i32, [vp, vp, vp, vp, vp, i64, vp, vp, vp, vp]),
    "mg_adam_step": (i32, [vp, vp, vp, vp, i64, f32, f32, f32, f32, f32, f32, vp]),
    "mg_selective_adam_step": (i32, [vp, vp, vp, vp, vp, vp, i64, i64, i64, f32, f32, f32, f32,
                                     vp]),
    "mg_selective_adam_advance_steps": (i32, [vp, vp, i64, i64, vp]),
    "mg_adam_multi": (i32, [vp, vp, vp, vp, i64, C.POINTER(AdamSegment), i32, f32, f32, f32, vp,
                            vp, i64, vp, i32, vp]),
    "mg_ssim_stack_blur_h": (i32, [vp, vp, vp, i32, i32, vp, vp]),
    "mg_ssim_blur15": (i32, [vp, vp, i32, i32, i32, vp, vp]),
    "mg_ssim_tail_forward": (i32, [vp, i32, i32, vp, vp]),
    "mg_ssim_tail_backward": (i32, [vp, vp, i32, i32, vp, vp]),
    "mg_ssim_chain_backward": (i32, [vp, vp, vp, i32, i32, vp, vp]),
    "mg_l1_ssim_scratch_bytes": (sz, [i32, i32]),
    "mg_l1_ssim_loss": (i32, [vp, vp, vp, i32, i32, f32, f32, f32, vp, vp, vp, sz, vp]),
    "mg_l1_ssim_loss_u8": (i32, [vp, vp, vp, i32, i32, f32, f32, f32, vp, vp, vp, sz, vp]),
    "mg_read_device_error": (i32, [C.POINTER(i32), vp]),
    "mg_peek_device_error": (i32, [vp, vp]),
    "mg_sort_lookback_selftest_scratch_bytes": (sz, []),
    "mg_sort_lookback_selftest": (i32, [C.c_uint32, vp, sz, vp]),
}

_lib = None
_lock = threading.Lock()


class NativeError(RuntimeError):
    """A non-zero mg_status from libmg_b200.so."""


def load() -> C.CDLL:
    """Load (building first if this checkout has no library yet) and bind."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists() or os.environ.get("MG_B200_REBUILD") == "1":
            build_native.build()
        if not LIB_PATH.exists():
            raise RuntimeError(f"libmg_b200.so not found at {LIB_PATH}; the CUDA backend "
                               "cannot run without it and does not fall back")
        lib = C.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def exported_symbols() -> list[str]:
    return list(SIGNATURES)


def check(status: int, what: str) -> None:
    if status != 0:
        msg = load().mg_last_error().decode(errors="replace")
        raise NativeError(f"{what} failed (mg_status {status}): {msg}")


def call(name: str, *args) -> None:
    """Call an mg_* entry point and raise on a non-zero status."""
    check(getattr(load(), name)(*args), name)


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def make_camera(viewmat: torch.Tensor, fx: float, fy: float, cx: float, cy: float, W: int,
                H: int, near: float, far: float, blur: float, max_radius: float,
                cam_center: torch.Tensor) -> Camera:
    """Pack one view's constants (rasterize.mm:226-242 makeParams). viewmat and
    cam_center are read on the host."""
    vm = viewmat.detach().to("cpu", torch.float32).contiguous().reshape(-1).tolist()
    cc = cam_center.detach().to("cpu", torch.float32).reshape(-1).tolist()
    cam = Camera()
    cam.viewmat[:] = vm
    cam.fx, cam.fy, cam.cx, cam.cy = float(fx), float(fy), float(cx), float(cy)
    cam.cam_center[:] = [cc[0], cc[1], cc[2], 0.0]
    cam.width, cam.height = int(W), int(H)
    cam.near_plane, cam.far_plane = float(near), float(far)
    cam.blur, cam.max_radius = float(blur), float(max_radius)
    return cam


DEVICE_ERRORS = {1: "a radix-sort look-back wait gave up (a predecessor tile never published)",
                 2: "a tile list reached past the sized pair count"}


class DeviceError(RuntimeError):
    """A kernel recorded a code in the device error word: its results are
    not trustworthy, so the caller refuses to continue (the reference's
    stance, metal_gauss/api.py:18-26)."""


def device_error(clear: bool = True) -> int:
    """Read (and clear) the device error word; 0 when nothing was recorded."""
    code = C.c_int32(0)
    call("mg_read_device_error", C.byref(code), stream())
    return code.value


def raise_device_error(code: int, where: str) -> None:
    """Clear the device error word and raise DeviceError for `code` (non-zero)
    observed by `where`."""
    device_error()
    raise DeviceError(f"{where}: device error {code}: "
                      f"{DEVICE_ERRORS.get(int(code), 'unknown code')}; results discarded")


def check_device_error(where: str) -> None:
    """Synchronising check of the device error word (raises DeviceError)."""
    code = device_error()
    if code:
        raise DeviceError(f"{where}: device error {code}: "
                          f"{DEVICE_ERRORS.get(int(code), 'unknown code')}; results discarded")


def library_path() -> Path:
    return LIB_PATH
