"""The C-ABI library loads (no GPU needed) and exports every entry point
that include/mg_b200.h declares; the Python binding covers all of them."""

import re

from metal_gauss_b200 import _lib

HEADER = _lib.build_native.ROOT / "include" / "mg_b200.h"


def declared() -> set[str]:
    text = HEADER.read_text()
    return set(re.findall(r"^\s*(?:mg_status|size_t|const char\*|int|uint64_t)\s+(mg_\w+)\s*\(",
                          text, re.M))


def test_header_declares_the_entry_points():
    names = declared()
    assert {"mg_preprocess_forward", "mg_preprocess_backward", "mg_bin_count", "mg_bin_write",
            "mg_rasterize_forward", "mg_rasterize_backward", "mg_adam_step",
            "mg_sort_pairs_u32", "mg_bin_prepare", "mg_bin_emit", "mg_l1_ssim_loss"} <= names


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    missing = [n for n in sorted(declared()) if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_covers_every_declared_symbol():
    assert declared() <= set(_lib.SIGNATURES)


def test_version_and_error_string():
    lib = _lib.load()
    assert lib.mg_version() >= 1
    assert isinstance(lib.mg_last_error(), bytes)


def test_scratch_queries_need_no_device():
    lib = _lib.load()
    assert lib.mg_sort_scratch_bytes(1 << 20, 32, 4) > 0
    assert lib.mg_bin_prepare_scratch_bytes(1000, 2500) > 4 * 1000 + 64 * 4 * 2500
    assert lib.mg_bin_emit_scratch_bytes(1000, 5000, 2500) > 4 * 5000
    # a batch of one view has the single-view layout; eight views eight times the rows
    assert lib.mg_bin_prepare_views_scratch_bytes(1000, 1, 2500) == \
        lib.mg_bin_prepare_scratch_bytes(1000, 2500)
    assert lib.mg_bin_prepare_views_scratch_bytes(1000, 8, 2500) > 8 * 40 * 1000
    assert lib.mg_bin_emit_views_scratch_bytes(1000, 8, 5000, 2500) > \
        lib.mg_bin_emit_scratch_bytes(1000, 5000, 2500)
    assert lib.mg_bin_prepare_views_scratch_bytes(1000, 0, 2500) == 0
    assert lib.mg_l1_ssim_scratch_bytes(64, 64) >= 9 * 64 * 64 * 4
    # counters + tile order + block walks + items + checkpoints (5 floats per
    # pixel slot per MG_RASTER_SEGMENT entries)
    rb = lib.mg_raster_scratch_bytes(800, 800, 16, 10_000_000)
    assert rb >= 4 * 5 * 256 * (10_000_000 // _lib.RASTER_SEGMENT)
    assert lib.mg_raster_scratch_bytes(0, 800, 16, 10) == 0
