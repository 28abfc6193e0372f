"""GPU parity: the sm_100a kernels against the CPU oracle and the reference.

Bar (BASELINE): projection outputs, tile keys, sort order and per-tile ranges
bit-exact; images within 1e-4 max abs of torch_ref; parameter gradients
within 1e-3 relative L2. Every call goes through libmg_b200.so.
"""

import math

import numpy as np
import pytest
import torch

import oracle
from metal_gauss_b200 import ext
from metal_gauss_b200.cuda_backend import render as cuda_render
from tests.golden.fixtures import load, rel_l2

pytestmark = pytest.mark.gpu

IMG_TOL = 1e-4
GRAD_TOL = 1e-3


def T(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return t if dtype is None else t.to(dtype)


def N(t):
    return t.detach().cpu().numpy()


def cam_args(K, vm, W, H, near=0.01, far=100.0, max_radius_frac=1.0):
    vm = torch.as_tensor(vm, dtype=torch.float32)
    K = torch.as_tensor(K, dtype=torch.float32)
    cc = -vm[:3, :3].T @ vm[:3, 3]
    return (vm, float(K[0, 0]), float(K[1, 1]), float(K[0, 2]), float(K[1, 2]), W, H, near, far,
            0.3, max_radius_frac * max(W, H), cc)


def random_scene(n, seed, W, H, sh_deg=3, f=None):
    g = np.random.default_rng(seed)
    means = (g.standard_normal((n, 3)) * 0.6 + [0, 0, 4]).astype(np.float32)
    quats = g.standard_normal((n, 4)).astype(np.float32)
    scales = (g.random((n, 3)) * 0.08 + 0.01).astype(np.float32)
    opac = (g.random(n) * 0.9 + 0.05).astype(np.float32)
    sh = (g.standard_normal((n, 16, 3)) * 0.3).astype(np.float32)
    f = f or 0.8 * max(W, H)
    K = np.array([[f, 0, W / 2], [0, f, H / 2], [0, 0, 1]], np.float32)
    return means, quats, scales, opac, sh, K


# ------------------------------------------------------------ preprocess

@pytest.mark.parametrize("layout", ["fused", "split"])
@pytest.mark.parametrize("deg", [0, 1, 2, 3])
def test_preprocess_forward_is_bit_exact(cuda, layout, deg):
    W, H = 320, 240
    means, quats, scales, opac, sh, K = random_scene(20000, 7 + deg, W, H)
    vm = np.eye(4, dtype=np.float32)
    vm[:3, 3] = [0.1, -0.2, 0.3]
    cam = oracle.camera(vm, K, W, H)
    if layout == "fused":
        ref = oracle.preprocess_forward(means, quats, scales, sh, None, opac, cam, deg)
        sh_t = T(sh)
        out = ext.preprocess_forward(T(means), T(quats), T(scales), sh_t, sh_t, T(opac),
                                     *cam_args(K, vm, W, H), deg)
    else:
        ref = oracle.preprocess_forward(means, quats, scales, sh[:, :1], sh[:, 1:], opac, cam, deg)
        out = ext.preprocess_forward(T(means), T(quats), T(scales), T(sh[:, :1]), T(sh[:, 1:]),
                                     T(opac), *cam_args(K, vm, W, H), deg)
    for name, o in zip(("uv", "conic", "depth", "rxy", "valid", "color"), out):
        assert np.array_equal(N(o), ref[name]), name
    assert ref["valid"].sum() > 1000


def test_preprocess_backward_matches_oracle(cuda):
    W, H = 320, 240
    means, quats, scales, opac, sh, K = random_scene(20000, 3, W, H)
    vm = np.eye(4, dtype=np.float32)
    cam = oracle.camera(vm, K, W, H)
    pre = oracle.preprocess_forward(means, quats, scales, sh[:, :1], sh[:, 1:], opac, cam, 3)
    g = np.random.default_rng(0)
    n = means.shape[0]
    d_uv = g.standard_normal((n, 2)).astype(np.float32)
    d_conic = g.standard_normal((n, 3)).astype(np.float32)
    d_color = g.standard_normal((n, 3)).astype(np.float32)
    d_color[::3] = 0.0                                    # zero-gradient fast path
    ref = oracle.preprocess_backward(means, quats, scales, sh[:, :1], sh[:, 1:], d_uv, d_conic,
                                     d_color, pre["valid"], cam, 3)
    out = ext.preprocess_backward(T(means), T(quats), T(scales), T(sh[:, :1]), T(sh[:, 1:]),
                                  T(d_uv), T(d_conic), T(d_color), T(pre["valid"]),
                                  *cam_args(K, vm, W, H), 3)
    for name, o, r in zip(("means", "quats", "scales", "sh", "sh_rest"), out,
                          (ref["means"], ref["quats"], ref["scales"], ref["sh"], ref["sh_rest"])):
        assert rel_l2(N(o), r) < 1e-5, name
    # invalid rows: zero scale/quat gradients; rows with zero d_color: zero SH grads
    inv = pre["valid"] == 0
    assert inv.any() and np.all(N(out[1])[inv] == 0) and np.all(N(out[2])[inv] == 0)
    assert np.all(N(out[4])[::3] == 0)


def test_preprocess_backward_reads_strided_gradients(cuda):
    """d_uv/d_conic/d_color may be row views into the packed (N,12) record."""
    W, H = 160, 120
    means, quats, scales, opac, sh, K = random_scene(3000, 5, W, H)
    vm = np.eye(4, dtype=np.float32)
    args = cam_args(K, vm, W, H)
    m, q, s, o, shd = T(means), T(quats), T(scales), T(opac), T(sh)
    valid = ext.preprocess_forward(m, q, s, shd, shd, o, *args, 3)[4]
    rec = torch.randn(3000, 12, device="cuda")
    a = ext.preprocess_backward(m, q, s, shd, shd, rec[:, 0:2], rec[:, 4:7], rec[:, 8:11], valid,
                                *args, 3)
    b = ext.preprocess_backward(m, q, s, shd, shd, rec[:, 0:2].contiguous(),
                                rec[:, 4:7].contiguous(), rec[:, 8:11].contiguous(), valid,
                                *args, 3)
    for x, y in zip(a[:4], b[:4]):
        assert torch.equal(x, y)


# ------------------------------------------------------------------ sort

@pytest.mark.parametrize("n", [0, 1, 2, 1000, 4097, 65536 + 17, 1_000_003])
@pytest.mark.parametrize("bits", [5, 12, 32])
def test_sort_pairs_u32_is_stable(cuda, n, bits):
    g = np.random.default_rng(n + bits)
    hi = min(1 << bits, 1 << 31)
    keys = g.integers(0, max(2, hi // 64 if n > 100 else hi), n).astype(np.int64)  # many ties
    keys = (keys & ((1 << bits) - 1)).astype(np.uint32)
    vals = np.arange(n, dtype=np.int32)
    k, v = ext.sort_pairs(T(keys.view(np.int32)), T(vals), bits)
    order = np.argsort(keys, kind="stable")
    assert np.array_equal(N(k).view(np.uint32), keys[order])
    assert np.array_equal(N(v), vals[order])


@pytest.mark.parametrize("n", [3, 5000, 300_001])
def test_sort_pairs_u64_matches_stable_argsort(cuda, n):
    g = np.random.default_rng(n)
    tiles = g.integers(0, 2500, n).astype(np.uint64)
    depth = g.random(n).astype(np.float32)
    depth[::7] = depth[0]                                  # exact ties
    keys = (tiles << np.uint64(32)) | depth.view(np.uint32).astype(np.uint64)
    vals = g.integers(0, 1 << 30, n).astype(np.int32)
    k, v = ext.sort_pairs(T(keys.view(np.int64)), T(vals), 44)
    order = np.argsort(keys, kind="stable")
    assert np.array_equal(N(k).view(np.uint64), keys[order])
    assert np.array_equal(N(v), vals[order])
    off = ext.tile_ranges(k, 2500)
    assert np.array_equal(N(off), np.searchsorted(keys[order] >> np.uint64(32),
                                                  np.arange(2501), side="left"))


# --------------------------------------------------------------- binning

@pytest.mark.parametrize("tile", [16, 32])
def test_binning_is_bit_exact_with_the_reference(cuda, tile):
    """Reference outputs: metal_backend.build_tile_lists with the ellipse test."""
    f = load("binning")
    W, H = int(f["W"]), int(f["H"])
    args = [T(f[k]) for k in ("pre_uv", "pre_rxy", "pre_conic", "opac", "pre_valid", "pre_depth")]
    ids, offsets, tx = ext.bin_and_sort(*args, W, H, tile)
    assert tx == math.ceil(W / tile)
    assert np.array_equal(N(ids), f[f"t{tile}_ids"])
    assert np.array_equal(N(offsets), f[f"t{tile}_offsets"])
    # the reference's own flow: bin_count -> cumsum -> bin_write -> sort -> ranges
    uv, rxy, conic, op, valid, depth = args
    tx, ty = math.ceil(W / tile), math.ceil(H / tile)
    counts = ext.bin_count(uv, rxy, conic, op, valid, W, H, tile, tx, ty)
    offs = torch.cumsum(counts, 0, dtype=torch.int64) - counts
    total = int(counts.sum())
    keys, kid = ext.bin_write(uv, rxy, conic, op, valid, depth, offs.to(torch.int32), total, W,
                              H, tile, tx, ty)
    sk, sv = ext.sort_pairs(keys, kid, 32 + math.ceil(math.log2(tx * ty)))
    assert np.array_equal(N(sv), f[f"t{tile}_ids"])
    assert np.array_equal(N(ext.tile_ranges(sk, tx * ty)), f[f"t{tile}_offsets"])


def test_binning_end_to_end_bit_exact_at_scale(cuda):
    """100k Gaussians at 800x800: projection then binning, GPU vs oracle."""
    W = H = 800
    means, quats, scales, opac, sh, K = random_scene(100_000, 11, W, H)
    vm = np.eye(4, dtype=np.float32)
    cam = oracle.camera(vm, K, W, H)
    ref = oracle.preprocess_forward(means, quats, scales, None, None, opac, cam, -1)
    r_ids, r_off, _ = oracle.build_tile_lists(ref["uv"], ref["rxy"], ref["conic"], opac,
                                              ref["valid"], ref["depth"], W, H, 16)
    o = ext.preprocess_forward(T(means), T(quats), T(scales), None, None, T(opac),
                               *cam_args(K, vm, W, H), -1)
    ids, off, _ = ext.bin_and_sort(o[0], o[3], o[1], T(opac), o[4], o[2], W, H, 16)
    assert r_ids.size > 500_000
    assert np.array_equal(N(ids), r_ids)
    assert np.array_equal(N(off), r_off)


@pytest.mark.parametrize("tile", [8, 16])
def test_binning_mixes_recorded_and_rewalked_rectangles(cuda, tile):
    """The emission expands the count walk's recorded decisions for tile
    rectangles of at most 64 tiles and walks larger ones again; a scene with
    both, against the oracle."""
    W, H = 400, 300
    means, quats, scales, opac, _, K = random_scene(20_000, 5, W, H)
    g = np.random.default_rng(6)
    big = g.random(scales.shape[0]) < 0.05
    scales[big] *= 8.0
    vm = np.eye(4, dtype=np.float32)
    cam = oracle.camera(vm, K, W, H)
    ref = oracle.preprocess_forward(means, quats, scales, None, None, opac, cam, -1)
    r_ids, r_off, _ = oracle.build_tile_lists(ref["uv"], ref["rxy"], ref["conic"], opac,
                                              ref["valid"], ref["depth"], W, H, tile)
    side = (2 * ref["rxy"] / tile + 1)[ref["valid"] != 0]
    span = side[:, 0] * side[:, 1]
    assert (span > 100).sum() > 50 and (span < 30).sum() > 1000  # both kinds present
    o = ext.preprocess_forward(T(means), T(quats), T(scales), None, None, T(opac),
                               *cam_args(K, vm, W, H), -1)
    ids, off, _ = ext.bin_and_sort(o[0], o[3], o[1], T(opac), o[4], o[2], W, H, tile)
    assert np.array_equal(N(ids), r_ids)
    assert np.array_equal(N(off), r_off)
    # with the saturation cut (the large rectangles' histogram adds, recount
    # and emission run as whole-warp walks): each tile keeps a front prefix of
    # its full list
    c_ids, c_off = _cut_lists(o, T(opac), W, H, tile)
    assert c_off[-1] <= r_off[-1]
    for t in range(len(r_off) - 1):
        kept = c_ids[c_off[t]:c_off[t + 1]]
        assert np.array_equal(kept, r_ids[r_off[t]:r_off[t] + kept.size]), t


def _cut_lists(o, opac, W, H, tile):
    """mg_bin_prepare / mg_bin_emit with the saturation cut on."""
    from metal_gauss_b200 import _lib
    from metal_gauss_b200._lib import ptr
    L = _lib.load()
    s = _lib.stream()
    uv, conic, depth, rxy, valid = o[0], o[1], o[2], o[3], o[4]
    n = uv.shape[0]
    n_tiles = -(-W // tile) * -(-H // tile)
    tot = torch.zeros(1, dtype=torch.int64, device="cuda")
    prep = torch.empty(L.mg_bin_prepare_scratch_bytes(n, n_tiles), dtype=torch.uint8,
                       device="cuda")
    _lib.call("mg_bin_prepare", ptr(uv), ptr(rxy), ptr(conic), ptr(opac), ptr(valid), ptr(depth),
              n, W, H, tile, 1, ptr(tot), ptr(prep), prep.numel(), s)
    m = int(tot.item())
    ids = torch.empty(max(m, 1), dtype=torch.int32, device="cuda")
    off = torch.empty(n_tiles + 1, dtype=torch.int32, device="cuda")
    emit = torch.empty(L.mg_bin_emit_scratch_bytes(n, m, n_tiles), dtype=torch.uint8,
                       device="cuda")
    _lib.call("mg_bin_emit", ptr(uv), ptr(rxy), ptr(conic), ptr(opac), n, m, W, H, tile, 1,
              ptr(prep), ptr(ids), ptr(off), ptr(emit), emit.numel(), s)
    return ids[:m].cpu().numpy(), off.cpu().numpy()


def test_binning_of_an_empty_and_an_invisible_scene(cuda):
    W, H = 64, 64
    ids, off, tx = ext.bin_and_sort(*(torch.zeros(0, k, device="cuda") for k in (2, 2, 3)),
                                    torch.zeros(0, device="cuda"),
                                    torch.zeros(0, dtype=torch.int32, device="cuda"),
                                    torch.zeros(0, device="cuda"), W, H, 16)
    assert ids.numel() == 0 and int(off[-1]) == 0 and off.numel() == 17
    n = 128
    means = torch.zeros(n, 3, device="cuda")
    means[:, 2] = -5.0                                    # behind the camera
    quats = torch.zeros(n, 4, device="cuda")
    quats[:, 0] = 1
    o = ext.preprocess_forward(means, quats, torch.full((n, 3), 0.01, device="cuda"), None, None,
                               torch.full((n,), 0.5, device="cuda"),
                               *cam_args(np.eye(3) * 100 + [[0, 0, 32], [0, 0, 32], [0, 0, -99]],
                                         np.eye(4), W, H), -1)
    assert int(o[4].sum()) == 0
    ids, off, _ = ext.bin_and_sort(o[0], o[3], o[1], torch.full((n,), 0.5, device="cuda"), o[4],
                                   o[2], W, H, 16)
    assert ids.numel() == 0 and int(off[-1]) == 0


# ---------------------------------------------------------------- raster

def _oracle_scene(n, W, H, seed, deg=3, tile=16):
    means, quats, scales, opac, sh, K = random_scene(n, seed, W, H)
    vm = np.eye(4, dtype=np.float32)
    cam = oracle.camera(vm, K, W, H)
    pre = oracle.preprocess_forward(means, quats, scales, sh, None, opac, cam, deg)
    ids, off, _ = oracle.build_tile_lists(pre["uv"], pre["rxy"], pre["conic"], opac, pre["valid"],
                                          pre["depth"], W, H, tile)
    return pre, opac, ids, off


def _raster_vs_oracle(pre, opac, ids, off, W, H, tile, bg, segmented, grad_tol):
    r_rgb, r_alpha, r_T, r_stop = oracle.rasterize_forward(pre["uv"], pre["conic"], opac,
                                                           pre["color"], ids, off, W, H, tile, bg)
    tx = math.ceil(W / tile)
    args = [T(pre["uv"]), T(pre["conic"]), T(opac), T(pre["color"])]
    state = [] if segmented else None
    rgb, alpha, Tt, stop = ext.rasterize_forward(*args, T(ids), T(off), W, H, tile, tx,
                                                 background=bg, state_out=state)
    assert np.abs(N(rgb) - r_rgb).max() < IMG_TOL
    assert np.abs(N(alpha) - r_alpha).max() < IMG_TOL
    assert (N(stop) == r_stop).mean() > 0.999
    g = np.random.default_rng(1)
    grgb = g.standard_normal((H, W, 3)).astype(np.float32)
    ga = g.standard_normal((H, W)).astype(np.float32)
    ref = oracle.rasterize_backward(pre["uv"], pre["conic"], opac, pre["color"], ids, off, r_T,
                                    r_stop, grgb, ga, W, H, tile, bg, r_alpha, True)
    got = N(ext.rasterize_backward_packed(*args, T(ids), T(off), Tt, stop, T(grgb), T(ga), W, H,
                                          tile, tx, True, background=bg, alpha=alpha,
                                          state=state[0] if segmented else None, rgb=rgb))
    for sl, name in ((slice(0, 2), "uv"), (slice(2, 3), "opacity"), (slice(3, 4), "absgrad"),
                     (slice(4, 7), "conic"), (slice(8, 11), "color")):
        assert rel_l2(got[:, sl], ref[:, sl]) < grad_tol, name
    assert ext.device_error() == 0
    return r_stop - off[:-1].min()


@pytest.mark.parametrize("segmented", [False, True])
@pytest.mark.parametrize("tile", [8, 12, 16, 32])
def test_rasterize_forward_and_backward_match_oracle(cuda, tile, segmented):
    W, H = 200, 130
    pre, opac, ids, off = _oracle_scene(6000, W, H, 2, tile=tile)
    bg = np.array([0.2, 0.5, 1.0], np.float32)
    _raster_vs_oracle(pre, opac, ids, off, W, H, tile, bg, segmented, 1e-4)


@pytest.mark.parametrize("tile", [12, 16])
def test_segmented_backward_on_long_lists(cuda, tile):
    """Faint, wide splats: lists of 6-7k entries that few pixels finish
    early, so the backward runs over twenty segments per warp block, each
    started from a forward checkpoint, next to blocks whose pixels stop
    inside a segment."""
    W, H = 72, 56
    g = np.random.default_rng(11)
    n = 12000
    means = np.stack([g.uniform(-1.2, 1.2, n), g.uniform(-0.9, 0.9, n),
                      g.uniform(3.0, 6.0, n)], 1).astype(np.float32)
    quats = g.standard_normal((n, 4)).astype(np.float32)
    scales = (g.random((n, 3)) * 0.25 + 0.05).astype(np.float32)
    opac = (g.random(n) * 0.03 + 0.006).astype(np.float32)
    sh = (g.standard_normal((n, 16, 3)) * 0.3).astype(np.float32)
    K = np.array([[60, 0, W / 2], [0, 60, H / 2], [0, 0, 1]], np.float32)
    cam = oracle.camera(np.eye(4, dtype=np.float32), K, W, H)
    pre = oracle.preprocess_forward(means, quats, scales, sh, None, opac, cam, 3)
    ids, off, _ = oracle.build_tile_lists(pre["uv"], pre["rxy"], pre["conic"], opac, pre["valid"],
                                          pre["depth"], W, H, tile)
    lens = np.diff(off)
    assert lens.max() > 8 * 256, "scene must produce lists spanning many segments"
    for segmented in (False, True):
        _raster_vs_oracle(pre, opac, ids, off, W, H, tile, None, segmented, 2e-4)


# ------------------------------------------------- whole render vs torch_ref

def _torch_inputs(f, keys=("means", "quats", "scales", "opac")):
    return [T(f[k]).requires_grad_(True) for k in keys]


@pytest.mark.parametrize("name,deg", [("cfg1", 0), ("sh3", 3)])
def test_render_and_gradients_match_torch_ref(cuda, name, deg):
    f = load(name)
    W, H = int(f["W"]), int(f["H"])
    m, q, s, o = _torch_inputs(f)
    sh = T(f["sh"]).requires_grad_(True)
    bg = tuple(f["background"].tolist()) if "background" in f else (0.0, 0.0, 0.0)
    rgb, alpha, info = cuda_render(m, q, s, o, sh, T(f["K"]), torch.from_numpy(f["viewmat"]), W,
                                   H, sh_degree=deg, background=bg)
    assert np.abs(N(rgb) - f["rgb"]).max() < IMG_TOL
    assert np.abs(N(alpha) - f["alpha"]).max() < IMG_TOL
    if name == "cfg1":
        loss = (rgb - T(f["target"])).abs().mean()
    else:
        loss = rgb.square().mean() + 0.1 * alpha.square().mean()
    loss.backward()
    for t, gk in ((m, "g_means"), (q, "g_quats"), (s, "g_scales"), (o, "g_opac")):
        assert rel_l2(N(t.grad), f[gk]) < GRAD_TOL, gk
    assert rel_l2(N(sh.grad)[:, :f["g_sh"].shape[1]], f["g_sh"]) < GRAD_TOL
    assert info["backend"] == "cuda" and info["isect_total"] > 0 and info["isect_dropped"] == 0


@pytest.mark.parametrize("tile", [8, 12, 16, 32])
def test_every_tile_size_matches_torch_ref(cuda, tile):
    f = load("tiles")
    W, H = int(f["W"]), int(f["H"])
    m, q, s, o, c = _torch_inputs(f, ("means", "quats", "scales", "opac", "colors"))
    rgb, alpha, _ = cuda_render(m, q, s, o, None, T(f["K"]), torch.from_numpy(f["viewmat"]), W, H,
                                colors=c, tile=tile)
    p = f"t{tile}_"
    assert np.abs(N(rgb) - f[p + "rgb"]).max() < IMG_TOL
    assert np.abs(N(alpha) - f[p + "alpha"]).max() < IMG_TOL
    (rgb.square().mean() + 0.1 * alpha.square().mean()).backward()
    for t, gk in ((m, "g_means"), (q, "g_quats"), (s, "g_scales"), (o, "g_opac"),
                  (c, "g_colors")):
        assert rel_l2(N(t.grad), f[p + gk]) < GRAD_TOL, gk


def test_full_size_view_matches_oracle(cuda):
    """A cfg2-sized view (100k Gaussians, 800x800, SH 3): forward and all
    parameter gradients against the oracle."""
    W = H = 800
    means, quats, scales, opac, sh, K = random_scene(100_000, 21, W, H)
    vm = np.eye(4, dtype=np.float32)
    rgb_r, alpha_r, st = oracle.render(means, quats, scales, opac, sh[:, :1], K, vm, W, H,
                                       sh_degree=3, sh_rest=sh[:, 1:])
    m, q, s, o = (T(x).requires_grad_(True) for x in (means, quats, scales, opac))
    dc, rest = T(sh[:, :1]).requires_grad_(True), T(sh[:, 1:]).requires_grad_(True)
    rgb, alpha, info = cuda_render(m, q, s, o, dc, T(K), torch.from_numpy(vm), W, H, sh_degree=3,
                                   sh_rest=rest)
    assert info["isect_total"] == st["ids"].size
    assert np.abs(N(rgb) - rgb_r).max() < IMG_TOL
    g = np.random.default_rng(4)
    grgb = (g.standard_normal((H, W, 3)) / (H * W)).astype(np.float32)
    (rgb * T(grgb)).sum().backward()
    ref = oracle.render_backward(st, grgb, None)
    for t, k in ((m, "means"), (q, "quats"), (s, "scales"), (o, "opacities")):
        assert rel_l2(N(t.grad), ref[k]) < GRAD_TOL, k
    assert rel_l2(N(dc.grad), ref["sh"]) < GRAD_TOL
    assert rel_l2(N(rest.grad), ref["sh_rest"]) < GRAD_TOL


# -------------------------------------------- behaviour ported from the reference

def intrinsics(W, H, f=None):
    f = f or 0.8 * max(W, H)
    K = torch.eye(3)
    K[0, 0], K[1, 1], K[0, 2], K[1, 2] = f, f, W / 2, H / 2
    return K


def scene(n=400, seed=0, device="cuda", requires_grad=False):
    torch.manual_seed(seed)
    means = (torch.randn(n, 3) * 0.6 + torch.tensor([0.0, 0.0, 4.0])).to(device)
    quats = torch.randn(n, 4).to(device)
    scales = (torch.rand(n, 3) * 0.10 + 0.03).to(device)
    opac = (torch.rand(n) * 0.7 + 0.15).to(device)
    cols = torch.rand(n, 3).to(device)
    out = [means, quats, scales, opac, cols]
    if requires_grad:
        out = [t.requires_grad_(True) for t in out]
    return out


def test_an_empty_scene_renders_the_background(cuda):
    W, H = 48, 32
    z = lambda *s: torch.zeros(*s, device="cuda")  # noqa: E731
    rgb, alpha, _ = cuda_render(z(0, 3), z(0, 4), z(0, 3), z(0), z(0, 16, 3), intrinsics(W, H),
                                torch.eye(4), W, H, background=(1.0, 0.0, 0.0))
    assert rgb.shape == (H, W, 3) and alpha.shape == (H, W)
    assert torch.equal(rgb, torch.tensor([1.0, 0.0, 0.0], device="cuda").expand(H, W, 3))
    assert float(alpha.max()) == 0.0


def test_refuses_cpu_tensors():
    m, q, s, o, c = scene(n=10, device="cpu")
    with pytest.raises(RuntimeError, match="requires CUDA tensors"):
        cuda_render(m, q, s, o, None, intrinsics(16, 16), torch.eye(4), 16, 16, colors=c)


def test_refuses_a_tile_the_gpu_cannot_dispatch(cuda):
    m, q, s, o, c = scene(n=50)
    with pytest.raises(RuntimeError, match="threads per threadgroup"):
        cuda_render(m, q, s, o, None, intrinsics(96, 64), torch.eye(4), 96, 64, colors=c,
                    tile=64)


@pytest.mark.parametrize("sh_degree", [0, 1, 2, 3])
def test_split_sh_matches_fused(cuda, sh_degree):
    g = torch.Generator().manual_seed(0)
    n, W, H = 4000, 96, 128
    means = (torch.randn(n, 3, generator=g) * 0.4).cuda()
    means[:, 2] += 3.0
    quats = torch.randn(n, 4, generator=g).cuda()
    scales = (torch.rand(n, 3, generator=g) * 0.05 + 0.01).cuda()
    opac = (torch.rand(n, generator=g) * 0.8 + 0.1).cuda()
    sh = (torch.randn(n, 16, 3, generator=g) * 0.3).cuda()
    K = torch.tensor([[100.0, 0, W / 2], [0, 100.0, H / 2], [0, 0, 1]])
    fused = sh.clone().requires_grad_(True)
    rgb_f, _, _ = cuda_render(means, quats, scales, opac, fused, K, torch.eye(4), W, H,
                              sh_degree=sh_degree)
    rgb_f.square().mean().backward()
    dc = sh[:, :1].clone().requires_grad_(True)
    rest = sh[:, 1:].clone().requires_grad_(True)
    rgb_s, _, _ = cuda_render(means, quats, scales, opac, dc, K, torch.eye(4), W, H,
                              sh_degree=sh_degree, sh_rest=rest)
    rgb_s.square().mean().backward()
    assert torch.equal(rgb_f, rgb_s)
    scale = float(fused.grad.abs().max())
    assert float((fused.grad[:, :1] - dc.grad).abs().max()) <= 1e-5 * scale
    assert float((fused.grad[:, 1:] - rest.grad).abs().max()) <= 1e-5 * scale


def test_split_gradient_is_not_doubled(cuda):
    m, q, s, o, _ = scene(n=800, seed=1)
    sh0 = torch.randn(800, 16, 3, device="cuda") * 0.3
    a = sh0.clone().requires_grad_(True)
    rgb, _, _ = cuda_render(m, q, s, o, a, intrinsics(96, 64), torch.eye(4), 96, 64)
    rgb.square().mean().backward()
    b = sh0.clone().requires_grad_(True)
    rgb2, _, _ = cuda_render(m, q, s, o, b, intrinsics(96, 64), torch.eye(4), 96, 64)
    (2.0 * rgb2).square().mean().backward()
    assert torch.allclose(b.grad, 4.0 * a.grad, rtol=1e-4, atol=1e-7)


def test_full_sh_with_sh_rest_is_rejected(cuda):
    m, q, s, o, _ = scene(n=50)
    sh = torch.randn(50, 16, 3, device="cuda")
    with pytest.raises(ValueError, match="DC band"):
        cuda_render(m, q, s, o, sh, intrinsics(32, 32), torch.eye(4), 32, 32, sh_rest=sh[:, 1:])


def test_offscreen_gaussians_get_exactly_zero_gradient(cuda):
    W, H, n = 64, 48, 300
    m0, q0, s0, o0, _ = scene(n=n, seed=13)
    off = torch.arange(n, device="cuda") % 2 == 1
    m0 = m0.clone()
    m0[off, 0] += 20.0
    sh0 = torch.randn(n, 16, 3, device="cuda") * 0.25
    m, q, s, sh = (t.clone().requires_grad_(True) for t in (m0, q0, s0, sh0))
    rgb, alpha, _ = cuda_render(m, q, s, o0, sh, intrinsics(W, H), torch.eye(4), W, H)
    (rgb.square().mean() + 0.1 * alpha.square().mean()).backward()
    for t in (m, q, s, sh):
        assert torch.isfinite(t.grad).all()
        assert float(t.grad[off].abs().max()) == 0.0


def test_absgrad_dominates_the_signed_norm(cuda):
    m, q, s, o, c = scene(n=300)
    m = m.clone().requires_grad_(True)
    absbuf = torch.zeros(300, device="cuda")
    rgb, _, info = cuda_render(m, q, s, o, None, intrinsics(96, 64), torch.eye(4), 96, 64,
                               colors=c, absgrad_out=absbuf)
    rgb.square().mean().backward()
    signed = info["uv"].grad.norm(dim=1)
    assert (absbuf >= 0).all() and absbuf.sum() > 0
    assert ((absbuf - signed) >= -1e-4).all()
    assert ((absbuf - signed) > 1e-6).any()


def test_antialias_matches_oracle_and_darkens(cuda):
    W, H = 96, 64
    torch.manual_seed(0)
    n = 400
    means = torch.randn(n, 3) * 0.6 + torch.tensor([0.0, 0.0, 4.0])
    quats = torch.randn(n, 4)
    scales = torch.rand(n, 3) * 0.03 + 0.004
    opac = torch.rand(n) * 0.7 + 0.15
    cols = torch.rand(n, 3)
    K = intrinsics(W, H)
    ref, _, _ = oracle.render(means.numpy(), quats.numpy(), scales.numpy(), opac.numpy(), None,
                              K.numpy(), np.eye(4, dtype=np.float32), W, H, colors=cols.numpy(),
                              antialias=True)
    args = [t.cuda() for t in (means, quats, scales, opac)]
    on, _, _ = cuda_render(*args, None, K, torch.eye(4), W, H, colors=cols.cuda(), antialias=True)
    off, _, _ = cuda_render(*args, None, K, torch.eye(4), W, H, colors=cols.cuda())
    assert np.abs(N(on) - ref).max() < 1e-4
    assert float((off - on).abs().max()) > 1e-4
    assert float(on.sum()) <= float(off.sum()) + 1e-3


def test_fused_antialias_gradient_matches_the_reference_expression(cuda):
    """antialias_opacity (one kernel each way) against torch autograd through
    the reference's antialias_scale expression (metal_backend.py:367-393)."""
    from metal_gauss_b200.cuda_backend import antialias_opacity, antialias_scale
    f = load("antialias")
    conic = torch.from_numpy(f["conic"]).cuda()
    g = torch.Generator(device="cuda").manual_seed(3)
    opac = torch.rand(conic.shape[0], device="cuda", generator=g) * 0.9 + 0.05
    up = torch.randn(conic.shape[0], device="cuda", generator=g)
    c1, o1 = conic.clone().double().requires_grad_(True), opac.clone().double().requires_grad_(True)
    ref = o1 * antialias_scale(c1, 0.3)
    (ref * up.double()).sum().backward()
    c2, o2 = conic.clone().requires_grad_(True), opac.clone().requires_grad_(True)
    got = antialias_opacity(c2, o2, 0.3)
    (got * up).sum().backward()
    assert float((got.detach() - ref.detach().float()).abs().max()) < 1e-6
    assert rel_l2(N(o2.grad), N(o1.grad)) < 1e-5
    assert rel_l2(N(c2.grad), N(c1.grad)) < 1e-4


def test_boundary_energy_matches_reference(cuda):
    f = load("boundary")
    W = H = 128
    F, Z = 100.0, 2.0
    K = torch.tensor([[F, 0, W / 2], [0, F, H / 2], [0, 0, 1.0]])
    sh = torch.zeros(1, 16, 3, device="cuda")
    sh[:, 0] = 1.0
    q = torch.tensor([[1.0, 0, 0, 0]], device="cuda")
    s = torch.full((1, 3), 0.04, device="cuda")
    o = torch.tensor([0.99], device="cuda")
    out = []
    for u in f["us"]:
        m = torch.tensor([[(u - W / 2) * Z / F, 0.0, Z]], dtype=torch.float32, device="cuda")
        rgb, _, _ = cuda_render(m, q, s, o, sh, K, torch.eye(4), W, H, tile=32)
        out.append(float(rgb.sum()))
    assert np.abs(np.array(out) - f["energy"]).max() < 1e-3
    steps = np.abs(np.diff(out))
    assert steps.max() <= 8 * max(np.median(steps), 1e-9)


# -------------------------------------------------------------- optimisers

def test_fused_adam_matches_torch_adam_over_many_steps(cuda):
    from metal_gauss_b200.fused_adam import FusedAdam
    shapes = [(5000, 3), (5000, 4), (5000, 1, 3), (5000, 15, 3), (5000,)]
    lrs = [1.6e-4, 1e-3, 2.5e-3, 1.25e-4, 1e-2]
    torch.manual_seed(7)
    A = [torch.randn(*s, device="cuda", requires_grad=True) for s in shapes]
    B = [a.detach().clone().requires_grad_(True) for a in A]
    oa = torch.optim.Adam([{"params": [t], "lr": l} for t, l in zip(A, lrs)], eps=1e-15)
    ob = FusedAdam([{"params": [t], "lr": l} for t, l in zip(B, lrs)], eps=1e-15)
    torch.manual_seed(11)
    for _ in range(30):
        for a, b in zip(A, B):
            g = torch.randn_like(a)
            a.grad, b.grad = g.clone(), g.clone()
        oa.step()
        ob.step()
    for a, b in zip(A, B):
        assert float((a - b).detach().abs().max() / a.detach().abs().max()) < 1e-5
    st = ob.state[B[0]]
    assert {"step", "exp_avg", "exp_avg_sq"} <= set(st) and st["exp_avg"].shape == B[0].shape


def test_selective_adam_matches_reference_trajectory(cuda):
    from metal_gauss_b200.selective_adam import SelectiveAdam
    f = load("selective_adam")
    ps = [T(f[f"p{i}"]).requires_grad_(True) for i in range(3)]
    opt = SelectiveAdam([{"params": [t], "lr": float(lr)} for t, lr in zip(ps, f["lrs"])],
                        eps=1e-15)
    for step in range(6):
        for i, t in enumerate(ps):
            t.grad = T(f[f"g{step}_{i}"])
        opt.step(T(f[f"mask{step}"]))
    for i, t in enumerate(ps):
        ref = f[f"final{i}"]
        assert np.abs(N(t) - ref).max() < 2e-6 * max(1.0, float(np.abs(ref).max()))
        assert np.array_equal(N(opt.state[t]["steps"]), f[f"steps{i}"])


def test_selective_adam_rows_mask_padding_and_dense_groups(cuda):
    from metal_gauss_b200.selective_adam import SelectiveAdam
    t = torch.ones(12, 2, device="cuda", requires_grad=True)
    aux = torch.randn(4, 3, device="cuda", requires_grad=True)
    aux_ref = aux.detach().clone().requires_grad_(True)
    opt = SelectiveAdam([{"params": [t], "lr": 1e-2}])
    opt.add_param_group({"params": [aux], "lr": 3e-3, "rowwise": False})
    dense = torch.optim.Adam([aux_ref], lr=3e-3, eps=1e-15)
    visible = torch.zeros(8, dtype=torch.bool, device="cuda")
    visible[:3] = True
    for _ in range(3):
        t.grad = torch.ones_like(t)
        aux.grad = torch.randn_like(aux)
        aux_ref.grad = aux.grad.clone()
        opt.step(visible)
        dense.step()
    assert not torch.equal(t[:3], torch.ones_like(t[:3]))
    assert torch.equal(t[3:], torch.ones_like(t[3:]))            # invisible + capacity rows
    assert torch.equal(opt.state[t]["steps"].cpu(),
                       torch.tensor([3.0] * 3 + [0.0] * 9))
    assert torch.allclose(aux, aux_ref, atol=1e-6) and "step" in opt.state[aux]
    with pytest.raises(TypeError):
        opt.step(visible.float())


# ---------------------------------------------------------------- SSIM / loss

def test_ssim_value_and_gradient_match_reference(cuda):
    from metal_gauss_b200.ssim import gaussian_kernel, l1_ssim_loss, ssim
    f = load("ssim")
    ker = gaussian_kernel(device="cuda")
    assert np.abs(N(ker[0, 0, 0]) - f["window"]).max() < 1e-7
    a = T(f["a"]).requires_grad_(True)
    v = ssim(a, T(f["b"]), ker)
    (g,) = torch.autograd.grad(v, a)
    assert abs(float(v) - float(f["ssim"])) < 1e-6
    assert rel_l2(N(g), f["g_ssim"]) < 1e-4
    a2 = T(f["a"]).requires_grad_(True)
    loss = l1_ssim_loss(a2, T(f["b"]), ker)
    (g2,) = torch.autograd.grad(loss, a2)
    assert abs(float(loss) - float(f["loss"])) < 1e-6
    assert rel_l2(N(g2), f["g_loss"]) < 1e-4
    x = torch.rand(80, 80, 3, device="cuda")
    assert abs(float(ssim(x, x, ker)) - 1.0) < 1e-5


@pytest.mark.parametrize("H,W", [(64, 64), (200, 300), (97, 131), (800, 800)])
def test_fused_loss_matches_oracle(cuda, H, W):
    g = np.random.default_rng(H * W)
    x = g.random((H, W, 3)).astype(np.float32)
    y = g.random((H, W, 3)).astype(np.float32)
    ref_loss, ref_grad = oracle.l1_ssim_loss(x, y)
    loss, grad = ext.l1_ssim_loss(T(x), T(y), T(oracle.gaussian_window()))
    assert abs(float(loss) - ref_loss) < 1e-5
    assert rel_l2(N(grad), ref_grad) < 1e-5


def test_device_error_word_is_clear(cuda):
    assert ext.device_error() == 0
