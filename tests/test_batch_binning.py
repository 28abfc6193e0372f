"""Batch binning (mg_bin_prepare_views / mg_bin_emit_views): every view's
gauss ids and tile offsets equal the lists of the per-view calls
(mg_bin_prepare / mg_bin_emit, themselves pinned to the reference's lists),
with and without the saturation cut, with shared and per-view opacities and a
view stride above the Gaussian count; views of wide and narrow depth range in
one batch; and the trainer and renderer give the same results
either way."""

import numpy as np
import pytest
import torch

from metal_gauss_b200 import _lib, scenes
from metal_gauss_b200._lib import ptr
from metal_gauss_b200.engine import Trainer
from metal_gauss_b200.renderer import Renderer
from tests.golden.fixtures import rel_l2
from tests.test_views import N_G, W, H, _forward_views, _scene

pytestmark = pytest.mark.gpu

TILE = 16
TX, TY = -(-W // TILE), -(-H // TILE)
N_TILES = TX * TY


def _per_view(out, v, n, opac, cut):
    L = _lib.load()
    s = _lib.stream()
    tot = torch.zeros(1, dtype=torch.int64, device="cuda")
    prep = torch.empty(L.mg_bin_prepare_scratch_bytes(n, N_TILES), dtype=torch.uint8,
                       device="cuda")
    _lib.call("mg_bin_prepare", ptr(out["uv"][v]), ptr(out["rxy"][v]), ptr(out["conic"][v]),
              ptr(opac), ptr(out["valid"][v]), ptr(out["depth"][v]), n, W, H, TILE, cut,
              ptr(tot), ptr(prep), prep.numel(), s)
    m = int(tot.item())
    ids = torch.empty(max(m, 1), dtype=torch.int32, device="cuda")
    off = torch.empty(N_TILES + 1, dtype=torch.int32, device="cuda")
    emit = torch.empty(L.mg_bin_emit_scratch_bytes(n, m, N_TILES), dtype=torch.uint8,
                       device="cuda")
    _lib.call("mg_bin_emit", ptr(out["uv"][v]), ptr(out["rxy"][v]), ptr(out["conic"][v]),
              ptr(opac), n, m, W, H, TILE, cut, ptr(prep), ptr(ids), ptr(off), ptr(emit),
              emit.numel(), s)
    return ids[:m].cpu().numpy(), off.cpu().numpy()


def _batch(out, V, n, stride, opac, opac_stride, cut):
    L = _lib.load()
    s = _lib.stream()
    tot = torch.zeros(V + 2, dtype=torch.int64, device="cuda")
    prep = torch.empty(L.mg_bin_prepare_views_scratch_bytes(n, V, N_TILES), dtype=torch.uint8,
                       device="cuda")
    _lib.call("mg_bin_prepare_views", ptr(out["uv"]), ptr(out["rxy"]), ptr(out["conic"]),
              ptr(opac), ptr(out["valid"]), ptr(out["depth"]), n, V, stride, opac_stride, W, H,
              TILE, cut, ptr(tot), ptr(prep), prep.numel(), s)
    t = tot.cpu().numpy()
    assert t[V + 1] == 0
    assert t[V] == t[:V].sum()
    m = int(t[V])
    ids = torch.empty(max(m, 1), dtype=torch.int32, device="cuda")
    off = torch.empty(V * (N_TILES + 1), dtype=torch.int32, device="cuda")
    emit = torch.empty(L.mg_bin_emit_views_scratch_bytes(n, V, m, N_TILES), dtype=torch.uint8,
                       device="cuda")
    _lib.call("mg_bin_emit_views", ptr(out["uv"]), ptr(out["rxy"]), ptr(out["conic"]), ptr(opac),
              n, V, stride, opac_stride, m, W, H, TILE, cut, ptr(prep), ptr(ids), ptr(off),
              ptr(emit), emit.numel(), s)
    ids, off = ids[:m].cpu().numpy(), off.cpu().numpy().reshape(V, N_TILES + 1)
    lists, base = [], 0
    for v in range(V):
        mv = int(t[v])
        lists.append((ids[base:base + mv], off[v]))
        base += mv
    return lists


@pytest.mark.parametrize("cut", [0, 1])
@pytest.mark.parametrize("V", [2, 8, 11])
def test_batch_lists_equal_the_per_view_lists(cuda, cut, V):
    _, d, views = _scene(3, V)
    out = _forward_views(d, views)
    n = N_G - 37  # a view stride above the Gaussian count
    lists = _batch(out, V, n, N_G, d["opac"], 0, cut)
    pairs = 0
    for v in range(V):
        ids, off = _per_view(out, v, n, d["opac"], cut)
        assert np.array_equal(lists[v][0], ids), f"view {v}"
        assert np.array_equal(lists[v][1], off), f"view {v}"
        pairs += ids.size
    assert pairs > 1000 * V


def test_batch_with_per_view_opacities(cuda):
    V = 6
    _, d, views = _scene(4, V)
    out = _forward_views(d, views)
    scale = torch.linspace(0.3, 1.0, V, device="cuda")[:, None]
    opac = (d["opac"][None, :] * scale).contiguous()
    lists = _batch(out, V, N_G, N_G, opac, N_G, 1)
    for v in range(V):
        ids, off = _per_view(out, v, N_G, opac[v], 1)
        assert np.array_equal(lists[v][0], ids) and np.array_equal(lists[v][1], off)
    # dimmer views keep fewer pairs
    assert lists[0][0].size < lists[-1][0].size


def test_views_without_pairs_in_a_batch(cuda):
    V = 4
    _, d, views = _scene(5, V)
    out = _forward_views(d, views)
    out["valid"][1].zero_()
    out["valid"][3].zero_()
    lists = _batch(out, V, N_G, N_G, d["opac"], 0, 1)
    assert lists[1][0].size == 0 and not lists[1][1].any()
    for v in (0, 2):
        ids, off = _per_view(out, v, N_G, d["opac"], 1)
        assert np.array_equal(lists[v][0], ids) and np.array_equal(lists[v][1], off)


def test_wide_depth_ranges_in_a_batch(cuda):
    """The batch's depth sort takes each view's rows as a segment of their
    own, keyed relative to the view's nearest visible depth. A view whose
    depths run from 0.01 to 90 (about 1.1e8 float patterns, past 2^24, so its
    top pass ranks while the other views' copy) among 39 views of narrow range
    gives the lists of its own binning, and so do its neighbours; the word
    after the batch total stays 0."""
    V, n = 40, 512
    g = torch.Generator().manual_seed(0)
    f32 = dict(dtype=torch.float32, device="cuda")
    uv = (torch.rand(V, n, 2, generator=g) * torch.tensor([W, H])).to(**f32)
    rxy = torch.full((V, n, 2), 6.0, **f32)
    conic = torch.tensor([0.05, 0.0, 0.05]).expand(V, n, 3).contiguous().to(**f32)
    valid = torch.ones(V, n, dtype=torch.int32, device="cuda")
    opac = torch.full((n,), 0.8, **f32)
    for lo, hi in ((0.5, 8.0), (0.01, 90.0)):
        depth = torch.linspace(2.0, 3.0, n).expand(V, n).contiguous().to(**f32)
        depth[17] = torch.linspace(lo, hi, n, **f32).flip(0)
        out = dict(uv=uv, rxy=rxy, conic=conic, valid=valid, depth=depth)
        for cut in (0, 1):
            lists = _batch(out, V, n, n, opac, 0, cut)
            for v in (0, 16, 17, 18, 39):
                ids, off = _per_view(out, v, n, opac, cut)
                assert np.array_equal(lists[v][0], ids), (lo, cut, v)
                assert np.array_equal(lists[v][1], off), (lo, cut, v)


def test_batch_entry_points_refuse_bad_arguments(cuda):
    L = _lib.load()
    tot = torch.zeros(4, dtype=torch.int64, device="cuda")
    buf = torch.empty(1024, dtype=torch.uint8, device="cuda")
    assert L.mg_bin_prepare_views(None, None, None, None, None, None, 10, 65, 10, 0, W, H, TILE,
                                  0, ptr(tot), ptr(buf), 1024, None) != 0
    assert L.mg_bin_prepare_views(None, None, None, None, None, None, 10, 2, 5, 0, W, H, TILE,
                                  0, ptr(tot), ptr(buf), 1024, None) != 0
    assert L.mg_bin_prepare_views(None, None, None, None, None, None, 10, 2, 10, 0, W, H, TILE,
                                  0, ptr(tot), ptr(buf), 16, None) != 0


def _trainer_run(p, views, targets, batch_binning, view_streams, bin_chunk):
    tr = Trainer({k: v.clone() for k, v in p.items()}, "cuda", sh_degree=3)
    tr.batch_binning, tr.view_streams, tr.bin_chunk = batch_binning, view_streams, bin_chunk
    tr._activate()
    stats = tr.forward_backward_views(views, targets, 1.0 / len(views))
    torch.cuda.synchronize()
    return tr, stats


@pytest.mark.parametrize("bb,streams,chunk", [(True, 3, 0), (True, 2, 2), (True, 1, 3),
                                              (False, 3, 0)])
def test_trainer_binning_and_streams_change_nothing(cuda, bb, streams, chunk):
    """Batch binning (whole step or chunks), and the view chains on several
    streams, against one view at a time on one stream."""
    p, _, _ = scenes.config("cfg3", n=N_G, seed=8)
    views = scenes.sphere_views(5, 4.0, W, H, 40.0, 9, hemisphere=True)
    g = torch.Generator().manual_seed(1)
    targets = [torch.rand(H, W, 3, generator=g).cuda() for _ in views]
    a, sa = _trainer_run(p, views, targets, bb, streams, chunk)
    b, sb = _trainer_run(p, views, targets, False, 1, 0)
    assert [s.pairs for s in sa] == [s.pairs for s in sb]
    assert float(a.loss.sum()) == pytest.approx(float(b.loss.sum()), rel=1e-6)
    for name in ("means", "quats", "log_scales", "logit_opac", "sh_dc", "sh_rest"):
        assert rel_l2(a.grad(name).cpu().numpy(), b.grad(name).cpu().numpy()) < 1e-5, name


def test_renderer_batch_binning_changes_nothing(cuda):
    p, _, _ = scenes.config("cfg3", n=N_G, seed=10)
    views = scenes.sphere_views(6, 4.0, W, H, 40.0, 11, hemisphere=True)
    outs = []
    for bb, streams in ((True, 3), (False, 1)):
        r = Renderer(p, "cuda", batch=4, antialias=True)
        r.batch_binning, r.view_streams = bb, streams
        outs.append(r.render(views))
    for (ra, aa), (rb, ab) in zip(*outs):
        assert torch.equal(ra, rb) and torch.equal(aa, ab)


def test_trainer_mixed_frame_sizes_bin_view_by_view(cuda):
    """Views of two sizes in one step: no batch binning (one frame size per
    batch), per-size frame buffers on the streams; the same results as one
    view at a time on one stream."""
    p, _, _ = scenes.config("cfg3", n=N_G, seed=12)
    views = (scenes.sphere_views(3, 4.0, W, H, 40.0, 13, hemisphere=True) +
             scenes.sphere_views(2, 4.0, 96, 64, 40.0, 14, hemisphere=True))
    g = torch.Generator().manual_seed(2)
    targets = [torch.rand(v.height, v.width, 3, generator=g).cuda() for v in views]
    a, sa = _trainer_run(p, views, targets, True, 4, 0)
    b, sb = _trainer_run(p, views, targets, False, 1, 0)
    assert [s.pairs for s in sa] == [s.pairs for s in sb]
    assert not a._bbs  # never batch-binned
    assert float(a.loss.sum()) == pytest.approx(float(b.loss.sum()), rel=1e-6)
    for name in ("means", "quats", "log_scales", "logit_opac", "sh_dc", "sh_rest"):
        assert rel_l2(a.grad(name).cpu().numpy(), b.grad(name).cpu().numpy()) < 1e-5, name
