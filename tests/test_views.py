"""Multi-view projection entry points of the training engine:
mg_preprocess_forward_views against the CPU oracle (bit-exact, every view,
including a batch longer than one launch's 16 cameras) and the visibility
count it adds; mg_preprocess_backward_views against the sum of the per-view
mg_preprocess_backward_accumulate calls it replaces."""

import numpy as np
import pytest
import torch

import oracle
from metal_gauss_b200 import _lib, scenes
from metal_gauss_b200._lib import G2D_STRIDE, ptr
from tests.golden.fixtures import rel_l2

pytestmark = pytest.mark.gpu

N_G, W, H = 20000, 160, 120


def _scene(seed, n_views):
    p, _, _ = scenes.config("cfg3", n=N_G, seed=seed)
    views = scenes.sphere_views(n_views, 4.0, W, H, 40.0, seed + 1, hemisphere=True)
    d = {k: v.cuda().float().contiguous() for k, v in p.items()}
    # activations on the host, shared with the oracle bit for bit
    d["scales"] = torch.from_numpy(_scales(p)).cuda()
    d["opac"] = torch.from_numpy(_opac(p)).cuda()
    return p, d, views


def _scales(p):
    return np.exp(p["log_scales"].numpy().astype(np.float32)).astype(np.float32)


def _opac(p):
    x = p["logit_opac"].numpy().astype(np.float32)
    return (1 / (1 + np.exp(-x))).astype(np.float32)


def _cam(view):
    vm = view.viewmat.float()
    K = view.K
    cc = -vm[:3, :3].T @ vm[:3, 3]
    return _lib.make_camera(vm, float(K[0, 0]), float(K[1, 1]), float(K[0, 2]), float(K[1, 2]),
                            view.width, view.height, 0.01, 100.0, 0.3, max(view.width, view.height),
                            cc)


def _forward_views(d, views, vis=None):
    V, n = len(views), N_G
    f32 = dict(dtype=torch.float32, device="cuda")
    out = dict(uv=torch.empty(V, n, 2, **f32), conic=torch.empty(V, n, 3, **f32),
               depth=torch.empty(V, n, **f32), rxy=torch.empty(V, n, 2, **f32),
               valid=torch.empty(V, n, dtype=torch.int32, device="cuda"),
               color=torch.empty(V, n, 3, **f32))
    cams = (_lib.Camera * V)(*[_cam(v) for v in views])
    _lib.call("mg_preprocess_forward_views", ptr(d["means"]), ptr(d["quats"]), ptr(d["scales"]),
              ptr(d["sh_dc"]), ptr(d["sh_rest"]), _lib.SH_SPLIT, ptr(d["opac"]),
              _lib.C.cast(cams, _lib.C.c_void_p), V, 3, n, n, ptr(out["uv"]), ptr(out["conic"]),
              ptr(out["depth"]), ptr(out["rxy"]), ptr(out["valid"]), ptr(out["color"]), ptr(vis),
              None, _lib.stream())
    return out


def test_multi_view_projection_is_bit_exact_with_the_oracle(cuda):
    p, d, views = _scene(31, 3)
    vis = torch.full((N_G,), 2.0, dtype=torch.float32, device="cuda")
    out = _forward_views(d, views, vis)
    pn = {k: v.numpy().astype(np.float32) for k, v in p.items()}
    scales, opac = _scales(p), _opac(p)
    count = np.zeros(N_G, np.float32)
    for v, view in enumerate(views):
        cam = oracle.camera(view.viewmat.numpy(), view.K.numpy(), W, H)
        ref = oracle.preprocess_forward(pn["means"], pn["quats"], scales, pn["sh_dc"],
                                        pn["sh_rest"], opac, cam, 3)
        for name in ("uv", "conic", "depth", "rxy", "valid", "color"):
            got = out[name][v].cpu().numpy()
            assert np.array_equal(got, ref[name].reshape(got.shape)), (v, name)
        count += ref["valid"]
        assert ref["valid"].sum() > 1000
    assert np.array_equal(vis.cpu().numpy(), 2.0 + count)


def test_more_views_than_one_launch_carries(cuda):
    """18 views (two launches of at most 16 cameras) equal the single-view
    entry point view by view."""
    _, d, views = _scene(33, 18)
    out = _forward_views(d, views)
    for v, view in enumerate(views):
        one = _forward_views(d, [view])
        for name in one:
            assert torch.equal(out[name][v], one[name][0]), (v, name)


def test_multi_view_adjoint_equals_the_per_view_sum(cuda):
    _, d, views = _scene(35, 3)
    V, n = len(views), N_G
    fw = _forward_views(d, views)
    g = torch.Generator(device="cuda").manual_seed(5)
    grad2d = torch.randn(V, n, G2D_STRIDE, device="cuda", generator=g) * 1e-3
    grad2d[fw["valid"] == 0] = 0.0
    cams = [_cam(v) for v in views]

    def zeros():
        return dict(means=torch.zeros(n, 3, device="cuda"), quats=torch.zeros(n, 4, device="cuda"),
                    scales=torch.zeros(n, 3, device="cuda"), logit=torch.zeros(n, device="cuda"))

    ref, ref_dpre = zeros(), torch.empty(V, n, 3, device="cuda")
    for v in range(V):
        _lib.call("mg_preprocess_backward_accumulate", ptr(d["means"]), ptr(d["quats"]),
                  ptr(d["scales"]), ptr(d["opac"]), ptr(d["sh_dc"]), ptr(d["sh_rest"]),
                  ptr(grad2d[v]), ptr(fw["valid"][v]), _lib.C.byref(cams[v]), 3, n,
                  ptr(ref["means"]), ptr(ref["quats"]), ptr(ref["scales"]), ptr(ref["logit"]),
                  None, None, ptr(fw["color"][v]), ptr(ref_dpre[v]), _lib.stream())
    got, dpre = zeros(), torch.empty(V, n, 3, device="cuda")
    arr = (_lib.Camera * V)(*cams)
    _lib.call("mg_preprocess_backward_views", ptr(d["means"]), ptr(d["quats"]), ptr(d["scales"]),
              ptr(d["opac"]), ptr(grad2d), ptr(fw["valid"]), ptr(fw["color"]),
              _lib.C.cast(arr, _lib.C.c_void_p), V, n, n, None, ptr(got["means"]),
              ptr(got["quats"]),
              ptr(got["scales"]), ptr(got["logit"]), ptr(dpre), _lib.stream())
    assert torch.equal(dpre, ref_dpre)
    for k in ref:
        assert float(ref[k].abs().max()) > 0, k
        assert rel_l2(got[k].cpu().numpy(), ref[k].cpu().numpy()) < 1e-6, k


def test_colour_after_the_projection_equals_the_fused_colour(cuda):
    """mg_sh_colour_views (the colour of a projection run without SH, as the
    trainer does on several GPUs so the SH rows can still be in flight) is bit
    for bit the fused projection's colour, for every view, with 0 where a
    Gaussian is not valid."""
    _, d, views = _scene(37, 5)
    fused = _forward_views(d, views)
    V, n = len(views), N_G
    cams = (_lib.Camera * V)(*[_cam(v) for v in views])
    geo = {k: torch.empty_like(v) for k, v in fused.items()}
    _lib.call("mg_preprocess_forward_views", ptr(d["means"]), ptr(d["quats"]), ptr(d["scales"]),
              None, None, _lib.SH_SPLIT, ptr(d["opac"]), _lib.C.cast(cams, _lib.C.c_void_p), V,
              -1, n, n, ptr(geo["uv"]), ptr(geo["conic"]), ptr(geo["depth"]), ptr(geo["rxy"]),
              ptr(geo["valid"]), None, None, None, _lib.stream())
    for name in ("uv", "conic", "depth", "rxy", "valid"):
        assert torch.equal(geo[name], fused[name]), name
    centres = (_lib.C.c_float * (3 * V))()
    for v in range(V):
        centres[3 * v:3 * v + 3] = list(cams[v].cam_center)[:3]
    colour = torch.full((V, n, 3), -1.0, device="cuda")
    _lib.call("mg_sh_colour_views", ptr(d["means"]), ptr(d["sh_dc"]), ptr(d["sh_rest"]),
              _lib.SH_SPLIT, _lib.C.cast(centres, _lib.C.c_void_p), V, 3, n, n,
              ptr(geo["valid"]), ptr(colour), _lib.stream())
    assert torch.equal(colour, fused["color"])
    assert bool((colour[geo["valid"] == 0] == 0).all())


def test_trainer_step_with_the_colour_split_equals_the_fused_step(cuda):
    """The trainer's colour split (projection without SH, colour after the
    binning; the default on several GPUs) gives the same loss and gradients as
    the fused projection on one GPU."""
    from metal_gauss_b200.engine import SEGMENTS, Trainer
    p, _, _ = scenes.config("cfg3", n=N_G, seed=39)
    views = scenes.sphere_views(3, 4.0, W, H, 40.0, 40, hemisphere=True)
    g = np.random.default_rng(39)
    targets = [torch.from_numpy(g.random((H, W, 3)).astype(np.float32)).cuda() for _ in views]
    fused = Trainer(p, cuda, sh_degree=3)
    split = Trainer(p, cuda, sh_degree=3)
    split.split_colour = True
    lf = float(fused.train_step(views, targets, 3))
    ls = float(split.train_step(views, targets, 3))
    # the images are identical; the views' losses are added in stream order
    assert abs(lf - ls) <= 1e-6 * abs(lf)
    assert torch.equal(fused._batch.color[:3], split._batch.color[:3])
    for name, _ in SEGMENTS:   # up to the order of the rasteriser's float atomics
        assert rel_l2(split.grad(name).cpu().numpy(), fused.grad(name).cpu().numpy()) < 1e-5, name
        # (Adam's first step follows the gradient's sign, so near-zero rows
        # may move either way: held to 1e-5 like the gradients)
        assert rel_l2(split.param(name).cpu().numpy(), fused.param(name).cpu().numpy()) < 1e-5, name
