"""Mip-Splatting's 3D filter on the GPU: mg_compute_3d_filter and
mg_apply_3d_filter (+ adjoint) against the reference's own values
(tests/golden/filter3d.npz, made by its mipfilter.py), and the training
engine with a filter set: its gradients against the CPU oracle carried
through the filter's adjoint (BASELINE: 1e-3 relative L2)."""

import numpy as np
import pytest
import torch

import oracle
from metal_gauss_b200 import mipfilter, scenes
from metal_gauss_b200.engine import SEGMENTS, Trainer
from tests.golden.fixtures import load, rel_l2

pytestmark = pytest.mark.gpu


class _View:
    def __init__(self, K, vm, w, h):
        self.K, self.viewmat = torch.from_numpy(K), torch.from_numpy(vm)
        self.width, self.height = int(w), int(h)


def test_compute_3d_filter_matches_reference(cuda):
    f = load("filter3d")
    views = [_View(K, vm, w, h) for K, vm, (w, h) in zip(f["K"], f["viewmat"], f["wh"])]
    got = mipfilter.compute_3d_filter(torch.from_numpy(f["means"]).cuda(), views).cpu().numpy()
    assert np.abs(got - f["filter"]).max() <= 1e-6 * float(f["filter"].max())
    assert np.all(got[:5] == got.max())


def test_apply_3d_filter_and_its_gradient_match_reference(cuda):
    f = load("filter3d")
    s = torch.from_numpy(f["scales"]).cuda().requires_grad_(True)
    o = torch.from_numpy(f["opac"]).cuda().requires_grad_(True)
    ns, no = mipfilter.apply_3d_filter(s, o, torch.from_numpy(f["filter"]).cuda())
    assert np.abs(ns.detach().cpu().numpy() - f["new_scales"]).max() < 1e-6
    assert np.abs(no.detach().cpu().numpy() - f["new_opac"]).max() < 1e-6
    ((ns * torch.from_numpy(f["g_scales"]).cuda()).sum()
     + (no * torch.from_numpy(f["g_opac"]).cuda()).sum()).backward()
    assert rel_l2(s.grad.cpu().numpy(), f["d_scales"]) < 1e-5
    assert rel_l2(o.grad.cpu().numpy(), f["d_opac"]) < 1e-5


def test_engine_step_with_the_3d_filter_matches_oracle(cuda):
    N, W, H = 20000, 160, 120
    p, _, _ = scenes.config("cfg3", n=N, seed=41)
    views = scenes.sphere_views(3, 4.0, W, H, 40.0, 42, hemisphere=True)
    g = np.random.default_rng(41)
    targets = [g.random((H, W, 3)).astype(np.float32) for _ in views[:2]]
    tr = Trainer(p, cuda, sh_degree=3)
    filt = tr.compute_filter_3d(views).cpu().numpy()
    pn = {k: v.numpy().astype(np.float32).copy() for k, v in p.items()}
    ref_f = oracle.compute_3d_filter(pn["means"], [(v.K.numpy(), v.viewmat.numpy(), W, H)
                                                   for v in views])
    assert np.abs(filt - ref_f).max() <= 1e-6 * float(ref_f.max())
    tr.train_step(views[:2], [torch.from_numpy(t).cuda() for t in targets], 2)

    scales = np.exp(pn["log_scales"]).astype(np.float32)
    opac = (1 / (1 + np.exp(-pn["logit_opac"]))).astype(np.float32)
    fs, fo = oracle.apply_3d_filter(scales, opac, filt)
    acc = {k: np.zeros_like(pn[k]) for k, _ in SEGMENTS}
    for v, t in zip(views[:2], targets):
        rgb, _, st = oracle.render(pn["means"], pn["quats"], fs, fo, pn["sh_dc"], v.K.numpy(),
                                   v.viewmat.numpy(), W, H, sh_degree=3, sh_rest=pn["sh_rest"],
                                   background=None)
        _, g_rgb = oracle.l1_ssim_loss(rgb, t)
        gr = oracle.render_backward(st, (g_rgb / 2).astype(np.float32))
        ds, do = oracle.apply_3d_filter_backward(scales, opac, filt, gr["scales"], gr["opacities"])
        acc["means"] += gr["means"]
        acc["quats"] += gr["quats"]
        acc["log_scales"] += ds * scales
        acc["logit_opac"] += do * opac * (1 - opac)
        acc["sh_dc"] += gr["sh"]
        acc["sh_rest"] += gr["sh_rest"]
    for name, _ in SEGMENTS:
        assert rel_l2(tr.grad(name).cpu().numpy(), acc[name]) < 1e-3, name
    # the filter widens and dims: the filtered activations the forward used
    assert float((tr.scales.cpu() - torch.from_numpy(scales)).min()) >= 0
    assert float((tr.opac.cpu() - torch.from_numpy(opac)).max()) <= 0


def test_renderer_applies_the_3d_filter(cuda):
    N, W, H = 20000, 160, 120
    p, _, _ = scenes.config("cfg3", n=N, seed=43)
    views = scenes.sphere_views(2, 4.0, W, H, 40.0, 44, hemisphere=True)
    from metal_gauss_b200.renderer import Renderer
    tr = Trainer(p, cuda, sh_degree=3)
    filt = tr.compute_filter_3d(views)
    out = Renderer(p, cuda, sh_degree=3, background=None, filter_3d=filt).render(views)
    pn = {k: v.numpy().astype(np.float32) for k, v in p.items()}
    fs, fo = oracle.apply_3d_filter(np.exp(pn["log_scales"]).astype(np.float32),
                                    (1 / (1 + np.exp(-pn["logit_opac"]))).astype(np.float32),
                                    filt.cpu().numpy())
    for (rgb, _), v in zip(out, views):
        ref, _, _ = oracle.render(pn["means"], pn["quats"], fs, fo, pn["sh_dc"], v.K.numpy(),
                                  v.viewmat.numpy(), W, H, sh_degree=3, sh_rest=pn["sh_rest"],
                                  background=None)
        assert np.abs(rgb.cpu().numpy() - ref).max() < 1e-4


def test_filter_when_no_camera_sees_anything(cuda):
    """Every Gaussian behind the camera: all take depth 1, as the reference
    does (mipfilter.py:70-73), and the result matches the oracle."""
    means = torch.zeros(100, 3)
    means[:, 2] = -10.0                                        # camera looks along +z
    K = np.array([[500.0, 0, 80], [0, 500.0, 60], [0, 0, 1]], np.float32)
    vm = np.eye(4, dtype=np.float32)
    got = mipfilter.compute_3d_filter(means.cuda(), [_View(K, vm, 160, 120)]).cpu().numpy()
    ref = oracle.compute_3d_filter(means.numpy(), [(K, vm, 160, 120)])
    assert np.array_equal(got, ref)
    assert np.allclose(got, (1.0 / 500.0) * np.sqrt(0.2), rtol=1e-6)


def test_filter_over_more_cameras_than_one_launch_takes(cuda):
    """150 cameras (three launches of at most 64): the running minimum is
    carried from chunk to chunk and the unseen fill uses the largest final
    minimum, as one pass over all cameras does (the oracle)."""
    N, W, H = 5000, 96, 72
    p, _, _ = scenes.config("cfg3", n=N, seed=43)
    views = scenes.sphere_views(150, 4.0, W, H, 40.0, 44, hemisphere=True)
    means = p["means"].float()
    got = mipfilter.compute_3d_filter(means.cuda(), views).cpu().numpy()
    ref = oracle.compute_3d_filter(means.numpy(), [(v.K.numpy(), v.viewmat.numpy(), W, H)
                                                   for v in views])
    assert np.abs(got - ref).max() <= 1e-6 * float(ref.max())
    # the later chunks matter: the first 64 cameras alone give another filter
    first = mipfilter.compute_3d_filter(means.cuda(), views[:64]).cpu().numpy()
    assert not np.array_equal(first, got)
