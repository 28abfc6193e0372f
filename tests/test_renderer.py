"""The forward-only renderer (renderer.Renderer): images against the CPU
oracle (1e-4 per pixel, with and without the antialias compensation), against
the drop-in `cuda_backend.render` of the same views, and unchanged by the
saturation cut; batches longer than the renderer's batch size."""

import numpy as np
import pytest
import torch

import oracle
from metal_gauss_b200 import cuda_backend, scenes
from metal_gauss_b200.renderer import Renderer

pytestmark = pytest.mark.gpu

N, W, H = 20000, 160, 120


def _scene(seed=21, n=N):
    p, _, _ = scenes.config("cfg3", n=n, seed=seed)
    views = scenes.sphere_views(3, 4.0, W, H, 40.0, seed + 1, hemisphere=True)
    return p, views


@pytest.mark.parametrize("antialias", [False, True])
def test_renderer_matches_oracle(cuda, antialias):
    p, views = _scene()
    r = Renderer(p, cuda, sh_degree=3, antialias=antialias, background=None)
    out = r.render(views)
    pn = {k: v.numpy().astype(np.float32) for k, v in p.items()}
    scales = np.exp(pn["log_scales"]).astype(np.float32)
    opac = (1 / (1 + np.exp(-pn["logit_opac"]))).astype(np.float32)
    for (rgb, alpha), v in zip(out, views):
        ref_rgb, ref_alpha, _ = oracle.render(pn["means"], pn["quats"], scales, opac,
                                              pn["sh_dc"], v.K.numpy(), v.viewmat.numpy(), W, H,
                                              sh_degree=3, sh_rest=pn["sh_rest"],
                                              background=None, antialias=antialias)
        assert np.abs(rgb.cpu().numpy() - ref_rgb).max() < 1e-4
        assert np.abs(alpha.cpu().numpy() - ref_alpha).max() < 1e-4
        assert float(alpha.max()) > 0.5  # the views see the scene


@pytest.mark.parametrize("antialias", [False, True])
def test_renderer_matches_drop_in_render(cuda, antialias):
    p, views = _scene(23)
    bg = (0.25, 0.5, 1.0)
    r = Renderer(p, cuda, sh_degree=3, antialias=antialias, background=bg)
    out = r.render(views)
    d = {k: v.to(cuda) for k, v in p.items()}
    for (rgb, alpha), v in zip(out, views):
        with torch.no_grad():
            ref_rgb, ref_alpha, _ = cuda_backend.render(
                d["means"], d["quats"], torch.exp(d["log_scales"]),
                torch.sigmoid(d["logit_opac"]), d["sh_dc"], v.K, v.viewmat, W, H, sh_degree=3,
                sh_rest=d["sh_rest"], background=bg, antialias=antialias)
        assert (rgb - ref_rgb).abs().max().item() < 1e-5
        assert (alpha - ref_alpha).abs().max().item() < 1e-5


def test_renderer_saturation_cut_keeps_images(cuda):
    """Dense scene of tile-covering Gaussians: the cut list renders the same
    image bit for bit (the dropped pairs lie behind every pixel's stop)."""
    p, _, _ = scenes.config("cfg3", n=100_000, seed=9)
    p["log_scales"] += float(np.log(4.0))
    views = scenes.sphere_views(2, 4.0, 320, 240, 40.0, 10, hemisphere=True)
    full = Renderer(p, cuda, sh_degree=3, saturation_cut=False).render(views)
    cut = Renderer(p, cuda, sh_degree=3, saturation_cut=True).render(views)
    for (a_rgb, a_alpha), (b_rgb, b_alpha) in zip(full, cut):
        assert torch.equal(a_rgb, b_rgb)
        assert torch.equal(a_alpha, b_alpha)


def test_renderer_batches_views(cuda):
    """Seven views through a batch of three (batches of 3, 3, 1) render what
    each view renders alone."""
    p, _ = _scene(25)
    views = scenes.sphere_views(7, 4.0, W, H, 40.0, 26, hemisphere=True)
    r = Renderer(p, cuda, sh_degree=3, batch=3)
    many = r.render(views)
    one = Renderer(p, cuda, sh_degree=3, batch=1)
    for (rgb, alpha), v in zip(many, views):
        (rgb1, alpha1), = one.render([v])
        assert torch.equal(rgb, rgb1)
        assert torch.equal(alpha, alpha1)
