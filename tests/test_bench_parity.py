"""Parity at the configurations the benchmark times, against the CPU oracle
(the reference's algorithm, pinned to fixtures from the reference's own code).

cfg3 is bench.py's workload: 1M Gaussians near the surfaces of 20 ellipsoids,
SH 3, 800x800, hemisphere cameras, the bench's seeded uint8 targets, the
engine's saturation cut on. Two views of one step go through
engine.Trainer.train_step, the public training call: the loss, the
per-Gaussian visibility count, the six parameter-segment gradients
(BASELINE: 1e-3 relative L2) and the selective-Adam update
(selective_adam.py:116-186) are compared with the oracle's. The same step
with the cut off gives a bit-identical loss and gradients within 1e-5.

cfg2 is one training step of the drop-in path the reference's trainer runs
(train.py:381-402): render through cuda_backend.render, 0.8 L1 + 0.2 (1 -
SSIM) through the fused SSIM, backward, then FusedAdam; image, loss and
gradients against the oracle, and the Adam update against the oracle's Adam
on the same gradient.
"""

import numpy as np
import pytest
import torch

import oracle
from metal_gauss_b200 import scenes
from metal_gauss_b200.engine import DEFAULT_LRS, SEGMENTS, Trainer
from tests.golden.fixtures import rel_l2

pytestmark = pytest.mark.gpu

GRAD_TOL = 1e-3   # BASELINE: parameter gradients within 1e-3 relative L2
IMG_TOL = 1e-4    # BASELINE: images within 1e-4 max abs


def _bench_workload(n_views: int):
    """bench.workload()'s scene, views and targets (its first n_views)."""
    p, views, spec = scenes.config("cfg3", n=1_000_000, seed=0)
    g = torch.Generator().manual_seed(1234)
    targets = [torch.randint(0, 256, (v.height, v.width, 3), dtype=torch.uint8, generator=g)
               for v in views[:n_views]]
    return p, views[:n_views], spec, targets


def _oracle_step(params, views, targets, batch, acts=None):
    """Loss, summed gradients in storage form, visibility counts and per-view
    pair counts (the reference's full lists) of a batch of views on the
    oracle, each view's loss and gradient scaled by 1/batch. `acts` =
    (scales, opacities) gives the activated values to project (default:
    numpy's exp / sigmoid of the parameters)."""
    names = [n for n, _ in SEGMENTS]
    acc = {k: np.zeros_like(params[k]) for k in names}
    n = params["means"].shape[0]
    vis = np.zeros(n, np.float32)
    pairs = []
    loss = 0.0
    if acts is None:
        scales = np.exp(params["log_scales"]).astype(np.float32)
        opac = (1 / (1 + np.exp(-params["logit_opac"]))).astype(np.float32)
    else:
        scales, opac = acts
    for v, t in zip(views, targets):
        rgb, _, st = oracle.render(params["means"], params["quats"], scales, opac,
                                   params["sh_dc"], v.K.numpy(), v.viewmat.numpy(), v.width,
                                   v.height, sh_degree=3, sh_rest=params["sh_rest"],
                                   background=None)
        lv, g_rgb = oracle.l1_ssim_loss(rgb, t)
        g = oracle.render_backward(st, (g_rgb / batch).astype(np.float32))
        loss += lv / batch
        acc["means"] += g["means"]
        acc["quats"] += g["quats"]
        acc["log_scales"] += g["scales"] * scales
        acc["logit_opac"] += g["opacities"] * opac * (1 - opac)
        acc["sh_dc"] += g["sh"]
        acc["sh_rest"] += g["sh_rest"]
        vis += st["pre"]["valid"]
        pairs.append(int(st["ids"].size))
    return loss, acc, vis, pairs


@pytest.fixture(scope="module")
def cfg3_two_views():
    p, views, spec, targets_u8 = _bench_workload(2)
    params0 = {k: np.ascontiguousarray(v.numpy(), np.float32) for k, v in p.items()}
    return p, params0, views, targets_u8, spec


def _engine_step(p, views, targets_u8, spec, cut: bool):
    dev = torch.device("cuda:0")
    tr = Trainer(p, dev, sh_degree=3, background=spec["background"], saturation_cut=cut)
    tg = [t.to(dev) for t in targets_u8]   # bytes on the device, as bench.py keeps them
    loss = float(tr.train_step(views, tg, 2))
    torch.cuda.synchronize()
    return tr, loss


def test_bench_step_matches_the_oracle(cuda, cfg3_two_views):
    p, params0, views, targets_u8, spec = cfg3_two_views
    tr, loss = _engine_step(p, views, targets_u8, spec, cut=True)
    # the oracle projects the activations the step projected (its prologue's
    # exp / sigmoid; Adam updates only the stored parameters)
    acts = (tr.scales.cpu().numpy(), tr.opac.cpu().numpy())
    targets = [t.numpy().astype(np.float32) / np.float32(255.0) for t in targets_u8]
    ref_loss, ref_g, ref_vis, ref_pairs = _oracle_step(params0, views, targets, 2, acts)
    assert abs(loss - ref_loss) <= 1e-5 * abs(ref_loss), (loss, ref_loss)
    vis = tr.visibility_count().cpu().numpy()
    assert np.array_equal(vis, ref_vis)
    assert (vis > 0).sum() > 100_000  # the views see a large share of the scene
    for name, _ in SEGMENTS:
        assert rel_l2(tr.grad(name).cpu().numpy(), ref_g[name]) < GRAD_TOL, name
    # the saturation cut removed most of the reference's pairs at this size
    # (which is why parity is checked here and not only on small scenes)
    for s, m_ref in zip(tr.last_stats, ref_pairs):
        assert 0 < s.pairs < 0.5 * m_ref, (s.pairs, m_ref)
    # selective Adam on the engine's own gradient, replayed on the oracle
    vis_u8 = (ref_vis > 0).astype(np.uint8)
    for name, _ in SEGMENTS:
        pp = params0[name].copy()
        m, v = np.zeros_like(pp), np.zeros_like(pp)
        steps = np.zeros(pp.shape[0], np.float32)
        oracle.selective_adam_step(pp, np.ascontiguousarray(tr.grad(name).cpu().numpy()), m, v,
                                   steps, vis_u8, DEFAULT_LRS[name])
        got = tr.param(name).cpu().numpy()
        assert np.abs(got - pp).max() <= 1e-6 * max(1.0, float(np.abs(pp).max())), name
        untouched = ref_vis == 0
        assert np.array_equal(got[untouched], params0[name][untouched]), name
    assert np.array_equal(tr.steps[:tr.n].cpu().numpy(), vis_u8.astype(np.float32))
    tr.check_device_error()


def test_bench_step_without_the_saturation_cut(cuda, cfg3_two_views):
    p, _, views, targets_u8, spec = cfg3_two_views
    cut, lc = _engine_step(p, views, targets_u8, spec, cut=True)
    full, lf = _engine_step(p, views, targets_u8, spec, cut=False)
    assert lc == lf  # each kept list is a front-to-back prefix: same images
    for a, b in zip(full.last_stats, cut.last_stats):
        assert b.pairs < 0.5 * a.pairs, (a.pairs, b.pairs)
    assert torch.equal(cut.visibility_count(), full.visibility_count())
    for name, _ in SEGMENTS:
        assert rel_l2(cut.grad(name).cpu().numpy(), full.grad(name).cpu().numpy()) < 1e-5, name
        assert rel_l2(cut.param(name).cpu().numpy(), full.param(name).cpu().numpy()) < 1e-6, name


def test_cfg2_drop_in_training_step(cuda):
    """One reference training step at cfg2 through the drop-in modules:
    activations (train.py:221-222), render, 0.8 L1 + 0.2 (1 - SSIM)
    (train.py:389-393), backward, FusedAdam with make_optimizer's learning
    rates (train.py:167-191)."""
    from metal_gauss_b200.cuda_backend import render
    from metal_gauss_b200.fused_adam import FusedAdam
    from metal_gauss_b200.ssim import gaussian_kernel, ssim

    p, views, spec = scenes.config("cfg2", seed=0)
    view = views[0]
    W, H = view.width, view.height
    target = scenes.random_target(W, H, 7)
    params0 = {k: np.ascontiguousarray(v.numpy(), np.float32) for k, v in p.items()}

    leaf = {k: v.detach().clone().cuda().requires_grad_(True) for k, v in p.items()}
    opt = FusedAdam([{"params": [leaf[k]], "lr": DEFAULT_LRS[k]} for k, _ in SEGMENTS],
                    eps=1e-15)
    scales, opac = torch.exp(leaf["log_scales"]), torch.sigmoid(leaf["logit_opac"])
    # the oracle projects the same activated values (the device's exp can
    # differ from numpy's in the last bit, which flips 1/255 blend decisions)
    acts = (scales.detach().cpu().numpy(), opac.detach().cpu().numpy())
    ref_loss, ref_g, _, _ = _oracle_step(params0, [view], [target.numpy()], 1, acts)
    ref_rgb, _, _ = oracle.render(params0["means"], params0["quats"], acts[0], acts[1],
                                  params0["sh_dc"], view.K.numpy(), view.viewmat.numpy(), W, H,
                                  sh_degree=3, sh_rest=params0["sh_rest"], background=None)
    rgb, alpha, info = render(leaf["means"], leaf["quats"], scales, opac, leaf["sh_dc"], view.K,
                              view.viewmat, W, H, sh_degree=3, sh_rest=leaf["sh_rest"],
                              background=spec["background"])
    assert np.abs(rgb.detach().cpu().numpy() - ref_rgb).max() < IMG_TOL
    gt = target.cuda()
    loss = 0.8 * (rgb - gt).abs().mean() + 0.2 * (1 - ssim(rgb, gt, gaussian_kernel()))
    assert abs(float(loss.detach()) - ref_loss) <= 1e-5 * abs(ref_loss)
    loss.backward()
    grads = {k: leaf[k].grad.detach().cpu().numpy().copy() for k, _ in SEGMENTS}
    for name, _ in SEGMENTS:
        assert rel_l2(grads[name], ref_g[name]) < GRAD_TOL, name
    opt.step()
    for name, _ in SEGMENTS:
        pp = params0[name].copy()
        m, v = np.zeros_like(pp), np.zeros_like(pp)
        oracle.adam_step(pp, np.ascontiguousarray(grads[name]), m, v, DEFAULT_LRS[name], 0.9,
                         0.999, 1e-15, 1)
        got = leaf[name].detach().cpu().numpy()
        assert np.abs(got - pp).max() <= 1e-6 * max(1.0, float(np.abs(pp).max())), name
    assert info["isect_total"] > 0
