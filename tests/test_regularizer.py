"""The MCMC regularisers of the reference's training loss (train.py:393-398):
mg_regularizer_grad against a plain torch fp32 expression of
aux * (opac_reg * mean(sigmoid(logit)) + scale_reg * mean(exp(log_scales)))
and its gradient, and the trainer's step with them against the step without
(the difference is exactly the regularisers' value and gradient)."""

import numpy as np
import pytest
import torch

from metal_gauss_b200 import _lib, scenes
from metal_gauss_b200._lib import ptr
from metal_gauss_b200.engine import Trainer
from tests.golden.fixtures import rel_l2

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n", [1, 1000, 300_001])
def test_regularizer_matches_torch(cuda, n):
    g = torch.Generator().manual_seed(n)
    logit = torch.randn(n, generator=g).cuda()
    ls = (torch.randn(n, 3, generator=g) - 3.0).cuda()
    c_o, c_s = 0.7 * 0.01, 0.7 * 0.02
    d_logit = torch.full((n,), 0.25, device="cuda")
    d_ls = torch.full((n, 3), -0.5, device="cuda")
    loss = torch.full((1,), 2.0, device="cuda")
    scratch = torch.empty(16, dtype=torch.uint8, device="cuda")
    _lib.call("mg_regularizer_grad", ptr(logit), ptr(ls), n, c_o, c_s, ptr(d_logit), ptr(d_ls),
              ptr(loss), ptr(scratch), 16, _lib.stream())
    lt = logit.clone().requires_grad_(True)
    st = ls.clone().requires_grad_(True)
    ref = c_o * torch.sigmoid(lt).mean() + c_s * torch.exp(st).mean()
    ref.backward()
    assert float(loss) == pytest.approx(2.0 + float(ref), rel=1e-6)
    # the added terms sit on 0.25 / -0.5: compare within a few ulps of those
    assert torch.allclose(d_logit - 0.25, lt.grad, rtol=1e-5, atol=1e-7)
    assert torch.allclose(d_ls + 0.5, st.grad, rtol=1e-5, atol=1e-7)


def test_regularizer_refuses_bad_arguments(cuda):
    L = _lib.load()
    x = torch.zeros(4, device="cuda")
    assert L.mg_regularizer_grad(ptr(x), ptr(x), 4, 0.1, 0.1, ptr(x), ptr(x), ptr(x), ptr(x), 8,
                                 None) != 0  # scratch too small
    assert L.mg_regularizer_grad(None, ptr(x), 4, 0.1, 0.1, ptr(x), ptr(x), ptr(x), ptr(x), 16,
                                 None) != 0


def test_trainer_step_carries_the_regularisers(cuda):
    n, W, H = 20000, 160, 120
    p, _, _ = scenes.config("cfg3", n=n, seed=21)
    views = scenes.sphere_views(3, 4.0, W, H, 40.0, 22, hemisphere=True)
    g = torch.Generator().manual_seed(3)
    targets = [torch.rand(H, W, 3, generator=g).cuda() for _ in views]

    def run(opac_reg, scale_reg):
        tr = Trainer({k: v.clone() for k, v in p.items()}, "cuda", sh_degree=3,
                     opac_reg=opac_reg, scale_reg=scale_reg)
        tr.active = n - 123  # the regularisers cover the active rows only
        tr.reg_weight = 0.6
        tr.view_streams = 1
        tr._activate()
        tr.G.zero_()
        tr.forward_backward_views(views, targets, 1.0 / len(views))
        if tr.opac_reg or tr.scale_reg:
            tr._regularize(1)
        torch.cuda.synchronize()
        return tr

    a, b = run(0.01, 0.02), run(0.0, 0.0)
    act = n - 123
    logit = p["logit_opac"][:act].float().cuda().requires_grad_(True)
    ls = p["log_scales"][:act].float().cuda().requires_grad_(True)
    ref = 0.6 * (0.01 * torch.sigmoid(logit).mean() + 0.02 * torch.exp(ls).mean())
    ref.backward()
    assert float(a.loss) - float(b.loss) == pytest.approx(float(ref), rel=1e-4)
    d_logit = (a.grad("logit_opac") - b.grad("logit_opac"))[:act]
    d_ls = (a.grad("log_scales") - b.grad("log_scales"))[:act]
    assert rel_l2(d_logit.cpu().numpy(), logit.grad.cpu().numpy()) < 1e-3
    assert rel_l2(d_ls.cpu().numpy(), ls.grad.cpu().numpy()) < 1e-3
    # rows past the active count are untouched
    assert torch.equal(a.grad("logit_opac")[act:], b.grad("logit_opac")[act:])
    assert np.isfinite(float(a.loss))
