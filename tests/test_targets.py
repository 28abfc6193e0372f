"""Targets as the reference's trainer holds them: 8-bit images divided by 255
(`v.image.to(device).float() / 255.0`, train.py:385). mg_l1_ssim_loss_u8
reads the bytes and must equal mg_l1_ssim_loss on x / 255 (IEEE float32
division, as numpy computes it) bit for bit; Trainer.train_step takes the
images as uint8 or float32, on the host (copied on a side stream while the
step bins) or on the device, with identical results."""

import numpy as np
import pytest
import torch

from metal_gauss_b200 import _lib, ext, scenes
from metal_gauss_b200._lib import ptr
from metal_gauss_b200.engine import SEGMENTS, Trainer
from tests.golden.fixtures import rel_l2

pytestmark = pytest.mark.gpu


def _div255(t: torch.Tensor) -> torch.Tensor:
    """x / 255 in float32 with IEEE division (numpy), on t's device."""
    return torch.from_numpy(t.cpu().numpy().astype(np.float32) / np.float32(255.0)).to(t.device)


def _loss(x, y, u8: bool):
    H, W = x.shape[:2]
    L = _lib.load()
    scratch = torch.empty(L.mg_l1_ssim_scratch_bytes(H, W), dtype=torch.uint8, device="cuda")
    win = torch.from_numpy(np.exp(-(np.arange(11) - 5.0) ** 2 / 4.5).astype(np.float32))
    win = (win / win.sum()).cuda()
    grad = torch.empty_like(x)
    loss = torch.zeros(1, device="cuda")
    fn = L.mg_l1_ssim_loss_u8 if u8 else L.mg_l1_ssim_loss
    _lib.check(fn(ptr(x), ptr(y), ptr(win), H, W, 0.8, 0.2, 0.5, ptr(grad), ptr(loss),
                  ptr(scratch), scratch.numel(), _lib.stream()), "loss")
    return loss, grad


@pytest.mark.parametrize("H,W", [(800, 800), (97, 131)])
def test_byte_target_loss_equals_the_float_loss(cuda, H, W):
    g = torch.Generator().manual_seed(H)
    x = torch.rand(H, W, 3, generator=g).cuda()
    y8 = torch.randint(0, 256, (H, W, 3), dtype=torch.uint8, generator=g).cuda()
    lf, gf = _loss(x, _div255(y8), u8=False)
    lb, gb = _loss(x, y8, u8=True)
    assert torch.equal(lf, lb) and torch.equal(gf, gb)
    assert ext.device_error() == 0


def test_train_step_takes_host_bytes(cuda):
    p, _, _ = scenes.config("cfg3", n=30_000, seed=41)
    views = scenes.sphere_views(3, 4.0, 160, 120, 40.0, 42, hemisphere=True)
    g = torch.Generator().manual_seed(41)
    u8 = [torch.randint(0, 256, (120, 160, 3), dtype=torch.uint8, generator=g) for _ in views]
    ref = Trainer(p, cuda, sh_degree=3)
    ref.view_streams = 1      # one stream: the views' losses are added in the same order
    l_ref = [float(ref.train_step(views, [_div255(t.cuda()) for t in u8], 3)) for _ in range(2)]
    tr = Trainer(p, cuda, sh_degree=3)
    tr.view_streams = 1
    pinned = [t.pin_memory() for t in u8]
    l_host = [float(tr.train_step(views, pinned, 3)) for _ in range(2)]
    assert l_host[0] == l_ref[0]      # same images, same targets: the same loss
    # the second step starts from parameters equal up to the order of the
    # rasteriser's float atomics
    assert abs(l_host[1] - l_ref[1]) <= 1e-6 * abs(l_ref[1])
    for name, _ in SEGMENTS:
        assert rel_l2(tr.param(name).cpu().numpy(), ref.param(name).cpu().numpy()) < 1e-6, name
    with pytest.raises(ValueError):
        tr.train_step(views, [t[..., :2] for t in pinned], 3)
