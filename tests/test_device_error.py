"""Failure detection on the GPU, exercised without a fault.

The only device-side wait on the training path is the radix sort's decoupled
look-back on a predecessor tile; it is bounded, and a wait that runs out
records code 1 in the device error word and returns. mg_sort_lookback_selftest
launches one onesweep pass whose predecessor never publishes, with a limit of
a few hundred rounds, so the wait runs out on purpose: the kernel must return
promptly, the code must be readable, the context must stay usable, and the
product paths (Trainer.train_step, engine.fit, Renderer.render) must refuse
to continue while the word is set -- the reference refuses rather than
continuing silently (metal_gauss/api.py:18-26).
"""

import time

import numpy as np
import pytest
import torch

from metal_gauss_b200 import _lib, ext, scenes
from metal_gauss_b200._lib import ptr

pytestmark = pytest.mark.gpu


def _trip_lookback(spin_limit: int = 256) -> None:
    L = _lib.load()
    scratch = torch.empty(L.mg_sort_lookback_selftest_scratch_bytes(), dtype=torch.uint8,
                          device="cuda")
    _lib.call("mg_sort_lookback_selftest", spin_limit, ptr(scratch), scratch.numel(),
              _lib.stream())
    torch.cuda.synchronize()


def test_lookback_wait_gives_up_and_records_its_code(cuda):
    assert ext.device_error() == 0
    t0 = time.perf_counter()
    _trip_lookback(256)
    assert time.perf_counter() - t0 < 5.0  # the pass returned
    # peeking copies the word without clearing it; reading clears it
    dst = torch.full((1,), -1, dtype=torch.int64, device="cuda")
    _lib.call("mg_peek_device_error", ptr(dst), _lib.stream())
    assert int(dst.item()) == 1
    assert ext.device_error() == 1
    assert ext.device_error() == 0
    # the context is still usable: a real sort afterwards is exact
    g = torch.Generator(device="cuda").manual_seed(3)
    n = 300_001
    keys = torch.randint(0, 2 ** 31 - 1, (n,), device="cuda", dtype=torch.int64,
                         generator=g).to(torch.int32)
    vals = torch.arange(n, device="cuda", dtype=torch.int32)
    sk, sv = ext.sort_pairs(keys.clone(), vals.clone(), 31)
    order = np.argsort(keys.cpu().numpy(), kind="stable")
    assert np.array_equal(sv.cpu().numpy(), order)
    assert ext.device_error() == 0


def test_selftest_rejects_limits_outside_its_range(cuda):
    L = _lib.load()
    scratch = torch.empty(L.mg_sort_lookback_selftest_scratch_bytes(), dtype=torch.uint8,
                          device="cuda")
    for bad in (0, (1 << 22) + 1):
        with pytest.raises(RuntimeError, match="spin_limit"):
            _lib.call("mg_sort_lookback_selftest", bad, ptr(scratch), scratch.numel(),
                      _lib.stream())
    assert ext.device_error() == 0


def _small_trainer(cuda, **kw):
    from metal_gauss_b200.engine import Trainer
    p, _, _ = scenes.config("cfg3", n=20_000, seed=5)
    views = scenes.sphere_views(2, 4.0, 160, 120, 40.0, 6, hemisphere=True)
    g = np.random.default_rng(5)
    targets = [torch.from_numpy(g.random((120, 160, 3)).astype(np.float32)).cuda()
               for _ in views]
    return Trainer(p, cuda, sh_degree=3, **kw), views, targets


@pytest.mark.parametrize("batch_binning", [True, False])
def test_training_refuses_to_step_over_a_device_error(cuda, batch_binning):
    tr, views, targets = _small_trainer(cuda)
    tr.batch_binning = batch_binning
    float(tr.train_step(views, targets, 2))
    before = tr.state_dict()
    _trip_lookback()
    with pytest.raises(_lib.DeviceError, match="look-back"):
        tr.train_step(views, targets, 2)
    torch.cuda.synchronize()
    # refused before its optimizer step: the parameters are untouched
    for k, v in tr.state_dict().items():
        assert torch.equal(v, before[k]), k
    # the word was cleared by the refusal; training resumes
    assert ext.device_error() == 0
    assert np.isfinite(float(tr.train_step(views, targets, 2)))
    tr.check_device_error()


def test_fit_checks_the_word_after_its_last_step(cuda):
    from metal_gauss_b200.engine import fit
    tr, views, targets = _small_trainer(cuda)

    def trip_after_last(step, loss):
        if step == 2:
            _trip_lookback()

    with pytest.raises(_lib.DeviceError):
        fit(tr, views, [t.cpu() for t in targets], steps=2, batch=2, opac_reg=0.0,
            scale_reg=0.0, callback=trip_after_last)
    assert ext.device_error() == 0


def test_renderer_refuses_to_return_frames_over_a_device_error(cuda):
    from metal_gauss_b200.renderer import Renderer
    p, _, _ = scenes.config("cfg3", n=20_000, seed=8)
    views = scenes.sphere_views(3, 4.0, 160, 120, 40.0, 9, hemisphere=True)
    r = Renderer(p, cuda, sh_degree=3, batch=2)
    assert len(r.render(views)) == 3
    _trip_lookback()
    with pytest.raises(_lib.DeviceError):
        r.render(views)
    assert ext.device_error() == 0
    assert len(r.render(views)) == 3
