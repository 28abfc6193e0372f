"""engine.fit's host-side schedule on the CPU, with a stand-in trainer that
records what fit asks of it: the views of each step (epoch permutations of
numpy's default_rng(seed), sharded over ranks), the means learning-rate decay,
the SH warm-up, the loss regularisers' weights and ramp (train.py:393-398),
and the 3D-filter / noise / relocation / growth calls (train.py:343-462)."""

import numpy as np
import pytest
import torch

from metal_gauss_b200.engine import fit


class _View:
    def __init__(self, i):
        self.i, self.width, self.height = i, 4, 3


class _Recorder:
    """The trainer surface fit uses, recording every call."""

    def __init__(self, rank=0, world=1, active=100):
        self.lrs = {"means": 1e-2}
        self.rank, self.world = rank, world
        self.active = active
        self.device = torch.device("cpu")
        self.sh_degree = 3
        self.opac_reg = self.scale_reg = 0.0
        self.reg_weight = 1.0
        self.steps, self.events = [], []

    def train_step(self, views, targets, global_batch):
        # host images go to the trainer as they are (bytes stay bytes)
        assert all(t.device.type == "cpu" and (t.dtype == torch.uint8 or float(t.max()) <= 1.0)
                   for t in targets)
        self.steps.append(dict(views=[v.i for v in views], lr=self.lrs["means"],
                               sh=self.sh_degree, reg=(self.opac_reg, self.scale_reg,
                                                       self.reg_weight), batch=global_batch))
        return torch.tensor([0.5 + len(self.steps)])

    def compute_filter_3d(self, views):
        self.events.append(("filter", len(self.steps) + 1))

    def add_noise(self, lr, weight):
        self.events.append(("noise", len(self.steps), lr, weight))

    def relocate(self):
        self.events.append(("relocate", len(self.steps)))

    def grow(self, target):
        self.events.append(("grow", len(self.steps), target))
        self.active = target
        return target

    def check_device_error(self):
        self.events.append(("device_error_check", len(self.steps)))


def _targets(n):
    return [np.full((3, 4, 3), 255, np.uint8) for _ in range(n)]


def test_views_lr_sh_and_regularisers():
    views = [_View(i) for i in range(5)]
    tr = _Recorder()
    losses = fit(tr, views, _targets(5), steps=10, batch=2, seed=7, lr_means_end=1e-4,
                 sh_warmup=3)
    assert losses == [1.5 + k for k in range(10)]
    # epoch permutations: every view once per epoch, a new permutation when used up
    rng = np.random.default_rng(7)
    order, oi, want = rng.permutation(5), 0, []
    for _ in range(10):
        step = []
        while len(step) < 2:
            if oi >= len(order):
                order, oi = rng.permutation(5), 0
            step.append(int(order[oi]))
            oi += 1
        want.append(step)
    assert [s["views"] for s in tr.steps] == want
    # geometric decay to lr_means_end at the last step
    lrs = [s["lr"] for s in tr.steps]
    assert lrs[-1] == pytest.approx(1e-4, rel=1e-9)
    assert all(a > b for a, b in zip(lrs, lrs[1:]))
    assert [s["sh"] for s in tr.steps] == [0, 0, 1, 1, 1, 2, 2, 2, 3, 3]
    # the reference's regularisers (0.01 / 0.01), ramped by max(0, 1 - step / (0.9 steps))
    for k, s in enumerate(tr.steps, start=1):
        o, c, w = s["reg"]
        assert (o, c) == (0.01, 0.01)
        assert w == pytest.approx(max(0.0, 1.0 - k / 9.0))
    assert tr.steps[-1]["reg"][2] == 0.0
    assert all(s["batch"] == 2 for s in tr.steps)


def test_regularisers_can_be_turned_off():
    tr = _Recorder()
    fit(tr, [_View(i) for i in range(3)], _targets(3), steps=2, batch=1, opac_reg=0.0,
        scale_reg=0.0)
    assert all(s["reg"][:2] == (0.0, 0.0) for s in tr.steps)


def test_ranks_render_their_share_of_the_same_batches():
    views = [_View(i) for i in range(6)]
    ranks = [_Recorder(rank=r, world=2) for r in range(2)]
    for tr in ranks:
        fit(tr, views, _targets(6), steps=4, batch=4, seed=3)
    single = _Recorder()
    fit(single, views, _targets(6), steps=4, batch=4, seed=3)
    for k in range(4):
        assert ranks[0].steps[k]["views"] + ranks[1].steps[k]["views"] == single.steps[k]["views"]
        assert ranks[0].steps[k]["batch"] == 4


def test_filter_noise_relocation_and_growth_schedule():
    views = [_View(i) for i in range(4)]
    tr = _Recorder(active=100)
    fit(tr, views, _targets(4), steps=10, batch=1, filter_3d_every=4, noise_weight=4e4,
        relocate_every=2, relocate_until=7, grow_to=200, grow_until=8)
    filt = [e[1] for e in tr.events if e[0] == "filter"]
    assert filt == [1, 4, 8]
    noise = [e for e in tr.events if e[0] == "noise"]
    assert [e[1] for e in noise] == list(range(1, 11)) and all(e[3] == 4e4 for e in noise)
    assert [e[1] for e in tr.events if e[0] == "relocate"] == [2, 4, 6]
    grow = [(e[1], e[2]) for e in tr.events if e[0] == "grow"]
    # growth on relocation steps up to grow_until, toward grow_to linearly
    assert grow == [(2, 125), (4, 150), (6, 175), (8, 200)]
    # the run ends with a synchronising check of the device error word, so a
    # failure in the last step's kernels is not returned as a result
    assert tr.events[-1] == ("device_error_check", 10)


def test_a_step_refuses_more_views_than_the_adjoint_table_holds():
    from metal_gauss_b200.engine import MAX_VIEWS_PER_STEP, Trainer
    with pytest.raises(ValueError, match="views per rank"):
        Trainer.forward_backward_views(object(), [None] * (MAX_VIEWS_PER_STEP + 1), [], 1.0)
