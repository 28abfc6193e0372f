"""3DGS-MCMC on the GPU (metal_gauss_b200.mcmc over mg_mcmc_*): relocate,
grow and add_noise replayed with the reference's own recorded draws
(tests/golden/mcmc.npz) reproduce its parameters, and reset exactly the
optimizer rows reset_adam_state would; the device generator's draws follow
the weights, the noise has the stated scale and the opacity gate."""

import numpy as np
import pytest
import torch

import oracle
from metal_gauss_b200 import mcmc
from tests.golden.fixtures import load

pytestmark = pytest.mark.gpu

KEYS = ("means", "quats", "log_scales", "logit_opac", "sh_dc", "sh_rest")


def _side(f, tag, when):
    return {k: torch.from_numpy(f[f"{tag}_{when}_{k}"]).cuda().contiguous() for k in KEYS}


class _Opt:
    """Optimizer stand-in with SelectiveAdam's state layout."""
    def __init__(self, params):
        self.state = {t: {"exp_avg": torch.ones_like(t), "exp_avg_sq": torch.ones_like(t),
                          "steps": torch.ones(t.shape[0], device=t.device)}
                      for t in params.values()}


def _check_reset(opt, params, rows):
    n = params["means"].shape[0]
    changed = np.zeros(n, bool)
    changed[rows] = True
    for t in params.values():
        st = opt.state[t]
        for key in ("exp_avg", "exp_avg_sq"):
            v = st[key].reshape(n, -1).cpu().numpy()
            assert np.all(v[changed] == 0) and np.all(v[~changed] == 1), key
        s = st["steps"].cpu().numpy()
        assert np.all(s[changed] == 0) and np.all(s[~changed] == 1)


def test_relocate_replays_the_reference(cuda):
    f = load("mcmc")
    p = _side(f, "reloc", "before")
    opt = _Opt(p)
    moved = mcmc.relocate(p, opt=opt, picks=torch.from_numpy(f["reloc_picks"]))
    assert moved == int(f["moved"])
    for k in KEYS:
        assert np.abs(p[k].cpu().numpy() - f[f"reloc_after_{k}"]).max() < 2e-5, k
    _, rows = oracle.mcmc_relocate({k: f[f"reloc_before_{k}"] for k in KEYS}, f["reloc_picks"])
    _check_reset(opt, p, rows)


def test_grow_replays_the_reference(cuda):
    f = load("mcmc")
    p = _side(f, "grow", "before")
    opt = _Opt(p)
    active = mcmc.grow(p, 260, 200, opt=opt, picks=torch.from_numpy(f["grow_picks"]))
    assert active == int(f["new_active"]) == 260
    for k in KEYS:
        assert np.abs(p[k].cpu().numpy() - f[f"grow_after_{k}"]).max() < 2e-5, k
    _, rows = oracle.mcmc_grow({k: f[f"grow_before_{k}"] for k in KEYS}, f["grow_picks"], 260,
                               200)
    _check_reset(opt, p, rows)


def test_add_noise_replays_the_reference(cuda):
    f = load("mcmc")
    p = _side(f, "noise", "before")
    mcmc.add_noise(p, 1.6e-4, 4e4, eps=torch.from_numpy(f["eps"]))
    assert np.abs(p["means"].cpu().numpy() - f["noise_after_means"]).max() < 1e-6
    for k in KEYS[1:]:
        assert torch.equal(p[k].cpu(), torch.from_numpy(f[f"noise_before_{k}"])), k


def _table(n_alive, n_dead, seed):
    g = torch.Generator().manual_seed(seed)
    n = n_alive + n_dead
    p = {"means": torch.zeros(n, 3), "quats": torch.randn(n, 4, generator=g),
         "log_scales": torch.full((n, 3), -3.0), "logit_opac": torch.full((n,), -9.0),
         "sh_dc": torch.zeros(n, 1, 3), "sh_rest": torch.zeros(n, 15, 3)}
    p["means"][:, 0] = torch.arange(n, dtype=torch.float32)   # a row's identity
    p["logit_opac"][:n_alive] = 2.0                            # opacity 0.88: alive
    return {k: v.cuda().contiguous() for k, v in p.items()}


def test_device_draws_follow_the_weights(cuda):
    """100k dead rows relocated onto 8 live rows weighted 1:2:...:8: every
    dead row lands on a live one, in proportion to its weight."""
    n_alive, n_dead = 8, 100_000
    p = _table(n_alive, n_dead, 1)
    w = torch.zeros(n_alive + n_dead, device="cuda")
    w[:n_alive] = torch.arange(1, n_alive + 1, dtype=torch.float32)
    assert mcmc.relocate(p, weights=w, seed=123) == n_dead
    src = p["means"][n_alive:, 0].round().long().cpu()
    hist = torch.bincount(src, minlength=n_alive).double()
    assert int(hist.sum()) == n_dead and hist[n_alive:].sum() == 0
    expect = torch.arange(1, n_alive + 1, dtype=torch.float64) / 36.0 * n_dead
    chi2 = float(((hist[:n_alive] - expect) ** 2 / expect).sum())
    assert chi2 < 30.0, chi2                                   # 7 dof: p < 1e-4
    # multiplicity 51 (the clamp): the copies and the targets are split
    o = torch.sigmoid(p["logit_opac"]).cpu()
    want = 1.0 - (1.0 - torch.sigmoid(torch.tensor(2.0))) ** (1.0 / 51)
    assert torch.allclose(o, torch.full_like(o, float(want)), rtol=1e-4)
    # the same seed draws the same rows
    q = _table(n_alive, n_dead, 1)
    mcmc.relocate(q, weights=w, seed=123)
    assert torch.equal(p["means"], q["means"])


def test_grow_clones_into_the_tail(cuda):
    p = _table(1000, 0, 2)
    cap = 1000
    p = {k: torch.cat([v, torch.zeros((600,) + v.shape[1:], device="cuda")]).contiguous()
         for k, v in p.items()}
    assert mcmc.grow(p, 1500, 1000, seed=7) == 1500
    src = p["means"][1000:1500, 0].round().long()
    assert int(src.min()) >= 0 and int(src.max()) < cap
    assert torch.all(p["logit_opac"][1500:] == 0)                # beyond the target: untouched
    assert mcmc.grow(p, 10_000, 1500, seed=8) == 1600            # clamped to the capacity


def test_noise_scale_and_gate(cuda):
    n = 200_000
    p = {"means": torch.zeros(n, 3), "quats": torch.tensor([[1.0, 0, 0, 0]]).repeat(n, 1),
         "log_scales": torch.full((n, 3), float(np.log(0.01))), "logit_opac": torch.full((n,), -9.0)}
    p["logit_opac"][n // 2:] = 3.0                             # opaque: gated off
    p = {k: v.cuda().contiguous() for k, v in p.items()}
    mcmc.add_noise(p, 1e-4, 4e4, seed=11)
    d = p["means"].cpu()
    low = d[: n // 2]
    o_low = 1.0 / (1.0 + np.exp(9.0))
    gate = 1.0 / (1.0 + np.exp(100.0 * (o_low - 0.005)))
    std = 0.01 * 1e-4 * 4e4 * gate
    assert abs(float(low.mean())) < 0.02 * std
    assert abs(float(low.std()) / std - 1.0) < 0.01
    assert float(d[n // 2:].abs().max()) < 1e-3 * std


# ------------------------------------------------------------ training engine

def _engine_scene(seed=51, n=20000, W=160, H=120):
    from metal_gauss_b200 import scenes
    p, _, _ = scenes.config("cfg3", n=n, seed=seed)
    p["logit_opac"][: n // 10] = -8.0                        # a tenth of the rows are dead
    views = scenes.sphere_views(4, 4.0, W, H, 40.0, seed + 1, hemisphere=True)
    g = np.random.default_rng(seed)
    targets = [torch.from_numpy(g.random((H, W, 3)).astype(np.float32)).cuda() for _ in views]
    return p, views, targets


def test_trainer_relocation_equals_the_drop_in_on_its_buffers(cuda):
    """Trainer.relocate on the flat buffers equals mcmc.relocate on the same
    parameters as a dict, and resets the trainer's Adam rows it changed."""
    from metal_gauss_b200.engine import SEGMENTS, Trainer
    p, views, targets = _engine_scene()
    tr = Trainer(p, cuda, sh_degree=3)
    tr.train_step(views[:2], targets[:2], 2)                  # non-zero Adam state
    d = {name: tr.param(name).clone().contiguous() for name, _ in SEGMENTS}
    opac = torch.sigmoid(d["logit_opac"])
    alive = (opac >= 0.005).nonzero(as_tuple=True)[0]
    n_dead = int((opac < 0.005).sum())
    picks = alive[torch.randint(0, alive.numel(), (n_dead,), device="cuda")]
    assert tr.relocate(picks=picks) == n_dead > 0
    mcmc.relocate(d, picks=picks)
    for name, _ in SEGMENTS:
        assert torch.equal(tr.param(name), d[name]), name
    dead = (opac < 0.005).nonzero(as_tuple=True)[0]
    changed = torch.cat([dead, torch.unique(picks)])
    for name, w in SEGMENTS:
        o = tr.offsets[name]
        m = tr.M[o:o + w * tr.n].view(tr.n, w)
        assert float(m[changed].abs().max()) == 0.0, name
    assert float(tr.steps[changed].abs().max()) == 0.0


def test_inactive_rows_are_not_rendered(cuda):
    """With active = k the trainer renders and differentiates only the first
    k rows: the same loss and gradients as a trainer holding only those."""
    from metal_gauss_b200.engine import SEGMENTS, Trainer
    from tests.golden.fixtures import rel_l2
    p, views, targets = _engine_scene(53)
    k = 15000
    full = Trainer(p, cuda, sh_degree=3)
    full.active = k
    part = Trainer({name: v[:k] for name, v in p.items()}, cuda, sh_degree=3)
    lf = float(full.train_step(views[:2], targets[:2], 2))
    lp = float(part.train_step(views[:2], targets[:2], 2))
    assert abs(lf - lp) < 1e-6
    for name, _ in SEGMENTS:
        assert rel_l2(full.grad(name)[:k].cpu().numpy(), part.grad(name).cpu().numpy()) < 1e-5
        assert float(full.grad(name)[k:].abs().max()) == 0.0, name


def test_fit_with_mcmc_grows_relocates_and_trains(cuda):
    from metal_gauss_b200.engine import Trainer, fit
    p, views, targets = _engine_scene(55)
    tr = Trainer(p, cuda, sh_degree=3, lrs={"means": 1e-3})
    tr.active = 12000
    losses = fit(tr, views, [t.cpu() for t in targets], steps=6, batch=2, noise_weight=4e4,
                 relocate_every=2, grow_to=20000, grow_until=6)
    assert tr.active == 20000
    assert all(np.isfinite(losses)) and losses[-1] < losses[0]
    opac = torch.sigmoid(tr.param("logit_opac")[: tr.active])
    assert float((opac < 0.005).float().mean()) < 0.05        # the dead tenth was relocated


def test_relocate_and_grow_edge_cases(cuda):
    """No dead rows, no live rows, non-finite weights (the reference falls
    back to opacity), growth to at most the current count: as mcmc.py."""
    p = _table(50, 0, 4)                                       # nothing dead
    before = {k: v.clone() for k, v in p.items()}
    assert mcmc.relocate(p, seed=1) == 0
    assert all(torch.equal(p[k], before[k]) for k in p)
    q = _table(0, 40, 5)                                       # nothing alive
    qb = {k: v.clone() for k, v in q.items()}
    assert mcmc.relocate(q, seed=1) == 0
    assert all(torch.equal(q[k], qb[k]) for k in q)
    r = _table(8, 1000, 6)
    w = torch.full((1008,), float("nan"), device="cuda")      # -> opacity weights
    assert mcmc.relocate(r, weights=w, seed=2) == 1000
    src = r["means"][8:, 0].round().long()
    assert int(src.max()) < 8                                  # all landed on live rows
    s = _table(30, 0, 7)
    sb = {k: v.clone() for k, v in s.items()}
    assert mcmc.grow(s, 20, 30, seed=3) == 30                  # target below active
    assert all(torch.equal(s[k], sb[k]) for k in s)
