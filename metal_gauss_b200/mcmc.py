"""3DGS-MCMC densification on the GPU (drop-in for metal_gauss/mcmc.py).

`relocate`, `grow` and `add_noise` keep the reference's signatures and
semantics (mcmc.py:52-192): dead Gaussians move onto live ones drawn in
proportion to `weights` (opacity by default) with the multiplicity
corrections of an n-way split applied to copies and targets, growth clones
drawn rows into the preallocated tail, and the exploration noise moves
near-transparent means along their own axes. The work runs in
`libmg_b200.so` over the parameter dict's rows and the optimizer's moment and
step rows (`reset_adam_state`'s rows are zeroed inside the same kernels).

The draws come from the library's counter-based generator with a seed taken
from torch's default generator, so `torch.manual_seed` makes a run
reproducible, but the draws are not torch.multinomial's / torch.randn's.
`picks` / `eps` fix them (what the parity tests use).
"""

from __future__ import annotations

import torch

from . import _lib
from ._lib import ptr

MAX_MULTIPLICITY = 51
_CORRECTED = ("logit_opac", "log_scales")


def _seed(seed) -> int:
    if seed is not None:
        return int(seed) & ((1 << 64) - 1)
    return int(torch.randint(0, 2 ** 62, (1,)).item())


def _segments(params: dict):
    keys = list(params)
    if "logit_opac" not in params or "log_scales" not in params:
        raise KeyError("MCMC needs 'logit_opac' and 'log_scales' parameters")
    n = params["logit_opac"].shape[0]
    segs = []
    for k in keys:
        t = params[k]
        if t.device.type != "cuda" or t.dtype != torch.float32 or not t.is_contiguous():
            raise RuntimeError(f"MCMC on the CUDA backend needs contiguous float32 CUDA tensors "
                               f"('{k}')")
        if t.shape[0] != n:
            raise ValueError(f"parameter '{k}' has {t.shape[0]} rows, expected {n}")
        segs.append(_lib.RowSegment(t.data_ptr(), int(t[0].numel()) if n else 1))
    arr = (_lib.RowSegment * len(segs))(*segs)
    return arr, len(segs), keys.index("logit_opac"), keys.index("log_scales"), n


def _opt_rows(opt, params: dict):
    rows = []
    if opt is not None:
        for t in params.values():
            st = opt.state.get(t)
            if not st:
                continue
            for key in ("exp_avg", "exp_avg_sq"):
                if key in st:
                    rows.append(_lib.RowSegment(st[key].data_ptr(), int(st[key][0].numel())))
            if "steps" in st:
                rows.append(_lib.RowSegment(st["steps"].data_ptr(), 1))
    return (_lib.RowSegment * max(1, len(rows)))(*rows), len(rows)


def _scratch(n: int, device) -> torch.Tensor:
    return torch.empty(_lib.load().mg_mcmc_scratch_bytes(n), dtype=torch.uint8, device=device)


def _weights(weights, n, device):
    if weights is None:
        return None
    return weights[:n].detach().to(device, torch.float32).contiguous()


@torch.no_grad()
def relocate(params: dict, dead_thresh: float = 0.005, opt=None, active: int | None = None,
             weights: torch.Tensor | None = None, seed: int | None = None,
             picks: torch.Tensor | None = None) -> int:
    """Move dead Gaussians (opacity < dead_thresh among the first `active`)
    onto live ones; zeroes the optimizer rows of every changed row. Returns
    how many moved."""
    segs, ns, il, isc, n = _segments(params)
    n_act = n if active is None else int(active)
    rows, nr = _opt_rows(opt, params)
    dev = params["logit_opac"].device
    w = _weights(weights, n_act, dev)
    pk = None if picks is None else picks.to(dev, torch.int32).contiguous()
    scratch = _scratch(n_act, dev)
    moved = _lib.C.c_int64(0)
    _lib.call("mg_mcmc_relocate", segs, ns, il, isc, rows, nr, n_act, float(dead_thresh), ptr(w),
              ptr(pk), _seed(seed), _lib.C.byref(moved), ptr(scratch), scratch.numel(),
              _lib.stream())
    return int(moved.value)


@torch.no_grad()
def grow(params: dict, target: int, active: int, opt=None,
         weights: torch.Tensor | None = None, seed: int | None = None,
         picks: torch.Tensor | None = None) -> int:
    """Activate Gaussians [active, target) by cloning weight-sampled live ones
    (parameters preallocated at the cap). Returns the new active count."""
    segs, ns, il, isc, n = _segments(params)
    rows, nr = _opt_rows(opt, params)
    dev = params["logit_opac"].device
    w = _weights(weights, int(active), dev)
    pk = None if picks is None else picks.to(dev, torch.int32).contiguous()
    scratch = _scratch(n, dev)
    out = _lib.C.c_int64(0)
    _lib.call("mg_mcmc_grow", segs, ns, il, isc, rows, nr, int(active), int(target), n, ptr(w),
              ptr(pk), _seed(seed), _lib.C.byref(out), ptr(scratch), scratch.numel(),
              _lib.stream())
    return int(out.value)


@torch.no_grad()
def add_noise(params: dict, lr_means: float, weight: float = 4e4, active: int | None = None,
              opacity_gate: float = 0.005, seed: int | None = None,
              eps: torch.Tensor | None = None) -> None:
    """SGLD-style exploration on the means of near-transparent Gaussians,
    drawn in each Gaussian's own frame and proportional to the current means
    learning rate."""
    n = params["means"].shape[0] if active is None else int(active)
    for k in ("means", "quats", "log_scales", "logit_opac"):
        t = params[k]
        if t.device.type != "cuda" or t.dtype != torch.float32 or not t.is_contiguous():
            raise RuntimeError(f"add_noise on the CUDA backend needs contiguous float32 CUDA "
                               f"tensors ('{k}')")
    e = None if eps is None else eps[:n].to(params["means"].device, torch.float32).contiguous()
    _lib.call("mg_mcmc_add_noise", ptr(params["means"]), ptr(params["quats"]),
              ptr(params["log_scales"]), ptr(params["logit_opac"]), n, float(lr_means),
              float(weight), float(opacity_gate), _seed(seed), ptr(e), _lib.stream())


@torch.no_grad()
def reset_adam_state(opt, params: dict, idx: torch.Tensor) -> None:
    """Zero the Adam moments (and per-row step counts) of rows `idx`
    (mcmc.py:107-121); relocate and grow already do this for their rows."""
    for t in params.values():
        st = opt.state.get(t)
        if not st:
            continue
        for key in ("exp_avg", "exp_avg_sq"):
            if key in st:
                st[key][idx] = 0.0
        if "steps" in st:
            st["steps"][idx] = 0.0
