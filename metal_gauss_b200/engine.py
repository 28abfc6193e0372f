"""Batched multi-view training step on one or more B200s.

The reference trains one view per step on one device (train.py:352-402).
This engine runs the same per-view math -- render, 0.8 L1 + 0.2 (1 - SSIM),
backward through the rasteriser and the fused preprocess, activation chain,
then selective (or dense) Adam -- over a batch of views, sharded across
ranks when torch.distributed is initialised:

  * every Gaussian parameter lives in ONE flat fp32 buffer in the trainer's
    storage form, 59 floats per Gaussian, as consecutive segments
    means (N,3) | quats (N,4) | log_scales (N,3) | logit_opac (N,) |
    sh_dc (N,1,3) | sh_rest (N,15,3);
  * the gradient buffer has the same segments plus the number of views in
    which each Gaussian was visible and the loss;
  * a step runs in three phases: (A) the projection and SH colour of every
    view in one launch, then the binning of all views of one frame size
    with one call per stage (one depth sort and one tile sort for the
    batch) and one host read of the pair totals; (B) per view, on one of
    `view_streams` CUDA streams in turn, packing, raster forward, fused loss
    and raster backward into the view's packed gradient records, so one
    view's raster tail overlaps the next views' work; (C) the projection and
    SH adjoints of all views in one launch each, ADDING into the flat
    gradient with the exp/sigmoid chain applied, then Adam;
  * the loss of a batch is the mean over its views, so each view's
    gradient is scaled by 1 / (global batch); the MCMC regularisers
    (train.py:393-398) and the antialias compensation (train.py
    --antialias) are options.

With several ranks the optimizer is sharded (ZeRO-1): the visibility counts
and the loss are all-reduced, the parameter gradient is reduce-scattered so
each rank holds the summed gradient of its own chunk, each rank runs Adam on
that chunk only, and the updated parameters are all-gathered, so every rank
again holds the full, identical parameter set for the next step.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from . import _lib, dp, ext
from ._lib import G2D_STRIDE, ptr

# (name, floats per Gaussian)
SEGMENTS = (("means", 3), ("quats", 4), ("log_scales", 3), ("logit_opac", 1), ("sh_dc", 3),
            ("sh_rest", 45))
FLOATS_PER_GAUSSIAN = sum(w for _, w in SEGMENTS)           # 59
SHAPES = {"means": (3,), "quats": (4,), "log_scales": (3,), "logit_opac": (), "sh_dc": (1, 3),
          "sh_rest": (15, 3)}
# views one rank renders per step (the multi-view SH adjoint's camera table)
MAX_VIEWS_PER_STEP = 64
# make_optimizer's learning rates (train.py:167-191) with its defaults
DEFAULT_LRS = {"means": 2e-4, "log_scales": 5e-3, "quats": 1e-3, "logit_opac": 1e-2,
               "sh_dc": 2.5e-3, "sh_rest": 2.5e-3 / 20.0}


@dataclass
class ViewStats:
    visible: int = 0
    pairs: int = 0
    walked: float = 0.0


class _ImageBuffers:
    """Frame scratch of one phase-B stream for one frame size: the views that
    stream renders use it one after another (their order on the stream
    serialises the reuse)."""

    def __init__(self, n: int, W: int, H: int, device):
        f32 = dict(dtype=torch.float32, device=device)
        self.rgb = torch.empty(H, W, 3, **f32)
        self.alpha = torch.empty(H, W, **f32)
        self.T = torch.empty(H, W, **f32)
        self.stop = torch.empty(H, W, dtype=torch.int32, device=device)
        self.grad_rgb = torch.empty(H, W, 3, **f32)
        nbytes = _lib.load().mg_l1_ssim_scratch_bytes(H, W)
        self.loss_scratch = torch.empty(nbytes, dtype=torch.uint8, device=device)
        self.tile_work = None
        self.splats = torch.empty(n, _lib.SPLAT_FLOATS, **f32)
        self.raster = torch.empty(0, dtype=torch.uint8, device=device)
        self.ids = torch.empty(0, dtype=torch.int32, device=device)
        self.offsets = None
        self.emit = torch.empty(0, dtype=torch.uint8, device=device)


class _ViewBatch:
    """View-major projection outputs (and, for training, raster gradient
    records and gated colour gradients) of up to `cap` views: row v * n + g
    belongs to Gaussian g in view v, so one multi-view launch fills or reads
    every view of a batch."""

    def __init__(self, n: int, cap: int, device, grads: bool = True,
                 per_view_opacity: bool = False):
        f32 = dict(dtype=torch.float32, device=device)
        self.n, self.cap = n, cap
        # antialiased training: each view's compensated opacities
        self.opac = torch.empty(cap, n, **f32) if per_view_opacity else None
        self.uv = torch.empty(cap, n, 2, **f32)
        self.conic = torch.empty(cap, n, 3, **f32)
        self.depth = torch.empty(cap, n, **f32)
        self.rxy = torch.empty(cap, n, 2, **f32)
        self.valid = torch.empty(cap, n, dtype=torch.int32, device=device)
        self.color = torch.empty(cap, n, 3, **f32)
        self.grad2d = torch.empty(cap, n, G2D_STRIDE, **f32) if grads else None
        self.dpre = torch.empty(cap, n, 3, **f32) if grads else None


class _ViewState:
    """View v's slice of a _ViewBatch plus its binning scratch, alive from
    phase A (projection + binning preparation of every view) to phase B."""

    def __init__(self, batch: _ViewBatch, v: int, device):
        self.n = batch.n
        self.prep = torch.empty(0, dtype=torch.uint8, device=device)
        self.bind(batch, v)

    def bind(self, batch: _ViewBatch, v: int) -> None:
        self.opac = None if batch.opac is None else batch.opac[v]
        self.uv, self.conic, self.depth = batch.uv[v], batch.conic[v], batch.depth[v]
        self.rxy, self.valid, self.color = batch.rxy[v], batch.valid[v], batch.color[v]
        self.grad2d = None if batch.grad2d is None else batch.grad2d[v]

    def prep_scratch(self, n_tiles: int) -> torch.Tensor:
        nbytes = _lib.load().mg_bin_prepare_scratch_bytes(self.n, n_tiles)
        if self.prep.numel() < nbytes:
            self.prep = torch.empty(nbytes, dtype=torch.uint8, device=self.prep.device)
        return self.prep


class _BatchBinning:
    """Binning of a batch of views of one frame size with one library call
    per stage (mg_bin_prepare_views / mg_bin_emit_views): one depth sort and
    one tile sort for the whole batch instead of one of each per view. View
    v's lists land in ids[base_v, base_v + m_v) with tile offsets from 0, the
    lists the per-view calls give."""

    def __init__(self, device):
        u8 = dict(dtype=torch.uint8, device=device)
        self.device = device
        self.prep = torch.empty(0, **u8)
        self.emit = torch.empty(0, **u8)
        self.ids = torch.empty(0, dtype=torch.int32, device=device)
        self.offsets = torch.empty(0, dtype=torch.int32, device=device)
        # per-view pair totals, the batch total, a reserved word (0) and the
        # device error word (copied in just before the one host read)
        self.totals = torch.zeros(67, dtype=torch.int64, device=device)
        self.bases: list[int] = []

    @staticmethod
    def fits(views, n: int) -> bool:
        """Whether views of n Gaussians each can be binned as one batch: 2..64
        views of one frame size, fewer than 2^30 - 1 (Gaussian, view) rows
        (the radix sort's key count)."""
        return (1 < len(views) <= 64 and len(views) * n < 2 ** 30 - 1 and
                len({(v.width, v.height) for v in views}) == 1)

    def prepare(self, batch: "_ViewBatch", first: int, V: int, n: int, W: int, H: int, tile: int,
                cut: int, opac: torch.Tensor, opac_stride: int) -> None:
        """Tile counts, depth sort and scan of views first..first+V-1 of
        `batch` (n Gaussians each; opacity rows from view `first` on when
        opac_stride is not 0); `read_totals` reads the result."""
        L = _lib.load()
        n_tiles = -(-W // tile) * -(-H // tile)
        nbytes = L.mg_bin_prepare_views_scratch_bytes(n, V, n_tiles)
        if self.prep.numel() < nbytes:
            self.prep = torch.empty(nbytes, dtype=torch.uint8, device=self.device)
        self.first = first
        op = opac[first] if opac_stride else opac
        _lib.check(L.mg_bin_prepare_views(
            ptr(batch.uv[first]), ptr(batch.rxy[first]), ptr(batch.conic[first]), ptr(op),
            ptr(batch.valid[first]), ptr(batch.depth[first]), n, V, batch.n, opac_stride, W, H,
            tile, cut, ptr(self.totals), ptr(self.prep), self.prep.numel(), _lib.stream()),
            "bin_prepare_views")

    def read_totals(self, V: int) -> list[int] | None:
        """The views' pair totals (one device->host read), or None when the
        batch has to be binned one view at a time (2^30 - 1 pairs or more,
        the tile sort's limit).
        The device error word rides on the same read: a kernel that gave up
        a bounded wait or met a bad index since the last check raises
        DeviceError here, before its results are used."""
        _lib.call("mg_peek_device_error", ptr(self.totals[V + 2:V + 3]), _lib.stream())
        t = self.totals[:V + 3].tolist()
        if t[V + 2]:
            _lib.raise_device_error(t[V + 2], "binning")
        if t[V] >= 2 ** 30 - 1:
            return None
        self.bases = [0] * V
        for v in range(1, V):
            self.bases[v] = self.bases[v - 1] + int(t[v - 1])
        return [int(x) for x in t[:V]]

    def emit_all(self, batch: "_ViewBatch", V: int, n: int, W: int, H: int, tile: int, cut: int,
                 opac: torch.Tensor, opac_stride: int, m_total: int) -> None:
        L = _lib.load()
        n_tiles = -(-W // tile) * -(-H // tile)
        if self.ids.numel() < max(m_total, 1):
            self.ids = torch.empty(int(max(m_total, 1) * 1.25), dtype=torch.int32,
                                   device=self.device)
        if self.offsets.numel() < V * (n_tiles + 1):
            self.offsets = torch.empty(V * (n_tiles + 1), dtype=torch.int32, device=self.device)
        ebytes = L.mg_bin_emit_views_scratch_bytes(n, V, m_total, n_tiles)
        if self.emit.numel() < ebytes:
            self.emit = torch.empty(int(ebytes * 1.25) + 256, dtype=torch.uint8,
                                    device=self.device)
        f = self.first
        op = opac[f] if opac_stride else opac
        _lib.check(L.mg_bin_emit_views(
            ptr(batch.uv[f]), ptr(batch.rxy[f]), ptr(batch.conic[f]), ptr(op), n, V, batch.n,
            opac_stride, m_total, W, H, tile, cut, ptr(self.prep), ptr(self.ids),
            ptr(self.offsets), ptr(self.emit), self.emit.numel(), _lib.stream()),
            "bin_emit_views")
        self.n_tiles = n_tiles

    def view(self, v: int, m: int) -> tuple[torch.Tensor, torch.Tensor]:
        """Gauss ids and tile offsets of the batch's view v (counted from
        `first`; views into the batch's arrays)."""
        base = self.bases[v]
        k = self.n_tiles + 1
        return self.ids[base:base + max(m, 1)], self.offsets[v * k:(v + 1) * k]


def _views_array(cams: list) -> "_lib.C.Array":
    return (_lib.Camera * len(cams))(*cams)


class Trainer:
    """Data-parallel batched trainer. `params` holds the trainer's storage
    tensors (means, quats, log_scales, logit_opac, sh_dc (N,1,3),
    sh_rest (N,15,3)); they are copied into the flat device buffer."""

    def __init__(self, params: dict, device="cuda", *, sh_degree: int = 3, tile: int = 16,
                 background=(0.0, 0.0, 0.0), lrs: dict | None = None, w_l1: float = 0.8,
                 w_ssim: float = 0.2, selective: bool = True, near: float = 0.01,
                 far: float = 100.0, max_radius_frac: float = 1.0, group=None,
                 betas=(0.9, 0.999), eps: float = 1e-15, shard_optimizer: bool | None = None,
                 saturation_cut: bool = True, opac_reg: float = 0.0, scale_reg: float = 0.0,
                 antialias: bool = False):
        self.device = torch.device(device)
        self.n = n = int(params["means"].shape[0])
        # rows < active are rendered and densified (3DGS-MCMC grows it toward
        # the capacity n); buffers are sized for the capacity
        self.active = n
        self.world = dp.world_size(group)
        self.rank = dp.rank(group)
        # ZeRO-1: with several ranks each one owns the optimizer state of a
        # contiguous range of Gaussian rows (gradient reduce-scatter, Adam on
        # the shard, parameter all-gather); rows are padded to a multiple of
        # the world size so every segment splits into equal row shards
        self.shard_optimizer = (self.world > 1) if shard_optimizer is None else shard_optimizer
        # drop each tile's pairs behind the depth where covering Gaussians
        # provably saturate every pixel (mg_bin_prepare): same images and
        # gradients, fewer pairs to emit and sort
        self.saturation_cut = int(bool(saturation_cut))
        # bin a step's views of one frame size together (one depth sort and
        # one tile sort for all of them); False bins them one at a time
        self.batch_binning = True
        # the MCMC regularisers of the training loss (train.py:393-398):
        # reg_weight * (opac_reg * mean(opacity) + scale_reg * mean(scale)) over
        # the active rows; fit() ramps reg_weight down as the reference does
        self.opac_reg, self.scale_reg = float(opac_reg), float(scale_reg)
        self.reg_weight = 1.0
        # Mip-Splatting's 2D antialias compensation (train.py --antialias,
        # metal_backend.py:506-511): each view draws with its compensated
        # opacities, and their adjoint is applied to the views' gradient
        # records before the projection adjoint
        self.antialias = bool(antialias)
        # phase B's per-view chains (pack, raster forward, loss, raster
        # backward) run on this many streams, each with its own frame
        # buffers, so one view's raster tail overlaps the next view's work
        self.view_streams = 4
        self._streams: list = []
        # views binned per batch binning call (0: all of a step's views); a
        # chunk's rendering on the streams overlaps the binning of the next
        self.bin_chunk = 0
        self._bin_stream = None
        self._reg_scratch = None
        self.n_pad = -(-n // self.world) * self.world if self.shard_optimizer else n
        self.sh_degree, self.tile = sh_degree, tile
        self.background = None if background is None or all(b == 0 for b in background) \
            else tuple(float(b) for b in background)
        self.w_l1, self.w_ssim = w_l1, w_ssim
        self.selective = selective
        self.near, self.far, self.max_radius_frac = near, far, max_radius_frac
        self.group = group
        self.betas, self.eps = betas, eps
        self.lrs = dict(DEFAULT_LRS, **(lrs or {}))
        f32 = dict(dtype=torch.float32, device=self.device)
        # segment starts rounded up to 64 floats (256 B): quaternions are read
        # as float4 and every segment stays aligned for vector access. The
        # geometry segments and the SH segments form two exchange groups, each
        # padded so it splits into equal 64-float-aligned chunks, one per rank
        # (the unit of the reduce-scatter / all-gather)
        unit = 64 * self.world
        self.offsets = {}
        off = 0
        for name, w in SEGMENTS:
            if name == "sh_dc":
                off = -(-off // unit) * unit
                self.geo_end = off
            self.offsets[name] = off
            off += (w * self.n_pad + 63) // 64 * 64
        self.p_total = -(-off // unit) * unit
        self.vis_offset = self.p_total
        # gradient buffer: parameter region | visibility counts | loss
        self.loss_offset = self.vis_offset + self.n_pad
        self.P = torch.zeros(self.p_total, **f32)
        self.G = torch.zeros(self.loss_offset + 64, **f32)
        self.M = torch.zeros(self.p_total, **f32)
        self.V = torch.zeros(self.p_total, **f32)
        self.steps = torch.zeros(self.n_pad, **f32)
        self._adam_rows = torch.empty(self.n_pad, **f32)  # per-row bias factors
        self.step_count = 0
        for name, _ in SEGMENTS:
            self.param(name).copy_(params[name].to(self.device, torch.float32).reshape(
                (n,) + SHAPES[name]))
        # the activations the forward projects: exp / sigmoid of the
        # parameters, widened and dimmed by the 3D filter when one is set
        self.scales = torch.empty(n, 3, **f32)
        self.opac = torch.empty(n, **f32)
        # Mip-Splatting's 3D filter (N,) or None; with it, the activations
        # before the filter are kept for the gradient chain
        self.filter_3d: torch.Tensor | None = None
        self._scales_act = torch.empty(0, **f32)
        self._opac_act = torch.empty(0, **f32)
        self.loss = self.G[self.loss_offset:self.loss_offset + 1]
        self.window = torch.empty(11, **f32)
        x = torch.arange(11, dtype=torch.float32) - 5
        w = torch.exp(-x ** 2 / (2 * 1.5 ** 2))
        self.window.copy_(w / w.sum())
        self._bufs: dict[tuple[int, int], _ImageBuffers] = {}
        self._batch: _ViewBatch | None = None
        self._states: list[_ViewState] = []
        # per-view pair totals of the one-view-at-a-time binning; the last
        # slot receives the device error word before the host reads them
        self._totals = torch.zeros(MAX_VIEWS_PER_STEP + 1, dtype=torch.int64, device=self.device)
        # one batch binning per chunk of a step's views
        self._bbs: list[_BatchBinning] = []
        self._cams: dict[int, _lib.Camera] = {}
        self.last_stats: list[ViewStats] = []
        # stage name -> list of (start, end) CUDA events, when timing is on;
        # timed_stages restricts the recording to those names (None: all)
        self.stage_events: dict[str, list] | None = None
        self.timed_stages: set | None = None
        # per-view list entries walked by the rasteriser (device scalars),
        # recorded while timing is on
        self.walked: list[torch.Tensor] = []
        # ZeRO-1 over several ranks: the geometry and SH groups are exchanged
        # asynchronously on communicators of their own; a step leaves its two
        # parameter all-gathers in flight, and the next step waits for the
        # geometry before its projection and for the SH rows only before the
        # colour of its views (computed after its binning)
        self._xchg = (dp.ZeroExchange([(0, self.geo_end), (self.geo_end, self.p_total)], group)
                      if self.world > 1 and self.shard_optimizer else None)
        self.split_colour = self._xchg is not None
        self._pending: dict[str, object] = {"geo": None, "sh": None}
        self._side = None
        self._colour_stream = None
        # host targets are copied on this stream while the step projects and
        # bins; the loss kernels wait for the copies' event
        self._copy_stream = None
        self._target_bufs: list[torch.Tensor] = []
        self._targets_ready = None

    # ---------------------------------------------------------------- timing

    def _begin(self, name: str):
        if self.stage_events is None or (self.timed_stages is not None
                                         and name not in self.timed_stages):
            return None
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        self.stage_events.setdefault(name, []).append((a, b))
        return b

    @staticmethod
    def _end(ev) -> None:
        if ev is not None:
            ev.record()

    def stage_times_ms(self) -> dict[str, list[float]]:
        """Per-stage event durations recorded since timing was switched on
        (call after a synchronize)."""
        return {k: [a.elapsed_time(b) for a, b in v] for k, v in (self.stage_events or {}).items()}

    # ------------------------------------------------------------- storage

    def _view(self, buf: torch.Tensor, name: str) -> torch.Tensor:
        w = dict(SEGMENTS)[name]
        o = self.offsets[name]
        return buf[o:o + w * self.n].view((self.n,) + SHAPES[name])

    def param(self, name: str) -> torch.Tensor:
        return self._view(self.P, name)

    def grad(self, name: str) -> torch.Tensor:
        return self._view(self.G, name)

    def parameters(self) -> dict:
        """The current parameters in the trainer's storage form (views into
        the flat device buffer): means, quats, log_scales, logit_opac,
        sh_dc (N,1,3), sh_rest (N,15,3)."""
        self.synchronize_params()
        return {name: self.param(name) for name, _ in SEGMENTS}

    def export_ply(self, path, filter_3d=None) -> None:
        """Write the current model as an INRIA-convention .ply, the file the
        reference's `train.export_ply` writes (see `metal_gauss_b200.ply`);
        with `filter_3d` (e.g. `trainer.filter_3d`) the filter is baked in."""
        from .ply import export_ply
        export_ply(self.parameters(), path, filter_3d=filter_3d)

    def compute_filter_3d(self, views, near: float = 0.2, margin: float = 0.15) -> torch.Tensor:
        """Mip-Splatting's 3D filter of the current means for the training
        cameras `views` (mipfilter.compute_3d_filter, mipfilter.py:30-76),
        used by every following step until it is recomputed or cleared
        (`trainer.filter_3d = None`)."""
        from .mipfilter import compute_3d_filter
        self.synchronize_params()
        self.filter_3d = compute_3d_filter(self.param("means"), views, near, margin)
        return self.filter_3d

    # ------------------------------------------------------------- MCMC

    def _mcmc_tables(self):
        """The Gaussian table as row segments: the parameter segments of P,
        then the Adam rows to reset (M and V in P's layout, the per-row step
        counts)."""
        self.synchronize_params()
        params = [_lib.RowSegment(self.P.data_ptr() + 4 * self.offsets[name], w)
                  for name, w in SEGMENTS]
        rows = [_lib.RowSegment(buf.data_ptr() + 4 * self.offsets[name], w)
                for buf in (self.M, self.V) for name, w in SEGMENTS]
        rows.append(_lib.RowSegment(self.steps.data_ptr(), 1))
        names = [name for name, _ in SEGMENTS]
        return ((_lib.RowSegment * len(params))(*params), len(params),
                names.index("logit_opac"), names.index("log_scales"),
                (_lib.RowSegment * len(rows))(*rows), len(rows))

    def _mcmc_seed(self, seed) -> int:
        # identical on every rank (the table is replicated), new every step
        if seed is not None:
            return int(seed)
        return (0x5EED * 1_000_003 + self.step_count) & (2 ** 63 - 1)

    def _mcmc_weights(self, weights):
        if weights is None:
            return None
        return weights[:self.active].to(self.device, torch.float32).contiguous()

    def relocate(self, dead_thresh: float = 0.005, weights: torch.Tensor | None = None,
                 seed: int | None = None, picks: torch.Tensor | None = None) -> int:
        """3DGS-MCMC relocation (mcmc.relocate, mcmc.py:52-121) of the active
        rows in the trainer's own buffers, Adam rows of every changed row
        reset. Returns how many dead Gaussians moved."""
        P, nP, il, isc, R, nR = self._mcmc_tables()
        w = self._mcmc_weights(weights)
        pk = None if picks is None else picks.to(self.device, torch.int32).contiguous()
        scratch = torch.empty(_lib.load().mg_mcmc_scratch_bytes(self.active), dtype=torch.uint8,
                              device=self.device)
        moved = _lib.C.c_int64(0)
        _lib.call("mg_mcmc_relocate", P, nP, il, isc, R, nR, self.active, float(dead_thresh),
                  ptr(w), ptr(pk), self._mcmc_seed(seed), _lib.C.byref(moved), ptr(scratch),
                  scratch.numel(), _lib.stream())
        return int(moved.value)

    def grow(self, target: int, weights: torch.Tensor | None = None, seed: int | None = None,
             picks: torch.Tensor | None = None) -> int:
        """3DGS-MCMC growth (mcmc.grow, mcmc.py:124-163): rows [active,
        target) cloned from weight-drawn active rows; returns the new active
        count."""
        P, nP, il, isc, R, nR = self._mcmc_tables()
        w = self._mcmc_weights(weights)
        pk = None if picks is None else picks.to(self.device, torch.int32).contiguous()
        scratch = torch.empty(_lib.load().mg_mcmc_scratch_bytes(self.n), dtype=torch.uint8,
                              device=self.device)
        out = _lib.C.c_int64(0)
        _lib.call("mg_mcmc_grow", P, nP, il, isc, R, nR, self.active, int(target), self.n, ptr(w),
                  ptr(pk), self._mcmc_seed(seed), _lib.C.byref(out), ptr(scratch),
                  scratch.numel(), _lib.stream())
        self.active = int(out.value)
        return self.active

    def add_noise(self, lr_means: float | None = None, weight: float = 4e4,
                  opacity_gate: float = 0.005, seed: int | None = None) -> None:
        """3DGS-MCMC exploration noise (mcmc.add_noise, mcmc.py:166-192) on the
        active means, scaled by the current means learning rate."""
        lr = self.lrs["means"] if lr_means is None else lr_means
        self.synchronize_params()
        _lib.call("mg_mcmc_add_noise", ptr(self.param("means")), ptr(self.param("quats")),
                  ptr(self.param("log_scales")), ptr(self.param("logit_opac")), self.active,
                  float(lr), float(weight), float(opacity_gate),
                  self._mcmc_seed(seed) ^ 0x9E3779B97F4A7C15, None, _lib.stream())

    def _filter_tensor(self) -> torch.Tensor | None:
        """The 3D filter as a contiguous (N,) device tensor (None when unset),
        with the pre-filter activation buffers the gradient chain needs."""
        if self.filter_3d is None:
            return None
        f = self.filter_3d.to(self.device, torch.float32).contiguous()
        if f.numel() != self.n:
            raise ValueError(f"filter_3d has {f.numel()} values for {self.n} Gaussians")
        self.filter_3d = f
        if self._scales_act.shape != self.scales.shape:
            self._scales_act = torch.empty_like(self.scales)
            self._opac_act = torch.empty_like(self.opac)
        return f

    def _activate(self) -> None:
        """The forward's scales and opacities: exp / sigmoid of the
        parameters (train.py:221-222), then the 3D filter when one is set
        (train.py:223-227). `train_step` does the same inside the projection
        kernel (`_prologue`); this form serves callers that drive
        `forward_backward_views` themselves."""
        self.synchronize_params()
        f = self._filter_tensor()
        if f is None:
            torch.exp(self.param("log_scales"), out=self.scales)
            torch.sigmoid(self.param("logit_opac"), out=self.opac)
            return
        torch.exp(self.param("log_scales"), out=self._scales_act)
        torch.sigmoid(self.param("logit_opac"), out=self._opac_act)
        _lib.call("mg_apply_3d_filter", ptr(self._scales_act), ptr(self._opac_act), ptr(f), self.n,
                  ptr(self.scales), ptr(self.opac), _lib.stream())

    def _prologue(self) -> "_lib.StepPrologue":
        """The start of a step for the projection kernel (mg_step_prologue):
        the activations (through the 3D filter when one is set), the
        geometry gradient rows and the loss set to zero, the visibility
        count written rather than added."""
        f = self._filter_tensor()
        pro = _lib.StepPrologue()
        pro.log_scales = ptr(self.param("log_scales"))
        pro.logit_opac = ptr(self.param("logit_opac"))
        if f is None:
            pro.act_scales, pro.act_opac = ptr(self.scales), ptr(self.opac)
        else:
            pro.filter_3d = ptr(f)
            pro.act_scales, pro.act_opac = ptr(self._scales_act), ptr(self._opac_act)
            pro.out_scales, pro.out_opac = ptr(self.scales), ptr(self.opac)
        for k, name in enumerate(("means", "quats", "log_scales", "logit_opac")):
            pro.zero[k] = ptr(self.grad(name))
            pro.zero_width[k] = dict(SEGMENTS)[name]
        pro.zero_word = ptr(self.loss)
        return pro

    def visibility_count(self) -> torch.Tensor:
        return self.G[self.vis_offset:self.vis_offset + self.n]

    def _segment(self, buf: torch.Tensor, name: str) -> torch.Tensor:
        """A whole padded segment (n_pad rows) of a flat buffer."""
        if name == "visibility":
            return buf[self.vis_offset:self.vis_offset + self.n_pad]
        w = dict(SEGMENTS)[name]
        o = self.offsets[name]
        return buf[o:o + w * self.n_pad]

    def state_dict(self) -> dict:
        self.synchronize_params()
        return {name: self.param(name).detach().clone() for name, _ in SEGMENTS}

    # --------------------------------------------------------------- views

    def _camera(self, view) -> _lib.Camera:
        key = id(view)
        cam = self._cams.get(key)
        if cam is None:
            vm = view.viewmat.to(torch.float32)
            K = view.K
            cc = -vm[:3, :3].T @ vm[:3, 3]
            cam = _lib.make_camera(vm, float(K[0, 0]), float(K[1, 1]), float(K[0, 2]),
                                   float(K[1, 2]), view.width, view.height, self.near, self.far,
                                   0.3, self.max_radius_frac * max(view.width, view.height), cc)
            self._cams[key] = cam
        return cam

    def _buffers(self, W: int, H: int, slot: int = 0) -> _ImageBuffers:
        b = self._bufs.get((W, H, slot))
        if b is None:
            b = _ImageBuffers(self.n, W, H, self.device)
            self._bufs[(W, H, slot)] = b
        return b

    def _phase_b_streams(self, V: int) -> list:
        """The streams phase B's view chains take turns on; none (the
        current stream) with one view, one stream asked for, or while every
        stage is being timed (overlapping stages would blur the split)."""
        k = min(int(self.view_streams), V)
        if k <= 1 or (self.stage_events is not None and self.timed_stages is None):
            return []
        while len(self._streams) < k:
            self._streams.append(torch.cuda.Stream(self.device))
        return self._streams[:k]

    def _ensure_views(self, V: int) -> None:
        """View-major buffers for V views (grown, never shrunk)."""
        if (self._batch is None or self._batch.cap < V or
                (self._batch.opac is None) == self.antialias):
            self._batch = _ViewBatch(self.n, V, self.device, per_view_opacity=self.antialias)
            for v, st in enumerate(self._states):
                st.bind(self._batch, v)
        while len(self._states) < V:
            self._states.append(_ViewState(self._batch, len(self._states), self.device))

    def _state(self, v: int) -> _ViewState:
        return self._states[v]

    def _project_views(self, views, begin_step: bool = False) -> None:
        """Phase A, first half: projection + SH colour of every view in one
        launch (parameters and SH rows read once), adding each Gaussian's
        count of valid views to the visibility count. With `begin_step` the
        same launch runs the step's prologue (`_prologue`)."""
        b = self._batch
        cams = _views_array([self._camera(view) for view in views])
        pro = _lib.C.byref(self._prologue()) if begin_step else None
        # with the colour split the SH rows are not read here (`_colour_views`
        # colours the views after the binning)
        colour = not self.split_colour
        ev = self._begin("preprocess_fwd")
        _lib.call("mg_preprocess_forward_views", ptr(self.param("means")),
                  ptr(self.param("quats")), ptr(self.scales),
                  ptr(self.param("sh_dc")) if colour else None,
                  ptr(self.param("sh_rest")) if colour else None, _lib.SH_SPLIT, ptr(self.opac),
                  _lib.C.cast(cams, _lib.C.c_void_p), len(views),
                  self.sh_degree if colour else -1, self.active, self.n,
                  ptr(b.uv), ptr(b.conic), ptr(b.depth), ptr(b.rxy), ptr(b.valid), ptr(b.color),
                  ptr(self.visibility_count()), pro, _lib.stream())
        if self.antialias:
            _lib.call("mg_antialias_opacity_views", ptr(b.conic), ptr(self.opac), self.active,
                      len(views), self.n, 0.3, ptr(b.opac), _lib.stream())
        self._end(ev)

    def _colour_views(self, views) -> None:
        """The SH colour of every view of the batch (mg_sh_colour_views), for a
        projection that skipped it; waits first for the previous step's SH
        all-gather."""
        self._wait("sh", "wait_sh_gather")
        centres = (_lib.C.c_float * (3 * len(views)))()
        for v, view in enumerate(views):
            cc = self._camera(view).cam_center
            centres[3 * v:3 * v + 3] = [cc[0], cc[1], cc[2]]
        b = self._batch
        ev = self._begin("colour")
        _lib.call("mg_sh_colour_views", ptr(self.param("means")), ptr(self.param("sh_dc")),
                  ptr(self.param("sh_rest")), _lib.SH_SPLIT,
                  _lib.C.cast(centres, _lib.C.c_void_p), len(views), self.sh_degree, self.active,
                  self.n, ptr(b.valid), ptr(b.color), _lib.stream())
        self._end(ev)

    def _view_opacities(self) -> tuple[torch.Tensor, int]:
        """The opacities the views draw with and their view stride (0: shared)."""
        if self.antialias:
            return self._batch.opac, self._batch.n
        return self.opac, 0

    def _opacity(self, st: "_ViewState") -> torch.Tensor:
        return st.opac if self.antialias else self.opac

    def _bin_chunk(self, c: int, first: int, chunk) -> tuple[list[int], "_BatchBinning | None"]:
        """Phase A, second half, for views first.. of a chunk: their pair
        totals (one host read) and, when binned together, the batch binning
        that holds their lists; otherwise each view's stage A ran into its
        own state and its pairs are emitted in phase B."""
        V = len(chunk)
        if self.batch_binning and _BatchBinning.fits(chunk, self.active):
            while len(self._bbs) <= c:
                self._bbs.append(_BatchBinning(self.device))
            bb = self._bbs[c]
            W, H = chunk[0].width, chunk[0].height
            ev = self._begin("bin_prepare")
            op, op_stride = self._view_opacities()
            bb.prepare(self._batch, first, V, self.active, W, H, self.tile, self.saturation_cut,
                       op, op_stride)
            self._end(ev)
            totals = bb.read_totals(V)
            if totals is not None:
                ev = self._begin("bin_emit")
                bb.emit_all(self._batch, V, self.active, W, H, self.tile, self.saturation_cut,
                            op, op_stride, sum(totals))
                self._end(ev)
                return totals, bb
        for i, view in enumerate(chunk):
            self._prepare(first + i, view)
        _lib.call("mg_peek_device_error", ptr(self._totals[-1:]), _lib.stream())
        t = self._totals.tolist()
        if t[-1]:
            _lib.raise_device_error(t[-1], "binning")
        return [int(x) for x in t[first:first + V]], None

    def _prepare(self, v: int, view) -> None:
        """Phase A, second half, for view v: tile counts, depth sort and the
        scan that yields the view's pair total."""
        L = _lib.load()
        s = _lib.stream()
        st = self._state(v)
        ev = self._begin("bin_prepare")
        prep = st.prep_scratch(-(-view.width // self.tile) * -(-view.height // self.tile))
        _lib.check(L.mg_bin_prepare(
            ptr(st.uv), ptr(st.rxy), ptr(st.conic), ptr(self._opacity(st)), ptr(st.valid),
            ptr(st.depth),
            self.active, view.width, view.height, self.tile, self.saturation_cut,
            ptr(self._totals[v:v + 1]), ptr(prep), prep.numel(), s), "bin_prepare")
        self._end(ev)

    def _stage_targets(self, targets) -> list[torch.Tensor]:
        """Device tensors of the step's targets (H, W, 3): float32 in [0, 1]
        or uint8 bytes, which the loss reads as x / 255 (the reference divides
        its byte images by 255, train.py:385). Device targets are used as they
        are; host targets are copied into resident buffers on a side stream,
        so the copy overlaps the step's projection and binning (it is
        asynchronous from pinned memory), and the loss kernels wait for it."""
        out = []
        host = [t for t in targets if t.device.type != "cuda"]
        self._targets_ready = None
        if host:
            if self._copy_stream is None:
                self._copy_stream = torch.cuda.Stream(self.device)
            # the previous step's loss kernels (joined into this stream) are
            # done with the buffers before they are overwritten
            self._copy_stream.wait_stream(torch.cuda.current_stream(self.device))
        k = 0
        for t in targets:
            if t.dtype not in (torch.uint8, torch.float32) or t.dim() != 3 or t.shape[2] != 3:
                raise ValueError("targets must be (H, W, 3) uint8 or float32 images")
            if t.device.type == "cuda":
                out.append(t.contiguous())
                continue
            while len(self._target_bufs) <= k:
                self._target_bufs.append(torch.empty(0, dtype=torch.uint8, device=self.device))
            buf = self._target_bufs[k]
            if buf.shape != t.shape or buf.dtype != t.dtype:
                buf = torch.empty(t.shape, dtype=t.dtype, device=self.device)
                self._target_bufs[k] = buf
            with torch.cuda.stream(self._copy_stream):
                buf.copy_(t, non_blocking=True)
            out.append(buf)
            k += 1
        if host:
            self._targets_ready = torch.cuda.Event()
            self._targets_ready.record(self._copy_stream)
        return out

    def _render_and_backprop(self, v: int, view, target: torch.Tensor, m: int,
                             scale: float, lists: tuple | None = None,
                             slot: int = 0) -> ViewStats:
        """Phase B for view v (its pair total m known on the host) on the
        current stream with frame buffer set `slot`: pair emission and tile
        sort (unless `lists`, the view's ids and tile offsets from a batch
        binning, are given), raster forward, fused loss and raster backward
        into the view's gradient records."""
        L = _lib.load()
        s = _lib.stream()
        W, H, n = view.width, view.height, self.active
        st = self._state(v)
        b = self._buffers(W, H, slot)
        tiles_x, tiles_y = -(-W // self.tile), -(-H // self.tile)
        n_tiles = tiles_x * tiles_y
        if b.tile_work is None or b.tile_work.numel() != n_tiles:
            b.tile_work = torch.empty(n_tiles, dtype=torch.int32, device=self.device)
        rbytes = L.mg_raster_scratch_bytes(W, H, self.tile, m)
        if b.raster.numel() < rbytes:
            b.raster = torch.empty(int(rbytes * 1.25) + 256, dtype=torch.uint8,
                                   device=self.device)
        if lists is not None:
            ids, offsets = lists
        else:
            if b.ids.numel() < max(m, 1):
                b.ids = torch.empty(int(max(m, 1) * 1.25), dtype=torch.int32,
                                    device=self.device)
            if b.offsets is None or b.offsets.numel() != n_tiles + 1:
                b.offsets = torch.empty(n_tiles + 1, dtype=torch.int32, device=self.device)
            ebytes = L.mg_bin_emit_scratch_bytes(n, m, n_tiles)
            if b.emit.numel() < ebytes:
                b.emit = torch.empty(int(ebytes * 1.25) + 256, dtype=torch.uint8,
                                     device=self.device)
            ev = self._begin("bin_emit")
            _lib.check(L.mg_bin_emit(ptr(st.uv), ptr(st.rxy), ptr(st.conic),
                                     ptr(self._opacity(st)), n, m, W, H, self.tile,
                                     self.saturation_cut, ptr(st.prep), ptr(b.ids),
                                     ptr(b.offsets), ptr(b.emit), b.emit.numel(), s),
                       "bin_emit")
            self._end(ev)
            ids, offsets = b.ids, b.offsets
        bg = None if self.background is None else (_lib.C.c_float * 3)(*self.background)
        bgp = None if bg is None else _lib.C.cast(bg, _lib.C.c_void_p)
        ev = self._begin("pack")
        _lib.check(L.mg_pack_splats(ptr(st.uv), ptr(st.conic), ptr(self._opacity(st)),
                                    ptr(st.color), n, ptr(b.splats), ptr(st.grad2d), s),
                   "pack_splats")
        self._end(ev)
        # tile walk lengths only in a fully instrumented pass (every stage
        # timed): their sum is a torch reduction, kept out of timed steps
        work = (b.tile_work if self.stage_events is not None and self.timed_stages is None
                else None)
        ev = self._begin("raster_fwd")
        _lib.check(L.mg_rasterize_forward(
            ptr(b.splats), ptr(ids), ptr(offsets), m, W, H, self.tile, tiles_x, bgp,
            ptr(b.rgb), ptr(b.alpha), ptr(b.T), ptr(b.stop), ptr(work), ptr(b.raster),
            b.raster.numel(), s), "rasterize_forward")
        self._end(ev)
        if work is not None:
            self.walked.append(work.sum())
        ev = self._begin("loss")
        if self._targets_ready is not None:
            torch.cuda.current_stream(self.device).wait_event(self._targets_ready)
        if tuple(target.shape) != (H, W, 3):
            raise ValueError(f"target of view {v} is {tuple(target.shape)}, not ({H}, {W}, 3)")
        loss_fn = L.mg_l1_ssim_loss_u8 if target.dtype == torch.uint8 else L.mg_l1_ssim_loss
        _lib.check(loss_fn(
            ptr(b.rgb), ptr(target), ptr(self.window), H, W, self.w_l1, self.w_ssim, scale,
            ptr(b.grad_rgb), ptr(self.loss), ptr(b.loss_scratch), b.loss_scratch.numel(), s),
            "l1_ssim_loss")
        self._end(ev)
        ev = self._begin("raster_bwd")
        _lib.check(L.mg_rasterize_backward(
            ptr(b.splats), ptr(ids), ptr(offsets), m, ptr(b.rgb), ptr(b.alpha), ptr(b.T),
            ptr(b.stop), ptr(b.grad_rgb), None, W, H, self.tile, tiles_x, bgp, 0, n,
            ptr(st.grad2d), 1, ptr(b.raster), b.raster.numel(), s), "rasterize_backward")
        self._end(ev)
        return ViewStats(pairs=m)

    def forward_backward_views(self, views, targets, scale: float,
                               begin_step: bool = False) -> list[ViewStats]:
        """Render this rank's views: scale * each loss is added into
        self.loss, scale * the views' gradients of means, quats, log-scales and
        opacity logits are added into self.G and the views' SH gradients are
        written into it (the SH adjoint covers all of a call's views at once
        and overwrites its rows). With `begin_step` the projection kernel
        first forms the activations and sets the geometry gradient rows, the
        visibility count and the loss to zero (what `train_step` uses);
        otherwise the caller has run `_activate` and the call adds to G. One
        device->host read per binning chunk (its views' pair totals, with the
        device error word)."""
        V = len(views)
        if V > MAX_VIEWS_PER_STEP:
            raise ValueError(f"a step takes at most {MAX_VIEWS_PER_STEP} views per rank, got "
                             f"{V} (split the batch over more ranks or steps)")
        if begin_step:
            # the projection reads (and its prologue writes) only geometry rows
            self._wait("geo", "wait_geo_gather")
        else:
            self.synchronize_params()
        self._ensure_views(V)
        self._project_views(views, begin_step)
        streams = self._phase_b_streams(V)
        main = torch.cuda.current_stream(self.device)
        # with the colour split, the views' colour waits for the previous
        # step's SH all-gather on a stream of its own, beside the binning
        # (the rendering waits for it); while every stage is timed it runs
        # after the first chunk's binning instead
        colour_done = None
        if self.split_colour and not (self.stage_events is not None and
                                      self.timed_stages is None):
            if self._colour_stream is None:
                self._colour_stream = torch.cuda.Stream(self.device)
            self._colour_stream.wait_stream(main)   # the projection's valid flags
            with torch.cuda.stream(self._colour_stream):
                self._colour_views(views)
            colour_done = torch.cuda.Event()
            colour_done.record(self._colour_stream)
        C = V if self.bin_chunk <= 0 else min(V, int(self.bin_chunk))
        # chunked binning runs on a high-priority stream: it is the critical
        # path while the earlier chunks' views render on the others
        bin_stream = main
        if streams and C < V:
            if self._bin_stream is None:
                self._bin_stream = torch.cuda.Stream(self.device, priority=-1)
            bin_stream = self._bin_stream
            bin_stream.wait_stream(main)
        stats: list = [None] * V
        for c, first in enumerate(range(0, V, C)):
            chunk = views[first:first + C]
            with torch.cuda.stream(bin_stream):
                totals, bb = self._bin_chunk(c, first, chunk)
                if c == 0 and self.split_colour and colour_done is None:
                    self._colour_views(views)
            if c == 0 and colour_done is not None:
                for sk in streams or [main]:
                    sk.wait_event(colour_done)
            if streams:
                # the chunk's views on the streams in turn, after its binning
                ready = torch.cuda.Event()
                ready.record(bin_stream)
                for sk in streams:
                    sk.wait_event(ready)
            for i, view in enumerate(chunk):
                v, m = first + i, int(totals[i])
                lists = None if bb is None else bb.view(i, m)
                if streams:
                    k = v % len(streams)
                    with torch.cuda.stream(streams[k]):
                        stats[v] = self._render_and_backprop(v, view, targets[v], m, scale,
                                                             lists, k)
                else:
                    stats[v] = self._render_and_backprop(v, view, targets[v], m, scale, lists)
        if bin_stream is not main:
            main.wait_stream(bin_stream)
        for sk in streams:  # the adjoints below wait for every view
            done = torch.cuda.Event()
            done.record(sk)
            main.wait_event(done)
        # the projection adjoint of all views at once (parameters read and
        # gradient rows updated once), then the SH adjoint likewise
        b = self._batch
        cams = _views_array([self._camera(view) for view in views])
        ev = self._begin("preprocess_bwd")
        if self.antialias:  # the compensation's adjoint on every view's records
            _lib.call("mg_antialias_grad2d_views", ptr(b.conic), ptr(self.opac), self.active, V,
                      self.n, 0.3, ptr(b.grad2d), _lib.stream())
        filt = self.filter_3d
        _lib.call("mg_preprocess_backward_views", ptr(self.param("means")),
                  ptr(self.param("quats")), ptr(self.scales if filt is None else self._scales_act),
                  ptr(self.opac if filt is None else self._opac_act), ptr(b.grad2d),
                  ptr(b.valid), ptr(b.color), _lib.C.cast(cams, _lib.C.c_void_p), V, self.active,
                  self.n, ptr(filt), ptr(self.grad("means")), ptr(self.grad("quats")),
                  ptr(self.grad("log_scales")), ptr(self.grad("logit_opac")), ptr(b.dpre),
                  _lib.stream())
        self._end(ev)
        centres = (_lib.C.c_float * (3 * V))()
        for v, view in enumerate(views):
            cc = self._camera(view).cam_center
            centres[3 * v:3 * v + 3] = [cc[0], cc[1], cc[2]]
        ev = self._begin("sh_bwd")
        _lib.call("mg_sh_backward_views", ptr(self.param("means")), ptr(self.param("sh_dc")),
                  ptr(self.param("sh_rest")), self.sh_degree, self.active,
                  _lib.C.cast(centres, _lib.C.c_void_p), ptr(b.dpre), V, self.n,
                  ptr(self.grad("means")), ptr(self.grad("sh_dc")), ptr(self.grad("sh_rest")),
                  _lib.stream())
        self._end(ev)
        return stats

    def owned_ranges(self) -> list[tuple[int, int]]:
        """Flat [lo, hi) ranges of the parameter region whose optimizer update
        this rank runs: the whole region, or under ZeRO-1 its chunk of the
        geometry group and its chunk of the SH group."""
        if self._xchg is None:
            return [(0, self.p_total)]
        return [self._xchg.owned(0), self._xchg.owned(1)]

    def _adam(self, ranges, flags: int = 0) -> None:
        """Adam over the flat ranges (segments clipped to them; a range may
        start or end inside a row), at the current step count."""
        segs = []
        for name, w in SEGMENTS:
            o = self.offsets[name]
            for c_lo, c_hi in ranges:
                b = max(c_lo, o) - o
                e = min(c_hi, o + w * self.n) - o
                if e > b:
                    segs.append(_lib.AdamSegment(o, w, self.lrs[name], b, e))
        b1, b2 = self.betas
        vis = self.visibility_count() if self.selective else None
        if segs:
            arr = (_lib.AdamSegment * len(segs))(*segs)
            _lib.call("mg_adam_multi", ptr(self.P), ptr(self.G), ptr(self.M), ptr(self.V), self.n,
                      arr, len(segs), b1, b2, self.eps, ptr(vis), ptr(self.steps),
                      self.step_count, ptr(self._adam_rows), flags, _lib.stream())
        elif vis is not None:  # no elements here: still form / advance the step counts
            _lib.call("mg_adam_multi", ptr(self.P), ptr(self.G), ptr(self.M), ptr(self.V), self.n,
                      (_lib.AdamSegment * 1)(_lib.AdamSegment(0, 1, 0.0, 0, 0)), 0, b1, b2,
                      self.eps, ptr(vis), ptr(self.steps), self.step_count, ptr(self._adam_rows),
                      flags, _lib.stream())

    def optimizer_step(self) -> None:
        """Adam over this rank's share (`owned_ranges`) in one launch."""
        self.synchronize_params()
        self.step_count += 1
        ev = self._begin("adam")
        self._adam(self.owned_ranges())
        self._end(ev)

    def train_step(self, views, targets, global_batch: int | None = None) -> torch.Tensor:
        """One optimisation step over this rank's `views`. `targets` are the
        views' images (H, W, 3): float32 in [0, 1] or uint8 bytes, on the
        device or on the host (host images are copied while the step projects
        and bins; pass pinned memory for an asynchronous copy). `global_batch`
        is the batch size summed over ranks (defaults to len(views) times the
        world size). Returns the batch-mean loss as a device tensor (1,),
        all-reduced across ranks."""
        world = self._world_size()
        gb = global_batch or len(views) * world
        targets = self._stage_targets(targets)
        # the activations and the zeroing of the accumulated gradient rows,
        # visibility counts and loss run inside the projection kernel; the SH
        # rows are overwritten by the SH adjoint
        self.last_stats = self.forward_backward_views(views, targets, 1.0 / gb, begin_step=True)
        if self.opac_reg or self.scale_reg:
            self._regularize(world)
        if self._xchg is not None:
            self._exchange_and_update()
            return self.loss
        if world > 1:
            ev = self._begin("allreduce")
            dp.all_reduce_(self.G, self.group)
            self._end(ev)
        self.optimizer_step()
        return self.loss

    def _exchange_and_update(self) -> None:
        """ZeRO-1 with the exchange overlapped. The visibility counts and the
        loss are all-reduced and both gradient groups reduce-scattered at once;
        the current stream waits only for the counts and the geometry chunk,
        updates it (forming the selective rows' bias factors and advancing the
        step counts) and starts its all-gather; a side stream waits for the SH
        chunk, updates it with the same factors (reading neither the counts,
        which the next step's projection rewrites, nor the step counts) and
        starts its all-gather. Neither gather is waited for here: the next
        step waits for the geometry before its projection and for the SH rows
        before its colour, which comes after its binning."""
        x = self._xchg
        main = torch.cuda.current_stream(self.device)
        ev = self._begin("exchange_wait")
        w_tail = x.all_reduce(self.G[self.vis_offset:], 0)   # visibility counts + loss
        w_geo = x.reduce_scatter(self.G, 0)
        w_sh = x.reduce_scatter(self.G, 1)
        w_tail.wait()
        w_geo.wait()
        self._end(ev)
        self.step_count += 1
        ev = self._begin("adam")
        self._adam([x.owned(0)])
        self._end(ev)
        self._pending["geo"] = x.all_gather(self.P, 0)
        if self._side is None:
            self._side = torch.cuda.Stream(self.device)
        self._side.wait_stream(main)   # the all-reduced counts and the row factors
        with torch.cuda.stream(self._side):
            w_sh.wait()
            self._adam([x.owned(1)], _lib.ADAM_ROW_FACTORS_READY | _lib.ADAM_KEEP_STEPS)
            self._pending["sh"] = x.all_gather(self.P, 1)

    def _regularize(self, world: int) -> None:
        """The MCMC regularisers (train.py:393-398) over the active rows: their
        gradient added into G and their value into the loss, a 1/world share
        on each rank (the ranks' gradients and losses are summed)."""
        if self._reg_scratch is None:
            self._reg_scratch = torch.empty(16, dtype=torch.uint8, device=self.device)
        w = self.reg_weight / world
        _lib.call("mg_regularizer_grad", ptr(self.param("logit_opac")),
                  ptr(self.param("log_scales")), self.active, w * self.opac_reg,
                  w * self.scale_reg, ptr(self.grad("logit_opac")), ptr(self.grad("log_scales")),
                  ptr(self.loss), ptr(self._reg_scratch), 16, _lib.stream())

    def _world_size(self) -> int:
        return dp.world_size(self.group)

    def _wait(self, kind: str, stage: str | None = None) -> None:
        """Make the current stream wait for the previous step's parameter
        all-gather of group `kind` ("geo" or "sh"), if one is in flight."""
        w = self._pending.get(kind)
        if w is None:
            return
        ev = self._begin(stage) if stage else None
        w.wait()
        self._end(ev)
        self._pending[kind] = None

    def synchronize_params(self) -> None:
        """Order the current stream after every parameter exchange still in
        flight, so P (and the optimizer state) may be read or changed. Every
        method that touches them outside a step calls it."""
        self._wait("geo")
        self._wait("sh")

    def check_device_error(self) -> None:
        """Synchronising check of the device error word; raises
        _lib.DeviceError when a kernel recorded a failure. Every step already
        checks the word for free at its pair-total read (the failures of the
        previous step's later kernels and of this step's binning); this one
        covers the last step too."""
        _lib.check_device_error("training step")

    # ------------------------------------------------------------ counters

    def bytes_per_step(self, views, stats: list[ViewStats] | None = None) -> float:
        """Algorithmic HBM bytes of one step on this rank: the compulsory
        traffic of the dataflow, every input read once and every output
        written once, stage by stage as commented below."""
        stats = stats or self.last_stats
        n = self.n
        nv = float(self.visibility_count().gt(0).sum()) if self.selective else n
        V = len(stats)
        # multi-view preprocess with the step prologue: parameters + SH rows
        # once, activations written (16 B), 11 gradient floats zeroed (44 B),
        # the visibility count written (4 B), 48 B out per view
        total = (44.0 + 192.0 + 16.0 + 44.0 + 4.0) * n + 48.0 * V * n
        # multi-view projection adjoint: parameters once; per view the gradient
        # record, valid flag, colour and gated colour gradient; one
        # read-modify-write of the 11 gradient floats
        total += 44.0 * n + (48.0 + 4.0 + 12.0 + 12.0) * V * n + 88.0 * n
        # SH adjoint over the views: means + SH rows in, per view the gated
        # colour gradient, SH gradient rows out, d_means read-modify-write
        total += (12.0 + 192.0 + 192.0 + 24.0) * n + 12.0 * V * n
        for v, st in zip(views, stats):
            P = v.width * v.height
            M = st.pairs
            total += 40 * n + 8 * n + 16 * n        # bin count, depth keys, scan
            total += 16 * n * 4                     # depth sort (4 passes x r/w 8 B)
            total += (36 + 8) * n + 8 * M           # pair emission
            total += 16 * M * math.ceil(math.log2(max(2, (v.width // self.tile + 1)
                                                       * (v.height // self.tile + 1))) / 8)
            total += 4 * M                          # ranges
            Wk = st.walked if st.walked else M
            total += (36 + 48 + 48) * n             # pack splat records, zero grad records
            total += 52 * Wk + 24 * P               # raster fwd (walked id + record)
            total += 27 * P                         # loss: image + uint8 target in, gradient out
            total += 52 * Wk + 36 * P + 48 * n      # raster bwd (+ gradient record)
        total += 28 * FLOATS_PER_GAUSSIAN * nv + 8 * n   # selective Adam
        return total


def fit(trainer: Trainer, views, targets, steps: int, batch: int = 8, *, seed: int = 0,
        lr_means_end: float | None = None, sh_warmup: int = 0, filter_3d_every: int = 0,
        noise_weight: float = 0.0, relocate_every: int = 0, relocate_until: int | None = None,
        grow_to: int | None = None, grow_until: int | None = None,
        opac_reg: float = 0.01, scale_reg: float = 0.01, callback=None) -> list[float]:
    """The reference's training loop (train.py:311-366) over batches of views.

    Views are drawn in epoch permutations (numpy's default_rng(seed), a new
    permutation whenever one is used up), `batch` per step; the means learning
    rate decays geometrically from its initial value to `lr_means_end` over
    `steps`; with `sh_warmup`, the SH degree grows by one band every
    `sh_warmup` steps up to 3. The appearance model is not part of this loop.
    The loss carries the reference's MCMC regularisers, `opac_reg` * mean opacity +
    `scale_reg` * mean scale over the active rows, ramped down by max(0, 1 -
    step / (0.9 steps)) (train.py:393-398; 0 turns them off). With
    `filter_3d_every`, Mip-Splatting's 3D filter is computed from all `views`
    before the first step and again every that many steps (train.py:343-380).
    3DGS-MCMC as train.py:416-462 runs it: with `noise_weight`, the
    exploration noise after every step at the current means learning rate;
    with `relocate_every`, relocation every that many steps before
    `relocate_until`, and with `grow_to`, growth of the active count from its
    value at the start toward `grow_to` by `grow_until` on the same steps.
    `targets` are (H, W, 3) uint8 or float images, moved to the device per
    step; returns the per-step losses (one host read per step). With several
    ranks every rank draws the same batches and renders its own share of
    each."""
    import numpy as np
    rng = np.random.default_rng(seed)
    order = rng.permutation(len(views))
    oi = 0
    lr0 = trainer.lrs["means"]
    decay = 1.0 if lr_means_end is None else (lr_means_end / max(lr0, 1e-12)) ** (1.0 / steps)
    rank_views = dp.shard(list(range(batch)), trainer.rank, trainer.world)
    start_active = trainer.active
    trainer.opac_reg, trainer.scale_reg = float(opac_reg), float(scale_reg)
    losses = []
    for step in range(1, steps + 1):
        idx = []
        while len(idx) < batch:
            if oi >= len(order):
                order = rng.permutation(len(views))
                oi = 0
            idx.append(int(order[oi]))
            oi += 1
        trainer.lrs["means"] = lr0 * decay ** step
        trainer.reg_weight = max(0.0, 1.0 - step / (0.9 * steps))
        trainer.sh_degree = min(3, step // sh_warmup) if sh_warmup else 3
        if filter_3d_every and (step == 1 or step % filter_3d_every == 0):
            trainer.compute_filter_3d(views)
        mine = [idx[i] for i in rank_views]
        # host images as they are (uint8 bytes or float32 in [0, 1]): the
        # trainer copies them while it bins and its loss reads bytes directly
        ts = []
        for i in mine:
            t = torch.as_tensor(targets[i])
            ts.append(t if t.dtype == torch.uint8 else t.float())
        losses.append(float(trainer.train_step([views[i] for i in mine], ts, batch)))
        if noise_weight:
            trainer.add_noise(trainer.lrs["means"], noise_weight)
        densify_now = bool(relocate_every) and step % relocate_every == 0
        if densify_now and step < (relocate_until if relocate_until is not None else steps + 1):
            trainer.relocate()
        if densify_now and grow_to is not None and step <= (grow_until or steps):
            frac = min(1.0, step / max(grow_until or steps, 1))
            trainer.grow(int(start_active + (grow_to - start_active) * frac))
        if callback is not None:
            callback(step, losses[-1])
    trainer.check_device_error()
    return losses

