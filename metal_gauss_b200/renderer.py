"""Forward-only rendering of many views on one GPU.

The reference's viewer and camera-path renderer call `render` under
`torch.no_grad()` view after view (viewer.py:477-485, render_path.py:
440-456). This renderer keeps the Gaussians resident in the form the kernels
read. Per batch of views it projects and colours every view in one launch,
runs the antialias opacity compensation of every view in one more when asked
for (metal_backend.py:506-511), and bins the views with the saturation cut
(one call per binning stage for all views of one frame size, one host read
per batch for the pair totals); then per view, on four streams in turn, it
packs the splats and runs a forward-only rasterisation that writes no
transmittance, stop indices or checkpoints and keeps no autograd state.
"""

from __future__ import annotations

import torch

from . import _lib
from ._lib import ptr
from .engine import _BatchBinning, _ViewBatch, _ViewState, _views_array


class _FrameBuffers:
    """Per-resolution scratch of the forward-only path (no transmittance,
    stop indices, gradients or loss scratch)."""

    def __init__(self, n: int, device):
        self.splats = torch.empty(n, _lib.SPLAT_FLOATS, dtype=torch.float32, device=device)
        self.raster = torch.empty(0, dtype=torch.uint8, device=device)
        self.ids = torch.empty(0, dtype=torch.int32, device=device)
        self.offsets = None
        self.emit = torch.empty(0, dtype=torch.uint8, device=device)


class Renderer:
    """`params` in the trainer's storage form (means, quats, log_scales,
    logit_opac, sh_dc (N,1,3), sh_rest (N,15,3)); activations, and
    Mip-Splatting's 3D filter when `filter_3d` (N,) is given, are applied
    once here."""

    def __init__(self, params: dict, device="cuda", *, sh_degree: int = 3, tile: int = 16,
                 background=(0.0, 0.0, 0.0), antialias: bool = False, near: float = 0.01,
                 far: float = 100.0, max_radius_frac: float = 1.0, saturation_cut: bool = True,
                 batch: int = 8, filter_3d=None):
        self.device = torch.device(device)
        f32 = dict(dtype=torch.float32, device=self.device)
        self.n = n = int(params["means"].shape[0])
        self.means = params["means"].to(**f32).reshape(n, 3).contiguous()
        self.quats = params["quats"].to(**f32).reshape(n, 4).contiguous()
        self.scales = torch.exp(params["log_scales"].to(**f32)).reshape(n, 3).contiguous()
        self.opac = torch.sigmoid(params["logit_opac"].to(**f32)).reshape(n).contiguous()
        if filter_3d is not None:  # Mip-Splatting's 3D filter, applied once (train.py:223-227)
            f = torch.as_tensor(filter_3d).to(**f32).reshape(n).contiguous()
            scales, opac = torch.empty_like(self.scales), torch.empty_like(self.opac)
            _lib.call("mg_apply_3d_filter", ptr(self.scales), ptr(self.opac), ptr(f), n,
                      ptr(scales), ptr(opac), _lib.stream())
            self.scales, self.opac = scales, opac
        self.sh_dc = params["sh_dc"].to(**f32).reshape(n, 1, 3).contiguous()
        self.sh_rest = params["sh_rest"].to(**f32).reshape(n, 15, 3).contiguous()
        self.sh_degree, self.tile = sh_degree, tile
        self.antialias = antialias
        self.near, self.far, self.max_radius_frac = near, far, max_radius_frac
        self.saturation_cut = int(bool(saturation_cut))
        self.background = None if background is None or all(b == 0 for b in background) \
            else tuple(float(b) for b in background)
        self.batch = batch
        self._batch = _ViewBatch(n, batch, self.device, grads=False)
        self._states = [_ViewState(self._batch, v, self.device) for v in range(batch)]
        self._bufs: dict = {}
        # per-view opacity after the antialias compensation (view-major)
        self._opac_view = torch.empty(batch if antialias else 0, n, **f32)
        # pair totals of the one-view-at-a-time binning, then the error word
        self._totals = torch.zeros(batch + 1, dtype=torch.int64, device=self.device)
        self._bb = _BatchBinning(self.device)
        self.batch_binning = True
        # views are packed and rasterised on this many streams in turn (one
        # view's raster tail overlaps the next view's work)
        self.view_streams = 4
        self._streams: list = []

    def _camera(self, view) -> _lib.Camera:
        vm = view.viewmat.to(torch.float32)
        K = view.K
        cc = -vm[:3, :3].T @ vm[:3, 3]
        return _lib.make_camera(vm, float(K[0, 0]), float(K[1, 1]), float(K[0, 2]),
                                float(K[1, 2]), view.width, view.height, self.near, self.far, 0.3,
                                self.max_radius_frac * max(view.width, view.height), cc)

    def _state(self, v: int) -> _ViewState:
        return self._states[v]

    def _opacity(self, v: int) -> torch.Tensor:
        return self._opac_view[v] if self.antialias else self.opac

    def _buffers(self, W: int, H: int, slot: int = 0) -> _FrameBuffers:
        b = self._bufs.get((W, H, slot))
        if b is None:
            b = _FrameBuffers(self.n, self.device)
            self._bufs[(W, H, slot)] = b
        return b

    def render(self, views, check: bool = True) -> list[tuple[torch.Tensor, torch.Tensor]]:
        """[(rgb (H,W,3), alpha (H,W))] device tensors, one pair per view.
        Each batch's pair-total read also checks the device error word; with
        `check` (default) one more synchronising read after the last batch
        covers its kernels, so a failed bounded wait or bad index raises
        _lib.DeviceError instead of returning wrong frames."""
        out = []
        for i in range(0, len(views), self.batch):
            out += self._render_batch(views[i:i + self.batch])
        if check:
            _lib.check_device_error("render")
        return out

    def _render_batch(self, views):
        L = _lib.load()
        s = _lib.stream()
        n = self.n
        b = self._batch
        cams = _views_array([self._camera(v) for v in views])
        # every view's projection + SH colour in one launch
        _lib.check(L.mg_preprocess_forward_views(
            ptr(self.means), ptr(self.quats), ptr(self.scales), ptr(self.sh_dc),
            ptr(self.sh_rest), _lib.SH_SPLIT, ptr(self.opac), _lib.C.cast(cams, _lib.C.c_void_p),
            len(views), self.sh_degree, n, n, ptr(b.uv), ptr(b.conic), ptr(b.depth), ptr(b.rxy),
            ptr(b.valid), ptr(b.color), None, None, s), "preprocess_forward_views")
        V = len(views)
        if self.antialias:
            # every view's compensated opacities in one launch, before binning
            # as the reference does: the exact tile test then uses the opacity
            # that is composited
            _lib.check(L.mg_antialias_opacity_views(ptr(b.conic), ptr(self.opac), n, V, n, 0.3,
                                                    ptr(self._opac_view), s),
                       "antialias_opacity_views")
        opac_all, opac_stride = (self._opac_view, n) if self.antialias else (self.opac, 0)
        totals = None
        if self.batch_binning and _BatchBinning.fits(views, n):
            W, H = views[0].width, views[0].height
            self._bb.prepare(self._batch, 0, V, n, W, H, self.tile, self.saturation_cut,
                             opac_all, opac_stride)
            totals = self._bb.read_totals(V)
            if totals is not None:
                self._bb.emit_all(self._batch, V, n, W, H, self.tile, self.saturation_cut,
                                  opac_all, opac_stride, sum(totals))
        batched = totals is not None
        if not batched:
            for v, view in enumerate(views):
                st = self._state(v)
                tiles = -(-view.width // self.tile) * -(-view.height // self.tile)
                prep = st.prep_scratch(tiles)
                _lib.check(L.mg_bin_prepare(
                    ptr(st.uv), ptr(st.rxy), ptr(st.conic), ptr(self._opacity(v)),
                    ptr(st.valid), ptr(st.depth), n, view.width, view.height, self.tile,
                    self.saturation_cut, ptr(self._totals[v:v + 1]), ptr(prep), prep.numel(),
                    s), "bin_prepare")
            _lib.call("mg_peek_device_error", ptr(self._totals[-1:]), s)
            t = self._totals.tolist()
            if t[-1]:
                _lib.raise_device_error(t[-1], "render binning")
            totals = t[:V]
        bg = None if self.background is None else (_lib.C.c_float * 3)(*self.background)
        bgp = None if bg is None else _lib.C.cast(bg, _lib.C.c_void_p)
        k = min(int(self.view_streams), V)
        while len(self._streams) < k:
            self._streams.append(torch.cuda.Stream(self.device))
        main = torch.cuda.current_stream(self.device)
        ready = torch.cuda.Event()
        ready.record(main)
        streams = self._streams[:k] if k > 1 else [main]
        if k > 1:
            for sk in streams:
                sk.wait_event(ready)
        out = []
        for v, (view, m) in enumerate(zip(views, totals)):
            # the outputs belong to the caller's stream, which waits below
            rgb = torch.empty(view.height, view.width, 3, dtype=torch.float32, device=self.device)
            alpha = torch.empty(view.height, view.width, dtype=torch.float32, device=self.device)
            with torch.cuda.stream(streams[v % k]):
                self._render_view(v, view, int(m), batched, v % k, rgb, alpha, bgp)
            out.append((rgb, alpha))
        if k > 1:
            for sk in streams:
                done = torch.cuda.Event()
                done.record(sk)
                main.wait_event(done)
        return out

    def _render_view(self, v: int, view, m: int, batched: bool, slot: int, rgb, alpha, bgp):
        """Pair lists (unless the batch has them), packing and the forward-only
        rasterisation of view v on the current stream."""
        L = _lib.load()
        s = _lib.stream()
        n = self.n
        st = self._states[v]
        opac = self._opacity(v)
        W, H = view.width, view.height
        b = self._buffers(W, H, slot)
        tiles_x, tiles_y = -(-W // self.tile), -(-H // self.tile)
        n_tiles = tiles_x * tiles_y
        rbytes = L.mg_raster_scratch_bytes(W, H, self.tile, m)
        if b.raster.numel() < rbytes:
            b.raster = torch.empty(int(rbytes * 1.25) + 256, dtype=torch.uint8,
                                   device=self.device)
        if batched:
            ids, offsets = self._bb.view(v, m)
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
            _lib.check(L.mg_bin_emit(ptr(st.uv), ptr(st.rxy), ptr(st.conic), ptr(opac), n,
                                     m, W, H, self.tile, self.saturation_cut, ptr(st.prep),
                                     ptr(b.ids), ptr(b.offsets), ptr(b.emit),
                                     b.emit.numel(), s), "bin_emit")
            ids, offsets = b.ids, b.offsets
        _lib.check(L.mg_pack_splats(ptr(st.uv), ptr(st.conic), ptr(opac), ptr(st.color),
                                    n, ptr(b.splats), None, s), "pack_splats")
        _lib.check(L.mg_rasterize_forward(
            ptr(b.splats), ptr(ids), ptr(offsets), m, W, H, self.tile, tiles_x, bgp,
            ptr(rgb), ptr(alpha), None, None, None, ptr(b.raster), b.raster.numel(), s),
            "rasterize_forward")
