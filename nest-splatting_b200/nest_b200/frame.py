"""The fused RVQ-driven frame: decode -> activate -> rasterize -> MLP -> mask/bg.

One `FrameRenderer.render(camera)` is one call of ns_render_frame on torch's
current stream. Scene tensors are uploaded once (the model: codebooks, base
attributes, hash table, MLP weights); the per-frame input is the RVQ index
stream, which `upload_indices` copies host -> device.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib
from ._lib import check, ptr
from .camera import Camera
from .raster import OTHER_CHANNELS, Scratch, pack_mlp
from .synth import Scene


class FrameRenderer:
    def __init__(self, scene: Scene, device="cuda", capacity: int | None = None, bg=(0.0, 0.0, 0.0)):
        if scene.codebooks is None:
            raise ValueError("the fused frame needs an RVQ scene")
        self.device = torch.device(device)
        d = self.device
        self.P = scene.P
        self.base = scene.base.to(d).contiguous()
        self.codebooks = scene.codebooks.to(d).contiguous()
        self.rvq_idx = scene.rvq_idx.to(d).contiguous()
        self.stages, self.entries, self.dims = scene.codebooks.shape
        self.mix = float(scene.mix)
        self.ap_level = scene.ap_level.to(d).contiguous()
        g = scene.grid
        self.grid = g
        self.table = g.table.to(d).contiguous()
        self.offsets = g.offsets.to(d).contiguous()
        self.gridrange = g.gridrange.float().to(d).contiguous()
        self.mlp = pack_mlp(scene.mlp).to(d)
        self.mlp_hidden = scene.mlp[0].shape[0]
        self.decoded = torch.empty((self.P, self.dims), dtype=torch.float32, device=d)
        self.radii = torch.empty((self.P,), dtype=torch.int32, device=d)
        self.scratch = Scratch()
        self.capacity = capacity or 4 * self.P
        self.bg = (C.c_float * 3)(*[float(x) for x in bg])
        self._out_shape = None
        self.num_rendered = 0

    def _outputs(self, cam: Camera):
        shape = (cam.height, cam.width)
        if self._out_shape != shape:
            d = self.device
            self.rgb = torch.empty((3,) + shape, dtype=torch.float32, device=d)
            self.features = torch.empty((self.grid.channels,) + shape, dtype=torch.float32, device=d)
            self.others = torch.empty((OTHER_CHANNELS,) + shape, dtype=torch.float32, device=d)
            self._out_shape = shape

    def settings(self, cam: Camera, view: torch.Tensor, proj: torch.Tensor) -> _lib.RasterSettings:
        s = _lib.RasterSettings()
        s.image_height, s.image_width = cam.height, cam.width
        s.tanfovx, s.tanfovy = cam.tanfovx, cam.tanfovy
        s.scale_modifier = 1.0
        s.viewmatrix, s.projmatrix = view.data_ptr(), proj.data_ptr()
        s.beta = 0.0
        s.levels = self.grid.levels
        s.level_scale_log2 = self.grid.S
        s.base_resolution = self.grid.base_resolution
        s.align_corners = int(self.grid.align_corners)
        s.interpolation = self.grid.interpolation
        s.channels = self.grid.channels
        s.level_dim = self.grid.level_dim
        s.table_fp16 = int(self.table.dtype == torch.float16)
        return s

    def upload_indices(self, host_idx: torch.Tensor) -> None:
        """Copies a (pinned) host index stream into the device buffer on the current stream."""
        self.rvq_idx.copy_(host_idx, non_blocking=True)

    def render(self, cam: Camera, view: torch.Tensor | None = None, proj: torch.Tensor | None = None,
               events=None, skip_decode: bool = False):
        """Renders one frame; returns the rgb [3,H,W] tensor (reused across calls).

        events: optional 2*NS_FRAME_STAGES torch.cuda.Event(enable_timing=True),
        recorded before/after decode, preprocess, binning, blend and MLP.
        skip_decode: `self.decoded` already holds the decoded attributes."""
        lib = _lib.load()
        self._outputs(cam)
        if view is None:
            view = cam.world_view_transform.to(self.device).contiguous()
        if proj is None:
            proj = cam.full_proj_transform.to(self.device).contiguous()
        st = self.settings(cam, view, proj)
        fin = _lib.FrameInputs()
        fin.P = self.P
        fin.rvq_idx, fin.codebooks = ptr(self.rvq_idx), ptr(self.codebooks)
        fin.stages, fin.entries, fin.dims = self.stages, self.entries, self.dims
        fin.base, fin.mix, fin.decoded = ptr(self.base), self.mix, ptr(self.decoded)
        fin.ap_level, fin.features = ptr(self.ap_level), ptr(self.table)
        fin.offsets, fin.gridrange = ptr(self.offsets), ptr(self.gridrange)
        fin.mlp_weights, fin.mlp_hidden = ptr(self.mlp), self.mlp_hidden
        fin.bg_host = C.cast(self.bg, C.c_void_p)
        ev_arr = None
        if events is not None:
            assert len(events) == 2 * _lib.NS_FRAME_STAGES
            ev_arr = (C.c_void_p * len(events))(*[e.cuda_event for e in events])
            fin.stage_events = C.cast(ev_arr, C.c_void_p)
        flags = _lib.NS_FLAG_SKIP_DECODE if skip_decode else 0
        fout = _lib.FrameOutputs()
        fout.rgb, fout.out_color = ptr(self.rgb), ptr(self.features)
        fout.out_others, fout.radii = ptr(self.others), ptr(self.radii)
        geom = self.scratch.geometry(self.P, self.device)
        image = self.scratch.image_buf(cam.width, cam.height, self.device)
        stream = _lib.stream_handle(self.device)
        n = C.c_int64(0)
        for _ in range(2):
            binning = self.scratch.bins(self.capacity, self.device)
            rc = lib.ns_render_frame(C.byref(st), C.byref(fin), C.byref(fout), geom.data_ptr(),
                                     geom.numel(), binning.data_ptr(), binning.numel(),
                                     image.data_ptr(), image.numel(), C.byref(n), flags, stream)
            if rc == _lib.NS_ERR_CAPACITY:
                self.capacity = int(n.value * 1.25) + 1024
                continue
            check("ns_render_frame", rc)
            break
        self.num_rendered = int(n.value)
        return self.rgb
