"""The fused RVQ-driven frame: decode -> activate -> rasterize -> MLP -> mask/bg.

One `FrameRenderer.render(camera)` is one call of ns_render_frame on torch's
current stream. Scene tensors are uploaded once (the model: codebooks, base
attributes, hash table, MLP weights); the per-frame input is the RVQ index
stream, which `upload_indices` copies host -> device. `FramePipeline` renders
a sequence of frames with each frame's host <-> device copies overlapping the
neighbouring frames' kernels.
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
        self._extra_flags = 0

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
               events=None, skip_decode: bool = False, rvq_idx: torch.Tensor | None = None,
               rgb: torch.Tensor | None = None):
        """Renders one frame; returns the rgb [3,H,W] tensor (reused across calls).

        events: optional 2*NS_FRAME_STAGES torch.cuda.Event(enable_timing=True),
        recorded before/after decode, preprocess, binning, blend and MLP.
        skip_decode: `self.decoded` already holds the decoded attributes.
        rvq_idx / rgb: device index stream to decode and image to write, in place
        of the renderer's own buffers."""
        lib = _lib.load()
        self._outputs(cam)
        idx_t = self.rvq_idx if rvq_idx is None else rvq_idx
        rgb_t = self.rgb if rgb is None else rgb
        if idx_t.shape != self.rvq_idx.shape or rgb_t.shape != self.rgb.shape:
            raise ValueError("rvq_idx / rgb do not match the renderer's buffers")
        if view is None:
            view = cam.world_view_transform.to(self.device).contiguous()
        if proj is None:
            proj = cam.full_proj_transform.to(self.device).contiguous()
        st = self.settings(cam, view, proj)
        fin = _lib.FrameInputs()
        fin.P = self.P
        fin.rvq_idx, fin.codebooks = ptr(idx_t), ptr(self.codebooks)
        # with skip_decode, `decoded` may hold only the leading attribute columns
        # (e.g. the 10 an exchange gathered): dims is then its row stride; the
        # decode writes every column, so it needs a full [P, dims] buffer
        if skip_decode:
            if self.decoded.dim() != 2 or self.decoded.shape[0] != self.P or self.decoded.shape[1] < 10 \
                    or not self.decoded.is_contiguous():
                raise ValueError("decoded must be a contiguous [P, >=10] buffer")
        elif tuple(self.decoded.shape) != (self.P, self.dims) or not self.decoded.is_contiguous():
            raise ValueError(f"decoding needs a contiguous [{self.P}, {self.dims}] `decoded` buffer")
        fin.stages, fin.entries = self.stages, self.entries
        fin.dims = self.decoded.shape[1] if skip_decode else self.dims
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
        flags = (_lib.NS_FLAG_SKIP_DECODE if skip_decode else 0) | self._extra_flags
        fout = _lib.FrameOutputs()
        fout.rgb, fout.out_color = ptr(rgb_t), ptr(self.features)
        fout.out_others, fout.radii = ptr(self.others), ptr(self.radii)
        geom = self.scratch.geometry(self.P, self.device)
        image = self.scratch.image_buf(cam.width, cam.height, self.device)
        stream = _lib.stream_handle(self.device)
        n = C.c_int64(0)
        if self._extra_flags & _lib.NS_FLAG_DEVICE_COUNT:
            binning = self.scratch.bins(self.capacity, self.device)
            check("ns_render_frame", lib.ns_render_frame(
                C.byref(st), C.byref(fin), C.byref(fout), geom.data_ptr(), geom.numel(), binning.data_ptr(),
                binning.numel(), image.data_ptr(), image.numel(), C.byref(n), flags, stream))
            return rgb_t
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
        return rgb_t


class FramePipeline:
    """A sequence of frames with the host <-> device copies off the critical path.

    Frame i's inputs (its RVQ index stream and its [2,4,4] view / projection
    matrices, from pinned host memory) are copied on an input stream while
    frame i-1 renders, and frame i's image is copied back on an output stream
    while frame i+1 renders. Two device buffers of each, guarded by CUDA
    events; every frame still copies its own inputs in and its image out.
    With a DecodeShard (several ranks), each rank copies its own rows of the
    index stream; frame i+1's decode and all-gather run on a side stream
    (views.DecodeRing) while frame i renders.
    graphs=True (single rank): each buffer set's frame is a FrameGraph, so no
    frame waits for the host and the host never waits inside a frame.
    """

    def __init__(self, renderer: FrameRenderer, shard=None, depth: int = 2, graphs: bool = False):
        self.fr = renderer
        self.shard = shard
        if graphs and shard is not None:
            raise ValueError("graphs=True renders unsharded frames only")
        self.graphs = [] if graphs else None
        if shard is not None and depth != 2:
            raise ValueError("sharded frames alternate between two attribute buffers: depth must be 2")
        self.ring = None
        if shard is not None:
            from .views import DecodeRing
            self.ring = DecodeRing(renderer.rvq_idx, renderer.dims, shard.world, shard.rank,
                                   columns=shard.columns)
        d = renderer.device
        self.in_stream = torch.cuda.Stream(device=d)
        self.out_stream = torch.cuda.Stream(device=d)
        src = renderer.rvq_idx if shard is None else shard.idx_shard
        self.idx = [torch.zeros_like(src) for _ in range(depth)]
        self.cam = [torch.empty((2, 4, 4), dtype=torch.float32, device=d) for _ in range(depth)]
        self.rgb = [None] * depth
        self.depth = depth
        self.ev_in = [torch.cuda.Event() for _ in range(depth)]     # inputs on the device
        self.ev_done = [torch.cuda.Event() for _ in range(depth)]   # frame rendered, inputs free
        self.ev_host = [torch.cuda.Event() for _ in range(depth)]   # image on the host
        self.used = [False] * depth

    def run(self, n: int, cam: Camera, host_idx, host_cam, host_rgb, before_frame=None):
        """Renders n frames of camera `cam`'s size. host_idx(i) and host_cam(i) return
        frame i's pinned host inputs (the full [P, stages] index stream; [2,4,4] view and
        projection matrices), host_rgb(i) its pinned host image [3,H,W]. before_frame(i),
        if given, runs on the compute stream before frame i. Returns with the last
        copy enqueued; synchronise the output stream (or the device) to read it."""
        fr, sh = self.fr, self.shard
        cs = torch.cuda.current_stream(fr.device)
        fr._outputs(cam)
        if sh is not None:
            return self._run_sharded(n, cam, host_idx, host_cam, host_rgb, before_frame, cs)
        for i in range(n):
            k = i % self.depth
            if self.rgb[k] is None or self.rgb[k].shape != fr.rgb.shape:
                self.rgb[k] = torch.empty_like(fr.rgb)
            with torch.cuda.stream(self.in_stream):
                if self.used[k]:
                    self.in_stream.wait_event(self.ev_done[k])
                self.idx[k].copy_(host_idx(i), non_blocking=True)
                self.cam[k].copy_(host_cam(i), non_blocking=True)
                self.ev_in[k].record(self.in_stream)
            cs.wait_event(self.ev_in[k])
            if self.used[k]:
                cs.wait_event(self.ev_host[k])
            if before_frame is not None:
                before_frame(i)
            if self.graphs is not None:
                if len(self.graphs) <= k:
                    self.graphs.append(FrameGraph(fr, cam, self.cam[k][0], self.cam[k][1], rvq_idx=self.idx[k],
                                                  rgb=self.rgb[k]))
                self.graphs[k].replay()
            else:
                fr.render(cam, self.cam[k][0], self.cam[k][1], rvq_idx=self.idx[k], rgb=self.rgb[k])
            self.ev_done[k].record(cs)
            with torch.cuda.stream(self.out_stream):
                self.out_stream.wait_event(self.ev_done[k])
                host_rgb(i).copy_(self.rgb[k], non_blocking=True)
                self.ev_host[k].record(self.out_stream)
            self.used[k] = True

    def _run_sharded(self, n, cam, host_idx, host_cam, host_rgb, before_frame, cs):
        from .views import shard_range
        fr, sh, ring = self.fr, self.shard, self.ring
        lo, hi = shard_range(sh.P, sh.world, sh.rank)

        def stage(i):
            # Frame i's inputs on the input stream, then its decode + all-gather on
            # the ring's stream (collectives in frame order on every rank).
            k = i % 2
            with torch.cuda.stream(self.in_stream):
                if self.used[k]:
                    self.in_stream.wait_event(self.ev_done[k])
                ring.shards[k].idx_shard[: hi - lo].copy_(host_idx(i)[lo:hi], non_blocking=True)
                self.cam[k].copy_(host_cam(i), non_blocking=True)
                self.ev_in[k].record(self.in_stream)
            ring.stream.wait_event(self.ev_in[k])
            ring.prefetch(i, fr.codebooks, _rvq_decode)

        if n > 0:
            stage(0)
        for i in range(n):
            k = i % 2
            if i + 1 < n:
                stage(i + 1)
            if self.rgb[k] is None or self.rgb[k].shape != fr.rgb.shape:
                self.rgb[k] = torch.empty_like(fr.rgb)
            cs.wait_event(self.ev_in[k])
            if self.used[k]:
                cs.wait_event(self.ev_host[k])
            if before_frame is not None:
                before_frame(i)
            fr.decoded = ring.acquire(i, cs)
            fr.render(cam, self.cam[k][0], self.cam[k][1], skip_decode=True, rgb=self.rgb[k])
            ring.release(i, cs)
            self.ev_done[k].record(cs)
            with torch.cuda.stream(self.out_stream):
                self.out_stream.wait_event(self.ev_done[k])
                host_rgb(i).copy_(self.rgb[k], non_blocking=True)
                self.ev_host[k].record(self.out_stream)
            self.used[k] = True


def _rvq_decode(idx, codebooks, out=None):
    from .raster import rvq_decode
    return rvq_decode(idx, codebooks, out=out)


class FrameGraph:
    """One frame recorded as a CUDA graph and replayed on the current stream.

    The frame runs with the device-side instance count (NS_FLAG_DEVICE_COUNT):
    binning never reads the count back, so nothing in the frame waits for the
    host and the whole decode -> preprocess -> binning -> blend -> MLP sequence
    replays as one graph launch. The binning buffers are sized from an ordinary
    frame of the same camera times `headroom`; a frame that outgrows them sets
    the device error word (ns_read_device_status) and renders nothing.
    Inputs are read from the renderer's buffers (rvq_idx, or `decoded` with
    skip_decode) and the given view / projection tensors, in place; the image
    lands in renderer.rgb.
    """

    def __init__(self, renderer: FrameRenderer, cam: Camera, view: torch.Tensor, proj: torch.Tensor,
                 skip_decode: bool = False, headroom: float = 1.5, rvq_idx: torch.Tensor | None = None,
                 rgb: torch.Tensor | None = None):
        fr = self.fr = renderer
        kw = dict(skip_decode=skip_decode, rvq_idx=rvq_idx, rgb=rgb)
        fr.render(cam, view, proj, **kw)  # sizes the buffers (host count)
        fr.capacity = max(fr.capacity, int(fr.num_rendered * headroom) + 1024)
        fr.scratch.bins(fr.capacity, fr.device)
        fr._extra_flags = _lib.NS_FLAG_DEVICE_COUNT
        try:
            side = torch.cuda.Stream(device=fr.device)
            side.wait_stream(torch.cuda.current_stream(fr.device))
            with torch.cuda.stream(side):
                fr.render(cam, view, proj, **kw)  # first device-count frame, uncaptured
            torch.cuda.current_stream(fr.device).wait_stream(side)
            torch.cuda.synchronize(fr.device)
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph, stream=side):
                fr.render(cam, view, proj, **kw)
        finally:
            fr._extra_flags = 0
        self.rgb = fr.rgb if rgb is None else rgb

    def replay(self) -> torch.Tensor:
        self.graph.replay()
        return self.rgb

    def status(self) -> int:
        """Reads and clears the frame's device error word (syncs the stream)."""
        lib = _lib.load()
        geom = self.fr.scratch.geom
        return lib.ns_read_device_status(geom.data_ptr(), self.fr.P, _lib.stream_handle(self.fr.device))
