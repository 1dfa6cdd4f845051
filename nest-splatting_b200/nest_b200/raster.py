"""Torch-facing wrappers of the C-ABI (device memory and streams come from torch).

Every function here enqueues the library's kernels on torch's current CUDA
stream. Tensors must be contiguous CUDA tensors of the stated dtypes.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import torch

from . import _lib
from ._lib import check, ptr

OTHER_CHANNELS = 14


def _require_cuda(*ts):
    for t in ts:
        if t is not None and (not t.is_cuda or not t.is_contiguous()):
            raise ValueError("expected contiguous CUDA tensors")


@dataclass
class RasterConfig:
    """Plain mirror of GaussianRasterizationSettings + HashGridSettings."""
    image_height: int
    image_width: int
    tanfovx: float
    tanfovy: float
    viewmatrix: torch.Tensor
    projmatrix: torch.Tensor
    scale_modifier: float = 1.0
    beta: float = 0.0
    if_contract: bool = False
    record_transmittance: bool = False
    max_intersections: int = 0
    prefiltered: bool = False
    levels: int = 16
    S: float = 0.0
    base_resolution: int = 16
    align_corners: bool = False
    interpolation: int = 0
    channels: int = 32
    level_dim: int = 2
    table_fp16: bool = True
    kernel_type: int = 0  # 0 Gaussian, 1 beta, 2 flex, 3 general
    deterministic: bool = False  # backward: fixed-point (bit-reproducible) table gradient
    render_mode: int = 0     # 0 baseline (levels 0: per-surfel colours); 4 cat, 6 adaptive, 7 adaptive_add,
    #                          8 hybrid_SH, 9 hybrid_SH_post, 10 hybrid_SH_raw, 11 residual_hybrid,
    #                          12 adaptive_cat, 13 adaptive_cat_fast, 14 adaptive_zero (| 256 inference)
    hybrid_levels: int = 0   # per-surfel feature levels of modes 4 / 12 / 14; modes 8-10: the decompose flag
    total_levels: int = 0    # all levels (mode 12 rows hold total_levels * level_dim + 1)
    sh_degree: int = 0       # level 0 with SH coefficients: the degree evaluated (0-3)
    campos: object = None    # level 0 with SH coefficients: camera centre, device tensor [3]

    @property
    def other_channels(self) -> int:
        """out_others channels: 14, and 17 in mode 11 (its SH colour in 14-16)."""
        return OTHER_CHANNELS + 3 if (int(self.render_mode) & 0xFF) == 11 else OTHER_CHANNELS

    @property
    def uses_rows(self) -> bool:
        """Samples read per-surfel rows (colors_precomp): every mode but 0, and level 0."""
        return int(self.render_mode) != 0 or int(self.levels) == 0

    def to_c(self) -> _lib.RasterSettings:
        s = _lib.RasterSettings()
        s.image_height = int(self.image_height)
        s.image_width = int(self.image_width)
        s.tanfovx = float(self.tanfovx)
        s.tanfovy = float(self.tanfovy)
        s.scale_modifier = float(self.scale_modifier)
        s.viewmatrix = self.viewmatrix.data_ptr()
        s.projmatrix = self.projmatrix.data_ptr()
        s.beta = float(self.beta)
        s.kernel_type = int(self.kernel_type)
        s.deterministic = int(bool(self.deterministic))
        s.render_mode = int(self.render_mode)
        s.hybrid_levels = int(self.hybrid_levels)
        s.total_levels = int(self.total_levels)
        s.if_contract = int(bool(self.if_contract))
        s.record_transmittance = int(bool(self.record_transmittance))
        s.max_intersections = int(self.max_intersections)
        s.prefiltered = int(bool(self.prefiltered))
        s.levels = int(self.levels)
        s.level_scale_log2 = float(self.S)
        s.base_resolution = int(self.base_resolution)
        s.align_corners = int(bool(self.align_corners))
        s.interpolation = int(self.interpolation)
        s.channels = int(self.channels)
        s.level_dim = int(self.level_dim)
        s.table_fp16 = int(bool(self.table_fp16))
        s.sh_degree = int(self.sh_degree)
        s.campos = None if self.campos is None else self.campos.data_ptr()
        return s


class Scratch:
    """Per-device scratch buffers reused across calls (grown on demand)."""

    def __init__(self):
        self.geom = None
        self.image = None
        self.binning = None
        self.capacity = 0

    @staticmethod
    def _ensure(buf, nbytes, device):
        if buf is None or buf.numel() < nbytes or buf.device != device:
            return torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=device)
        return buf

    def geometry(self, P, device):
        lib = _lib.load()
        self.geom = self._ensure(self.geom, lib.ns_geometry_scratch_bytes(P), device)
        return self.geom

    def image_buf(self, W, H, device):
        lib = _lib.load()
        self.image = self._ensure(self.image, lib.ns_image_scratch_bytes(W, H), device)
        return self.image

    def bins(self, capacity, device):
        lib = _lib.load()
        if self.binning is None or capacity > self.capacity or self.binning.device != device:
            self.capacity = int(capacity)
            self.binning = torch.empty(lib.ns_binning_scratch_bytes(self.capacity), dtype=torch.uint8,
                                       device=device)
        return self.binning


def rasterize_forward(cfg: RasterConfig, means3D, scales, rotations, opacities, homotrans, ap_level,
                      features, offsets, gridrange, scratch: Scratch | None = None,
                      capacity_hint: int | None = None, shapes=None, colors_precomp=None, shs=None,
                      transmat_precomp=None):
    """Forward rasterization through ns_rasterize_forward. Every render mode but
    0 (and level 0) reads the per-surfel rows `colors_precomp` (contiguous fp32);
    level 0 may take SH coefficients `shs` [P, M, 3] instead (colours evaluated
    at cfg.sh_degree from cfg.campos, C = 3). `transmat_precomp` [P, 9]
    (contiguous fp32, columns Tu, Tv, Tw) replaces the transforms built from
    scales and rotations (which may then be None; homotrans is required).

    Returns (num_rendered, out_color [C,H,W], out_others [14,H,W] ([17,H,W] in
    mode 11), radii [P] int32, cover_pixels [P,1], trans_avg [P,1], scratch).
    """
    lib = _lib.load()
    dev = means3D.device
    P = means3D.shape[0]
    H, W = int(cfg.image_height), int(cfg.image_width)
    Cc = int(cfg.channels)
    _require_cuda(means3D, scales, rotations, opacities, homotrans, ap_level, features, offsets,
                  gridrange, cfg.viewmatrix, cfg.projmatrix)
    out_color = torch.zeros((Cc, H, W), dtype=torch.float32, device=dev)
    out_others = torch.zeros((cfg.other_channels, H, W), dtype=torch.float32, device=dev)
    radii = torch.zeros((P,), dtype=torch.int32, device=dev)
    rec_P = P if cfg.record_transmittance else 0
    cover = torch.zeros((rec_P, 1), dtype=torch.float32, device=dev)
    trans = torch.zeros((rec_P, 1), dtype=torch.float32, device=dev)
    if P == 0:
        return 0, out_color, out_others, radii, cover, trans, scratch
    scratch = scratch or Scratch()
    settings = cfg.to_c()
    surf = _lib.Surfels()
    surf.P = P
    surf.means3D, surf.scales, surf.rotations = ptr(means3D), ptr(scales), ptr(rotations)
    surf.opacities, surf.homotrans, surf.ap_level = ptr(opacities), ptr(homotrans), ptr(ap_level)
    surf.features, surf.offsets, surf.gridrange = ptr(features), ptr(offsets), ptr(gridrange)
    surf.shapes = ptr(shapes)
    _set_transmats(surf, transmat_precomp, homotrans, P)
    if cfg.uses_rows:
        if colors_precomp is None and (shs is None or cfg.render_mode != 0):
            raise ValueError(f"render_mode {cfg.render_mode} with {cfg.levels} levels needs colors_precomp")
        if colors_precomp is not None:
            _require_cuda(colors_precomp)
            surf.colors_precomp = ptr(colors_precomp)
        else:
            _set_shs(cfg, surf, shs, P)
    outs = _lib.RasterOutputs()
    outs.out_color, outs.out_others, outs.radii = ptr(out_color), ptr(out_others), ptr(radii)
    outs.cover_pixels = ptr(cover) if rec_P else None
    outs.trans_avg = ptr(trans) if rec_P else None
    geom = scratch.geometry(P, dev)
    image = scratch.image_buf(W, H, dev)
    cap = max(scratch.capacity, capacity_hint or 4 * P, 1024)
    stream = _lib.stream_handle(dev)
    n = C.c_int64(0)
    for _ in range(2):
        binning = scratch.bins(cap, dev)
        rc = lib.ns_rasterize_forward(C.byref(settings), C.byref(surf), C.byref(outs),
                                      geom.data_ptr(), geom.numel(), binning.data_ptr(),
                                      binning.numel(), image.data_ptr(), image.numel(), C.byref(n),
                                      0, stream)
        if rc == _lib.NS_ERR_CAPACITY:
            cap = int(n.value * 1.25) + 1024
            continue
        check("ns_rasterize_forward", rc)
        break
    return int(n.value), out_color, out_others, radii, cover, trans, scratch


def _set_shs(cfg: RasterConfig, surf, shs, P: int) -> None:
    if shs.numel() % (3 * max(P, 1)) or shs.dtype != torch.float32 or not shs.is_contiguous():
        raise ValueError("shs must be contiguous fp32 [P, M, 3]")
    if cfg.campos is None:
        raise ValueError("SH colours need cfg.campos (the camera centre, device [3])")
    _require_cuda(shs, cfg.campos)
    surf.shs = ptr(shs)
    surf.sh_coeffs = shs.numel() // (3 * max(P, 1))


def _set_transmats(surf, transmat_precomp, homotrans, P: int) -> None:
    if transmat_precomp is None:
        return
    if transmat_precomp.numel() != 9 * P or transmat_precomp.dtype != torch.float32:
        raise ValueError("transmat_precomp must be fp32 [P, 9]")
    if homotrans is None:
        raise ValueError("precomputed transforms need homotrans (the hit point's frame)")
    _require_cuda(transmat_precomp)
    surf.transmat_precomp = ptr(transmat_precomp)


def read_binning(scratch: Scratch, P: int, width: int, height: int, num_rendered: int) -> dict:
    """What the last forward call on `scratch` left in it (ns_read_binning):
    point_list [num_rendered] int32 (surfel ids per tile in depth order),
    ranges [tiles, 2] int32, tile_rects [P, 4] int16 (x0, y0, x1, y1),
    depths [P], pixel_boxes [P, 4] (x0, x1, y0, y1), means2D [P, 2]."""
    lib = _lib.load()
    dev = scratch.geom.device
    tiles = ((width + 15) // 16) * ((height + 15) // 16)
    out = dict(point_list=torch.empty(max(num_rendered, 1), dtype=torch.int32, device=dev),
               ranges=torch.empty((tiles, 2), dtype=torch.int32, device=dev),
               tile_rects=torch.empty((max(P, 1), 4), dtype=torch.int16, device=dev),
               depths=torch.empty(max(P, 1), dtype=torch.float32, device=dev),
               pixel_boxes=torch.empty((max(P, 1), 4), dtype=torch.float32, device=dev),
               means2D=torch.empty((max(P, 1), 2), dtype=torch.float32, device=dev))
    binning = scratch.binning
    check("ns_read_binning", lib.ns_read_binning(
        scratch.geom.data_ptr(), scratch.geom.numel(), P, ptr(binning), 0 if binning is None else binning.numel(),
        scratch.image.data_ptr(), scratch.image.numel(), width, height, num_rendered, ptr(out["point_list"]),
        ptr(out["ranges"]), ptr(out["tile_rects"]), ptr(out["depths"]), ptr(out["pixel_boxes"]),
        ptr(out["means2D"]), _lib.stream_handle(dev)))
    out["point_list"] = out["point_list"][:num_rendered]
    return {k: v[:P] if k in ("tile_rects", "depths", "pixel_boxes", "means2D") else v for k, v in out.items()}


def rasterize_backward(cfg: RasterConfig, means3D, scales, rotations, opacities, homotrans, ap_level, features,
                       offsets, gridrange, radii, num_rendered: int, scratch: Scratch, dL_dcolor, dL_dothers,
                       return_accumulators: bool = False, shapes=None, colors_precomp=None, shs=None,
                       transmat_precomp=None):
    """Backward rasterization (render_mode 0) through ns_rasterize_backward.

    `scratch` and every input must be the ones of the forward call. Returns a dict
    of fp32 gradients: means3D [P,3], means2D [P,3] (densification statistic),
    opacity [P,1], scales [P,2], rotations [P,4], table [rows, level_dim],
    gradsum [P,1]; for kernel_type 1-3 (`shapes` [P] as in the forward) also
    shapes [P]; for the modes that read per-surfel rows (`colors_precomp` as in
    the forward) also colors_precomp (same shape); for level 0 from SH (`shs` as
    in the forward) also shs [P, M, 3], the colour's mean gradient included in
    means3D; with `transmat_precomp` (as in the forward) also transmat_precomp
    [P, 9], and zeros for means3D, scales and rotations. With
    return_accumulators, also "accum": the render pass's
    per-surfel accumulators [P,20] (dL/dM 9, dL/dT[0].z, dL/dT[1].z, opacity,
    dL/dnormal 3, gradsum, dL/dmean2D 2, dL/dshape, 1 unused), for tests.
    """
    lib = _lib.load()
    dev = means3D.device
    P = means3D.shape[0]
    dL_dcolor = dL_dcolor.contiguous().float()
    dL_dothers = dL_dothers.contiguous().float()
    _require_cuda(means3D, scales, rotations, opacities, homotrans, ap_level, features, offsets, gridrange, radii,
                  dL_dcolor, dL_dothers)
    rows = int(features.shape[0])
    g = dict(means3D=torch.empty((P, 3), dtype=torch.float32, device=dev),
             means2D=torch.empty((P, 3), dtype=torch.float32, device=dev),
             opacity=torch.empty((P, 1), dtype=torch.float32, device=dev),
             scales=torch.empty((P, 2), dtype=torch.float32, device=dev),
             rotations=torch.empty((P, 4), dtype=torch.float32, device=dev),
             table=torch.empty((rows, int(cfg.level_dim)), dtype=torch.float32, device=dev),
             gradsum=torch.empty((P, 1), dtype=torch.float32, device=dev))
    if cfg.kernel_type != 0:
        if shapes is None or shapes.numel() != P:
            raise ValueError(f"kernel_type {cfg.kernel_type} needs shapes with one value per surfel")
        shapes = shapes.contiguous().float().reshape(-1)
        _require_cuda(shapes)
        g["shapes"] = torch.empty((P,), dtype=torch.float32, device=dev)
    if transmat_precomp is not None:
        g["transmat_precomp"] = torch.empty((P, 9), dtype=torch.float32, device=dev)
    if cfg.uses_rows and colors_precomp is None and shs is not None and cfg.render_mode == 0:
        g["shs"] = torch.zeros_like(shs)
    elif cfg.uses_rows:
        if colors_precomp is None:
            raise ValueError(f"render_mode {cfg.render_mode} with {cfg.levels} levels needs colors_precomp")
        colors_precomp = colors_precomp.contiguous().float()
        _require_cuda(colors_precomp)
        g["colors_precomp"] = torch.zeros_like(colors_precomp)
    if P == 0:
        g["table"].zero_()
        return g
    settings = cfg.to_c()
    surf = _lib.Surfels()
    surf.P = P
    surf.means3D, surf.scales, surf.rotations = ptr(means3D), ptr(scales), ptr(rotations)
    surf.opacities, surf.homotrans, surf.ap_level = ptr(opacities), ptr(homotrans), ptr(ap_level)
    surf.features, surf.offsets, surf.gridrange = ptr(features), ptr(offsets), ptr(gridrange)
    if cfg.kernel_type != 0:
        surf.shapes = ptr(shapes)
    _set_transmats(surf, transmat_precomp, homotrans, P)
    if "shs" in g:
        _set_shs(cfg, surf, shs, P)
    elif cfg.uses_rows:
        surf.colors_precomp = ptr(colors_precomp)
    gi = _lib.GradsIn(ptr(dL_dcolor), ptr(dL_dothers), ptr(radii))
    go = _lib.GradsOut(ptr(g["means3D"]), ptr(g["means2D"]), ptr(g["opacity"]), ptr(g["scales"]),
                       ptr(g["rotations"]), ptr(g["table"]), rows, ptr(g["gradsum"]),
                       ptr(g["shapes"]) if "shapes" in g else None,
                       ptr(g["colors_precomp"]) if "colors_precomp" in g else None,
                       ptr(g["shs"]) if "shs" in g else None,
                       ptr(g["transmat_precomp"]) if "transmat_precomp" in g else None)
    nbytes = (lib.ns_backward_scratch_bytes_deterministic(P, rows, int(cfg.level_dim)) if cfg.deterministic
              else lib.ns_backward_scratch_bytes(P))
    acc = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    check("ns_rasterize_backward",
          lib.ns_rasterize_backward(C.byref(settings), C.byref(surf), C.byref(gi), C.byref(go),
                                    scratch.geom.data_ptr(), scratch.geom.numel(), scratch.binning.data_ptr(),
                                    scratch.binning.numel(), scratch.image.data_ptr(), scratch.image.numel(),
                                    int(num_rendered), acc.data_ptr(), acc.numel(), _lib.stream_handle(dev)))
    if return_accumulators:
        g["accum"] = acc[: P * 80].view(torch.float32).reshape(P, 20)
    return g


def mark_visible(means3D, viewmatrix, projmatrix) -> torch.Tensor:
    lib = _lib.load()
    _require_cuda(means3D, viewmatrix, projmatrix)
    P = means3D.shape[0]
    present = torch.zeros((P,), dtype=torch.bool, device=means3D.device)
    check("ns_mark_visible", lib.ns_mark_visible(P, ptr(means3D), ptr(viewmatrix), ptr(projmatrix),
                                                 ptr(present), _lib.stream_handle(means3D.device)))
    return present


def pack_mlp(weights) -> torch.Tensor:
    """Packs fp16 [out,in] matrices back to back (the ns_mlp_forward layout)."""
    return torch.cat([w.reshape(-1) for w in weights]).to(torch.float16).contiguous()


def mlp_forward(feat_chw: torch.Tensor, packed_weights: torch.Tensor, alpha=None, bg=None,
                hidden: int = 64) -> torch.Tensor:
    """RGB [3, ...] = sigmoid(MLP(features)) * (alpha > 0) (+ (1-alpha) bg)."""
    lib = _lib.load()
    Cin = feat_chw.shape[0]
    npix = feat_chw[0].numel()
    _require_cuda(feat_chw, packed_weights, alpha)
    rgb = torch.empty((3,) + tuple(feat_chw.shape[1:]), dtype=torch.float32, device=feat_chw.device)
    bg_arr = None
    if bg is not None:
        b = [float(x) for x in (bg.tolist() if torch.is_tensor(bg) else bg)]
        bg_arr = (C.c_float * 3)(*b)
    check("ns_mlp_forward", lib.ns_mlp_forward(ptr(feat_chw), Cin, npix, ptr(packed_weights), hidden, 3,
                                               ptr(alpha), C.cast(bg_arr, C.c_void_p) if bg_arr else None,
                                               ptr(rgb), _lib.stream_handle(feat_chw.device)))
    return rgb


def mlp_backward(feat_chw: torch.Tensor, packed_weights: torch.Tensor, dL_drgb: torch.Tensor,
                 alpha=None, hidden: int = 64):
    """(dL/dfeat [C, ...], dL/dweights fp32 in the packed layout) of mlp_forward
    without the background term, from dL/drgb [3, ...]."""
    lib = _lib.load()
    Cin = feat_chw.shape[0]
    npix = feat_chw[0].numel()
    g = dL_drgb.float().contiguous()
    _require_cuda(feat_chw, packed_weights, alpha, g)
    dfeat = torch.empty_like(feat_chw, dtype=torch.float32)
    dW = torch.empty(packed_weights.numel(), dtype=torch.float32, device=feat_chw.device)
    check("ns_mlp_backward", lib.ns_mlp_backward(ptr(feat_chw), Cin, npix, ptr(packed_weights), hidden, 3,
                                                 ptr(alpha), ptr(g), ptr(dfeat), ptr(dW),
                                                 _lib.stream_handle(feat_chw.device)))
    return dfeat, dW


def normal_error(allmap: torch.Tensor, viewmatrix: torch.Tensor, rays_d: torch.Tensor,
                 ray_o: torch.Tensor) -> torch.Tensor:
    """Depth-normal consistency error [H, W] of the training loss (ns_normal_error):
    1 - <world rendered normal, depth_to_normal(expected depth) * alpha>."""
    lib = _lib.load()
    _require_cuda(allmap, viewmatrix, rays_d, ray_o)
    H, W = allmap.shape[1], allmap.shape[2]
    err = torch.empty((H, W), dtype=torch.float32, device=allmap.device)
    check("ns_normal_error", lib.ns_normal_error(ptr(allmap), ptr(viewmatrix), ptr(rays_d), ptr(ray_o), W, H,
                                                 ptr(err), _lib.stream_handle(allmap.device)))
    return err


def normal_error_backward(allmap: torch.Tensor, viewmatrix: torch.Tensor, rays_d: torch.Tensor,
                          ray_o: torch.Tensor, dL_derr: torch.Tensor) -> torch.Tensor:
    """d loss / d allmap (all channels; 5 and up zero) from d loss / d err. dL_derr is
    [H, W], or a broadcast view of one value (stride 0, as the gradient of a mean)."""
    lib = _lib.load()
    _require_cuda(allmap, viewmatrix, rays_d, ray_o)
    H, W = allmap.shape[1], allmap.shape[2]
    if dL_derr.numel() == 1 or all(st == 0 for st in dL_derr.stride()):
        g, stride = dL_derr[(0,) * dL_derr.dim()].reshape(1).float().contiguous(), 0
    else:
        g, stride = dL_derr.reshape(H, W).float().contiguous(), 1
    out = torch.empty_like(allmap)
    out[5:].zero_()
    scratch = torch.empty(lib.ns_normal_error_scratch_bytes(W, H), dtype=torch.uint8, device=allmap.device)
    check("ns_normal_error_backward",
          lib.ns_normal_error_backward(ptr(allmap), ptr(viewmatrix), ptr(rays_d), ptr(ray_o), W, H, ptr(g), stride,
                                       ptr(out), ptr(scratch), scratch.numel(), _lib.stream_handle(allmap.device)))
    return out


def rvq_decode(idx: torch.Tensor, codebooks: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    lib = _lib.load()
    _require_cuda(idx, codebooks)
    assert idx.dtype == torch.uint8 and codebooks.dtype == torch.float32
    n, K = idx.shape
    Kc, E, D = codebooks.shape
    assert Kc == K
    if out is None:
        out = torch.empty((n, D), dtype=torch.float32, device=idx.device)
    check("ns_rvq_decode", lib.ns_rvq_decode(ptr(idx), ptr(codebooks), ptr(out), n, K, E, D,
                                             _lib.stream_handle(idx.device)))
    return out


def radix_sort_pairs(keys: torch.Tensor, vals: torch.Tensor, end_bit: int = 64):
    """Stable sort of (int64 key viewed as u64, int32 value viewed as u32) pairs."""
    lib = _lib.load()
    _require_cuda(keys, vals)
    n = keys.numel()
    ko, vo = torch.empty_like(keys), torch.empty_like(vals)
    ka, va = torch.empty_like(keys), torch.empty_like(vals)
    temp = torch.empty(max(1, lib.ns_radix_sort_temp_bytes(n)), dtype=torch.uint8, device=keys.device)
    check("ns_radix_sort_pairs", lib.ns_radix_sort_pairs(ptr(keys), ptr(vals), ptr(ko), ptr(vo), ptr(ka),
                                                         ptr(va), n, end_bit, ptr(temp), temp.numel(),
                                                         _lib.stream_handle(keys.device)))
    return ko, vo
