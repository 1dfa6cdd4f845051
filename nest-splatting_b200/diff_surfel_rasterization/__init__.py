"""Drop-in replacement of the reference's `diff_surfel_rasterization` module.

Same names, fields and call signatures as
submodules/diff-surfel-rasterization/diff_surfel_rasterization/__init__.py of
NilKel/nest-splatting (GaussianRasterizationSettings :277-293,
HashGridSettings :295-302, GaussianRasterizer :304-396, rasterize_gaussians
:21-66, _RasterizeGaussians :68-275, compute_relocation :398-414). The forward
and backward passes run the sm_100a kernels of libnest_b200.so through its
C-ABI; there is no CPU fallback. Built: render_mode 0 (baseline hash grid,
level_dim 2; level 0: per-surfel colours), the Gaussian splat kernel
(kernel_type 0) and the beta / flex / general kernels (kernel_type 1-3,
per-surfel `shapes`, whose gradient comes back in shapes' slot), forward and
backward; render modes 4 (cat), 6 (adaptive), 7 (adaptive_add), 12
(adaptive_cat) and 14 (adaptive_zero), forward (12-14 also with the inference
flag 256) and backward (training rules; mode 13, adaptive_cat_fast, forward
only as in the reference; the per-surfel rows' gradient, blend weight
included, comes back in colors_precomp's slot), the per-surfel features read
from colors_precomp and the level word hashgrid_settings.L = total << 16 |
active << 8 | hybrid as the reference's renderer encodes it
(gaussian_renderer/__init__.py:216-241, 334-447); the spherical-harmonic
hybrids 8 (hybrid_SH), 9 (hybrid_SH_post) and 10 (hybrid_SH_raw) with a
single 3-wide hash level and the level word decompose << 24 | SH degree << 16
| 1 << 8, and 11 (residual_hybrid: hash features in out_color, the rows' SH
colour in out_others channels 14-16, so out_others has 17 channels), forward
and backward (:570-686). The dual-grid modes 1-3 and 5 of the reference's
surface-potential renderer raise NotImplementedError instead of silently
rendering nothing as the reference does for shapes it was not compiled for.

Precomputed splat-to-pixel transforms (cov3D_precomp [P, 9], the reference's
transMat_precomp) replace scales and rotations, as the reference's renderer
passes them on its compute_cov3D_python path; homotrans is then required, and
their gradient comes back in cov3D_precomp's slot.

Backward (__init__.py:174-275 of the reference): the 21 gradients come back in
argument order; means2D's slot carries the densification statistic and
ap_level's slot dL_gradsum, homotrans gets None (its gradient is folded into
means, scales and rotations), sh gets zeros and colors_precomp zeros in mode 0
(which never reads them). Level 0 takes colors_precomp or, like the
reference's warm-up renders, SH coefficients (`shs`, evaluated at
raster_settings.sh_degree from raster_settings.campos); their gradient comes
back in sh's slot.

`features` may be fp32 (as the reference stores the table) or fp16 (read as
fp16 pairs by the kernels, half the L2 traffic).

Under `torch.use_deterministic_algorithms(True)` the backward reduces the
hash-table gradient in 64-bit fixed point, so it is bit-identical from run to
run (the per-surfel gradients keep float atomics, as in the reference).
"""
from __future__ import annotations

import math
import os
import sys
from typing import NamedTuple

import torch
import torch.nn as nn

_PKG_ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if _PKG_ROOT not in sys.path:
    sys.path.insert(0, _PKG_ROOT)

from nest_b200 import raster as _raster  # noqa: E402


def cpu_deep_copy_tuple(input_tuple):
    return tuple(item.cpu().clone() if isinstance(item, torch.Tensor) else item for item in input_tuple)


def rasterize_gaussians(means3D, means2D, sh, colors_precomp, opacities, scales, rotations,
                        cov3Ds_precomp, homotrans, ap_level, features, offsets, gridrange,
                        features_diffuse, offsets_diffuse, gridrange_diffuse, raster_settings,
                        hashgrid_settings, render_mode, shapes, kernel_type):
    return _RasterizeGaussians.apply(means3D, means2D, sh, colors_precomp, opacities, scales, rotations,
                                     cov3Ds_precomp, homotrans, ap_level, features, offsets, gridrange,
                                     features_diffuse, offsets_diffuse, gridrange_diffuse, raster_settings,
                                     hashgrid_settings, render_mode, shapes, kernel_type)


def _nonempty(t):
    return t if (t is not None and t.numel() > 0) else None


def _shape_dims(hashgrid_settings):
    sd = hashgrid_settings.shape_dims
    if sd is not None and torch.is_tensor(sd) and sd.numel() == 3:
        return [int(x) for x in sd.tolist()]
    return [0, 0, 3]


class _RasterizeGaussians(torch.autograd.Function):
    @staticmethod
    def forward(ctx, means3D, means2D, sh, colors_precomp, opacities, scales, rotations, cov3Ds_precomp,
                homotrans, ap_level, features, offsets, gridrange, features_diffuse, offsets_diffuse,
                gridrange_diffuse, raster_settings, hashgrid_settings, render_mode, shapes, kernel_type):
        mode = int(render_mode)
        base_mode = mode & 0xFF
        if base_mode not in (0, 4, 6, 7, 8, 9, 10, 11, 12, 13, 14) or (mode >> 8) > 1 or \
                ((mode >> 8) and base_mode not in (12, 13, 14)):
            raise NotImplementedError(f"render_mode {render_mode}: 0 (baseline hash grid; level 0: per-surfel "
                                      f"colours), 4 (cat), 6 (adaptive), 7 (adaptive_add), 8 (hybrid_SH), "
                                      f"9 (hybrid_SH_post), 10 (hybrid_SH_raw), 11 (residual_hybrid), "
                                      f"12 (adaptive_cat), 13 (adaptive_cat_fast), 14 (adaptive_zero) are built; "
                                      f"the dual-grid modes 1-3 and 5 of the surface-potential renderer are not")
        if int(kernel_type) not in (0, 1, 2, 3):
            raise NotImplementedError(f"kernel_type {kernel_type}: 0-3 are built")
        shp = _nonempty(shapes)
        if int(kernel_type) != 0:
            if shp is None or shp.numel() != means3D.shape[0]:
                raise RuntimeError(f"kernel_type {kernel_type} needs shapes with one value per surfel")
            shp = shp.detach().contiguous().float().reshape(-1)
        else:
            shp = None
        # Precomputed splat-to-pixel transforms (the reference's transMat_precomp,
        # passed as cov3D_precomp by its renderer's compute_cov3D_python path,
        # gaussian_renderer/__init__.py:64-76): [P, 9] columns Tu, Tv, Tw; the
        # hit point then needs homotrans.
        Ts = _nonempty(cov3Ds_precomp)
        if Ts is not None:
            Ts = Ts.detach().contiguous().float().reshape(-1, 9)
            if Ts.shape[0] != means3D.shape[0]:
                raise RuntimeError("cov3D_precomp must hold 9 values per surfel")
            if _nonempty(homotrans) is None:
                raise RuntimeError("precomputed transforms need homotrans (the surfels' plane frames)")
        if means3D.ndim != 2 or means3D.shape[1] != 3:
            raise RuntimeError("means3D must have dimensions (num_points, 3)")
        L = int(hashgrid_settings.L)
        hybrid = total = 0
        gauss = None
        shs_in = None
        if base_mode == 0 and L <= 0:
            # level 0 (forward.cu:1093-1096): the per-surfel colours are blended, either
            # colors_precomp or the SH colours preprocess evaluates (:414-423)
            gauss = _nonempty(colors_precomp)
            if gauss is not None:
                gauss = gauss.detach().contiguous().float()
            else:
                shs_in = _nonempty(sh)
                if shs_in is None:
                    raise RuntimeError("level 0 needs colors_precomp or SH coefficients")
                shs_in = shs_in.detach().contiguous().float().reshape(means3D.shape[0], -1, 3)
            L = 0
            if _nonempty(features) is None:  # the C-ABI wants a table; level 0 reads none
                features = torch.zeros((1, 2), dtype=torch.float32, device=means3D.device)
                offsets = torch.zeros(1, dtype=torch.int32, device=means3D.device)
                gridrange = torch.tensor([-1.0, 1.0], device=means3D.device)
        elif L <= 0 or _nonempty(features) is None:
            raise RuntimeError(f"render_mode {mode} needs hash-grid features and levels")
        elif base_mode == 6:
            # adaptive: the level word is the number of hash levels; rows of C channels
            gauss = _nonempty(colors_precomp)
            if gauss is None:
                raise RuntimeError("render_mode 6 needs colors_precomp (per-surfel features)")
            gauss = gauss.detach().contiguous().float()
        elif base_mode == 7:
            # adaptive_add: level word total << 16 | active hash levels << 8
            total, L = (L >> 16) & 0xFF, (L >> 8) & 0xFF
            gauss = _nonempty(colors_precomp)
            if gauss is None:
                raise RuntimeError("render_mode 7 needs colors_precomp (per-surfel features + weight)")
            gauss = gauss.detach().contiguous().float()
        elif base_mode in (8, 9, 10):
            # hybrid_SH / _post / _raw (gaussian_renderer/__init__.py:598-686): level word
            # decompose << 24 | SH degree << 16 | hash levels (1) << 8; one 3-wide level;
            # rows of 3 raw SH colours (48 SH coefficients for 9)
            hybrid, total, L = (L >> 24) & 0xFF, (L >> 16) & 0xFF, (L >> 8) & 0xFF
            gauss = _nonempty(colors_precomp)
            if gauss is None:
                raise RuntimeError(f"render_mode {mode} needs colors_precomp (per-surfel SH colours)")
            gauss = gauss.detach().contiguous().float()
            width = 48 if base_mode == 9 else 3
            if gauss.reshape(means3D.shape[0], -1).shape[1] != width:
                raise RuntimeError(f"render_mode {mode} needs colors_precomp rows of {width} values")
            if _nonempty(features) is not None and features.shape[-1] != 3:
                raise RuntimeError(f"render_mode {mode} reads a hash table of 3 values per row")
        elif base_mode == 11:
            # residual_hybrid (:570-596): level word total << 16 | hash levels << 8 | hybrid;
            # rows of 48 SH coefficients; hash features from channel 0
            total, L, hybrid = (L >> 16) & 0xFF, (L >> 8) & 0xFF, L & 0xFF
            gauss = _nonempty(colors_precomp)
            if gauss is None:
                raise RuntimeError("render_mode 11 needs colors_precomp (per-surfel SH coefficients)")
            gauss = gauss.detach().contiguous().float()
            if gauss.reshape(means3D.shape[0], -1).shape[1] != 48:
                raise RuntimeError("render_mode 11 needs colors_precomp rows of 48 SH coefficients")
        elif base_mode != 0:
            # The reference's level word: total << 16 | active hash levels << 8 | hybrid.
            total, active, hybrid = (L >> 16) & 0xFF, (L >> 8) & 0xFF, L & 0xFF
            if base_mode == 4:
                # Mode 4 queries every level of the (fine-levels-only) table: the last
                # offset that grows (forward.cu:1236-1242).
                offs = offsets.detach().to("cpu", torch.int64).reshape(-1).tolist()
                L = max([i for i in range(1, min(len(offs), 17)) if offs[i] > offs[i - 1]], default=0)
            else:
                L = active
            gauss = _nonempty(colors_precomp)
            if gauss is None:
                raise RuntimeError(f"render_mode {mode} needs colors_precomp (per-surfel features)")
            gauss = gauss.detach().contiguous().float()
        _, HS, OS = _shape_dims(hashgrid_settings)
        if base_mode == 0 and L == 0 and OS == 0:
            OS = gauss.shape[-1] if gauss is not None else 3
        if shs_in is not None:
            OS = 3
        if base_mode in (8, 10):
            OS = 3
        elif base_mode == 9:
            OS = 48  # the 48 coefficients the kernel's case 9 writes
        elif base_mode == 11:
            OS = HS if OS == 0 else OS  # dual buffers: the hash features' HS channels
        feats = features.contiguous()
        if feats.dtype not in (torch.float16, torch.float32):
            feats = feats.float()
        cfg = _raster.RasterConfig(
            image_height=int(raster_settings.image_height), image_width=int(raster_settings.image_width),
            tanfovx=float(raster_settings.tanfovx), tanfovy=float(raster_settings.tanfovy),
            viewmatrix=raster_settings.viewmatrix.contiguous().float(),
            projmatrix=raster_settings.projmatrix.contiguous().float(),
            scale_modifier=float(raster_settings.scale_modifier), beta=float(raster_settings.beta),
            if_contract=bool(raster_settings.if_contract),
            record_transmittance=bool(raster_settings.record_transmittance),
            max_intersections=int(raster_settings.max_intersections),
            prefiltered=bool(raster_settings.prefiltered), levels=L, S=float(hashgrid_settings.S),
            base_resolution=int(hashgrid_settings.H), align_corners=bool(hashgrid_settings.align_corners),
            interpolation=int(hashgrid_settings.interpolation), channels=int(OS),
            level_dim=int(feats.shape[1]), table_fp16=feats.dtype == torch.float16,
            kernel_type=int(kernel_type), deterministic=torch.are_deterministic_algorithms_enabled(),
            render_mode=mode, hybrid_levels=hybrid, total_levels=total,
            sh_degree=int(raster_settings.sh_degree) if shs_in is not None else 0,
            campos=raster_settings.campos.detach().contiguous().float() if shs_in is not None else None)
        ap = _nonempty(ap_level)
        sc, ro = _nonempty(scales), _nonempty(rotations)
        args = (means3D.detach().contiguous().float(), None if sc is None else sc.detach().contiguous().float(),
                None if ro is None else ro.detach().contiguous().float(),
                opacities.detach().contiguous().float().reshape(-1),
                None if _nonempty(homotrans) is None else homotrans.detach().contiguous().float().reshape(-1, 16),
                None if ap is None else ap.detach().contiguous().float().reshape(-1), feats.detach(),
                offsets.contiguous().to(torch.int32), gridrange.contiguous().float())
        num_rendered, color, others, radii, cover, trans, scratch = _raster.rasterize_forward(
            cfg, *args, shapes=shp, colors_precomp=gauss, shs=shs_in, transmat_precomp=Ts)
        ctx.cfg = cfg
        ctx.args = args
        ctx.radii = radii
        ctx.num_rendered = num_rendered
        ctx.scratch = scratch
        ctx.shapes = dict(opacities=opacities.shape, ap_level=ap_level.shape, features=features.dtype,
                          sh=sh.shape, colors_precomp=colors_precomp.shape,
                          shapes=None if shp is None else shapes.shape)
        ctx.shape_values = shp
        ctx.gauss = gauss
        ctx.shs = shs_in
        ctx.Ts = Ts
        ctx.cov_shape = cov3Ds_precomp.shape
        ctx.mark_non_differentiable(radii)
        return color, radii, others, trans, cover

    @staticmethod
    def backward(ctx, grad_out_color, grad_radii, grad_depth, grad_0, grad_1):
        if (ctx.cfg.render_mode >> 8) != 0 or (ctx.cfg.render_mode & 0xFF) == 13:
            raise NotImplementedError(f"backward of render_mode {ctx.cfg.render_mode}: the inference flag and "
                                      f"mode 13 have no backward (the reference's has none either)")
        dev = ctx.radii.device
        H, W = ctx.cfg.image_height, ctx.cfg.image_width
        if grad_out_color is None:
            grad_out_color = torch.zeros((ctx.cfg.channels, H, W), dtype=torch.float32, device=dev)
        if grad_depth is None:
            grad_depth = torch.zeros((_raster.OTHER_CHANNELS, H, W), dtype=torch.float32, device=dev)
        g = _raster.rasterize_backward(ctx.cfg, *ctx.args, ctx.radii, ctx.num_rendered, ctx.scratch,
                                       grad_out_color, grad_depth, shapes=ctx.shape_values,
                                       colors_precomp=ctx.gauss, shs=ctx.shs, transmat_precomp=ctx.Ts)
        ctx.scratch = None
        need = ctx.needs_input_grad
        sh = ctx.shapes

        def zeros_if(i, shape):
            return torch.zeros(shape, dtype=torch.float32, device=dev) if need[i] else None

        gradsum = g["gradsum"].reshape(sh["ap_level"]) if (need[9] and len(sh["ap_level"]) and
                                                          sh["ap_level"][0] == g["gradsum"].shape[0]) else None
        return (g["means3D"] if need[0] else None,
                g["means2D"] if need[1] else None,
                (g["shs"].reshape(sh["sh"]) if "shs" in g else zeros_if(2, sh["sh"])) if need[2] else None,
                (g["colors_precomp"].reshape(sh["colors_precomp"]) if "colors_precomp" in g
                 else zeros_if(3, sh["colors_precomp"])) if need[3] else None,
                g["opacity"].reshape(sh["opacities"]) if need[4] else None,
                g["scales"] if need[5] and ctx.Ts is None else None,
                g["rotations"] if need[6] and ctx.Ts is None else None,
                g["transmat_precomp"].reshape(ctx.cov_shape) if (need[7] and ctx.Ts is not None) else None,
                None,  # homotrans: folded into means / scales / rotations
                gradsum,
                g["table"].to(sh["features"]) if need[10] else None,
                None, None, None, None, None, None, None, None,
                g["shapes"].reshape(sh["shapes"]) if (need[19] and sh["shapes"] is not None) else None,
                None)


class GaussianRasterizationSettings(NamedTuple):
    image_height: int
    image_width: int
    tanfovx: float
    tanfovy: float
    bg: torch.Tensor
    scale_modifier: float
    viewmatrix: torch.Tensor
    projmatrix: torch.Tensor
    sh_degree: int
    campos: torch.Tensor
    prefiltered: bool
    debug: bool
    beta: float
    if_contract: bool
    record_transmittance: bool
    max_intersections: int = 0  # 0 means no limit


class HashGridSettings(NamedTuple):
    L: int
    S: float
    H: int
    align_corners: bool
    interpolation: int
    shape_dims: torch.Tensor  # [GS, HS, OS]


class GaussianRasterizer(nn.Module):
    def __init__(self, raster_settings, hashgrid_settings):
        super().__init__()
        self.raster_settings = raster_settings
        self.hashgrid_settings = hashgrid_settings

    def markVisible(self, positions):
        with torch.no_grad():
            rs = self.raster_settings
            return _raster.mark_visible(positions.contiguous().float(), rs.viewmatrix.contiguous().float(),
                                        rs.projmatrix.contiguous().float())

    def forward(self, means3D, means2D, opacities, shs=None, colors_precomp=None, scales=None, rotations=None,
                cov3D_precomp=None, homotrans=None, ap_level=None, features=None, offsets=None, gridrange=None,
                features_diffuse=None, offsets_diffuse=None, gridrange_diffuse=None, render_mode=0, shapes=None,
                kernel_type=0):
        if (shs is None and colors_precomp is None) or (shs is not None and colors_precomp is not None):
            raise Exception('Please provide excatly one of either SHs or precomputed colors!')
        if ((scales is None or rotations is None) and cov3D_precomp is None) or \
                ((scales is not None or rotations is not None) and cov3D_precomp is not None):
            raise Exception('Please provide exactly one of either scale/rotation pair or precomputed 3D covariance!')
        dev = means3D.device
        empty = lambda dtype=torch.float32: torch.empty(0, dtype=dtype, device=dev)  # noqa: E731
        shs = empty() if shs is None else shs
        colors_precomp = empty() if colors_precomp is None else colors_precomp
        scales = empty() if scales is None else scales
        rotations = empty() if rotations is None else rotations
        cov3D_precomp = empty() if cov3D_precomp is None else cov3D_precomp
        homotrans = empty() if homotrans is None else homotrans
        ap_level = empty() if ap_level is None else ap_level
        features = empty() if features is None else features
        offsets = empty(torch.int32) if offsets is None else offsets
        gridrange = empty() if gridrange is None else gridrange
        features_diffuse = empty() if features_diffuse is None else features_diffuse
        offsets_diffuse = empty(torch.int32) if offsets_diffuse is None else offsets_diffuse
        gridrange_diffuse = empty() if gridrange_diffuse is None else gridrange_diffuse
        shapes = empty() if shapes is None else shapes
        return rasterize_gaussians(means3D, means2D, shs, colors_precomp, opacities, scales, rotations,
                                   cov3D_precomp, homotrans, ap_level, features, offsets, gridrange,
                                   features_diffuse, offsets_diffuse, gridrange_diffuse, self.raster_settings,
                                   self.hashgrid_settings, render_mode, shapes, kernel_type)


def compute_relocation(opacity_old, scale_old, N, binoms, n_max):
    """3DGS-MCMC relocation (cuda_rasterizer/utils.cu:4-32), a torch restatement.

    Outside the render hot path; kept so that callers of the reference module
    find the same function.
    """
    N = N.int()
    new_opacity = 1.0 - torch.pow(1.0 - opacity_old, 1.0 / N.float())
    denom = torch.zeros_like(opacity_old)
    for i in range(1, int(n_max) + 1):
        active = (N >= i).float()
        for k in range(i):
            coeff = binoms[i - 1, k]
            term = ((-1.0) ** k / math.sqrt(k + 1)) * torch.pow(new_opacity, k + 1)
            denom = denom + active * coeff * term
    coeff = opacity_old / denom
    new_scale = coeff.reshape(-1, 1) * scale_old
    return new_opacity, new_scale
