"""The per-frame maps of the reference's render() (its render_pkg), from the
rasterizer's allmap, in one kernel (ns_allmap_decode).

Restates gaussian_renderer/__init__.py:763-797 (alpha, view-to-world normal,
median and expected depth with nan_to_num, surf_depth by depth_ratio,
surf_normal = depth_to_normal(surf_depth) * alpha) and the keys it returns
(:1035-1045). `render_maps_torch` is the same computation in plain torch, kept
as the fp32 reference the kernel is tested against.
"""
from __future__ import annotations

import torch

from . import _lib
from ._lib import check, ptr
from .train import _camera_rays, depth_to_normal

ALLMAP_DEPTH, ALLMAP_ALPHA, ALLMAP_NORMAL, ALLMAP_MEDIAN, ALLMAP_DIST, ALLMAP_COUNT = 0, 1, 2, 5, 6, 7


def render_maps(allmap: torch.Tensor, cam, depth_ratio: float = 0.0) -> dict:
    """render_pkg maps of a frame: rend_alpha, rend_normal, rend_dist, surf_depth,
    surf_normal, gaussian_num, depth_expected, depth_median ([C, H, W] each)."""
    lib = _lib.load()
    dev = allmap.device
    allmap = allmap.detach().float().contiguous()
    H, W = allmap.shape[1], allmap.shape[2]
    rays_d, rays_o = _camera_rays(cam, dev)
    vm = cam.world_view_transform.to(dev).float().contiguous()
    out = torch.empty((9, H, W), dtype=torch.float32, device=dev)
    check("ns_allmap_decode", lib.ns_allmap_decode(ptr(allmap), ptr(vm), ptr(rays_d.contiguous()),
                                                   ptr(rays_o.contiguous()), W, H, float(depth_ratio), ptr(out),
                                                   _lib.stream_handle(dev)))
    return {
        "rend_alpha": allmap[ALLMAP_ALPHA:ALLMAP_ALPHA + 1],
        "rend_normal": out[0:3],
        "rend_dist": allmap[ALLMAP_DIST:ALLMAP_DIST + 1],
        "surf_depth": out[5:6],
        "surf_normal": out[6:9],
        "gaussian_num": allmap[ALLMAP_COUNT:ALLMAP_COUNT + 1],
        "depth_expected": out[3:4],
        "depth_median": out[4:5],
    }


def render_maps_torch(allmap: torch.Tensor, cam, depth_ratio: float = 0.0) -> dict:
    """The same maps with the reference's torch expressions."""
    alpha = allmap[1:2]
    wv = cam.world_view_transform.to(allmap.device)
    rend_normal = (allmap[2:5].permute(1, 2, 0) @ wv[:3, :3].T).permute(2, 0, 1)
    median = torch.nan_to_num(allmap[5:6], 0, 0)
    expected = torch.nan_to_num(allmap[0:1] / alpha, 0, 0)
    surf_depth = expected * (1 - depth_ratio) + depth_ratio * median
    surf_normal = depth_to_normal(cam, surf_depth).permute(2, 0, 1) * alpha.detach()
    return {"rend_alpha": alpha, "rend_normal": rend_normal, "rend_dist": allmap[6:7], "surf_depth": surf_depth,
            "surf_normal": surf_normal, "gaussian_num": allmap[7:8], "depth_expected": expected,
            "depth_median": median}
