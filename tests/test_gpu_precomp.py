"""GPU parity of precomputed splat-to-pixel transforms (the reference's
transMat_precomp, passed as cov3D_precomp by its renderer's
compute_cov3D_python path, gaussian_renderer/__init__.py:64-76;
forward.cu:366-380, backward.cu:2082-2088, 2128-2158) against the oracle,
whose restatement is pinned to float64 autograd in test_oracle_backward.py."""
import numpy as np
import pytest
import torch

import diff_surfel_rasterization as dsr
from helpers import api_inputs, compare, small_scene
from nest_b200 import raster
from oracle import oracle

pytestmark = pytest.mark.gpu


def precomp_case(seed):
    """A small scene whose transforms are the oracle's own, each entry scaled by
    1 + 1e-2 N(0, 1) so they are not those of any scale / rotation pair."""
    sc = small_scene(n=1500, seed=seed)
    inp = api_inputs(sc)
    cam = sc.camera
    pre = oracle.preprocess(inp["means3D"].numpy(), inp["scales"].numpy(), inp["rotations"].numpy(),
                            inp["opacities"].numpy(), cam.world_view_transform.numpy(),
                            cam.full_proj_transform.numpy(), cam.width, cam.height)
    g = torch.Generator().manual_seed(seed)
    Ts = torch.from_numpy(pre["transMat"]) * (1 + 1e-2 * torch.randn(pre["transMat"].shape, generator=g))
    return sc, inp, Ts.float().contiguous()


def oracle_forward(sc, inp, Ts):
    cam = sc.camera
    g = sc.grid
    out, pre, _ = oracle.forward(inp["means3D"].numpy(), None, None, inp["opacities"].numpy(),
                                 inp["homotrans"].numpy(), inp["ap_level"].numpy(), g.table.float().numpy(),
                                 g.offsets.numpy(), g.gridrange.numpy(), cam.world_view_transform.numpy(),
                                 cam.full_proj_transform.numpy(), cam.width, cam.height, g.channels, g.level_dim,
                                 g.levels, g.S, g.base_resolution, transmat_precomp=Ts.numpy())
    return out, pre


def test_precomputed_transforms_forward_match_oracle():
    sc, inp, Ts = precomp_case(130)
    cam, g = sc.camera, sc.grid
    dev = "cuda"
    out, pre = oracle_forward(sc, inp, Ts)
    assert (pre["radii"] > 0).sum() > 100
    rs = dsr.GaussianRasterizationSettings(
        image_height=cam.height, image_width=cam.width, tanfovx=cam.tanfovx, tanfovy=cam.tanfovy,
        bg=torch.zeros(3, device=dev), scale_modifier=1.0, viewmatrix=cam.world_view_transform.to(dev),
        projmatrix=cam.full_proj_transform.to(dev), sh_degree=0, campos=cam.camera_center.to(dev),
        prefiltered=False, debug=False, beta=0.0, if_contract=False, record_transmittance=False,
        max_intersections=0)
    hs = dsr.HashGridSettings(L=g.levels, S=g.S, H=g.base_resolution, align_corners=False, interpolation=0,
                              shape_dims=torch.tensor([0, g.channels, g.channels], dtype=torch.int32, device=dev))
    r = dsr.GaussianRasterizer(rs, hs)
    P = sc.P
    with torch.no_grad():
        color, radii, allmap, _, _ = r(
            means3D=inp["means3D"].to(dev), means2D=torch.zeros(P, 3, device=dev), shs=None,
            colors_precomp=torch.zeros(P, 3, device=dev), opacities=inp["opacities"].to(dev),
            cov3D_precomp=Ts.to(dev), homotrans=inp["homotrans"].to(dev), ap_level=inp["ap_level"].to(dev),
            features=g.table.to(dev), offsets=g.offsets.to(dev), gridrange=g.gridrange.to(dev), render_mode=0)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(radii.cpu().numpy(), pre["radii"])
    allmap = allmap.cpu().numpy()
    assert not out["out_others"][2:4].any() and out["out_others"][4].min() < -0.5  # the view axis, facing the camera
    compare(out, color.cpu().numpy(), allmap)


def test_precomputed_transforms_backward_match_oracle():
    """The transforms' gradient (render pass plus the centre's term), opacity,
    table, densification sum and statistic against the oracle; means, scales
    and rotations get zeros."""
    from test_gpu_backward import check_all, upstream
    sc, inp, Ts = precomp_case(131)
    cam, g = sc.camera, sc.grid
    gc, go = upstream(sc, seed=6)
    cfg = raster.RasterConfig(
        image_height=cam.height, image_width=cam.width, tanfovx=cam.tanfovx, tanfovy=cam.tanfovy,
        viewmatrix=cam.world_view_transform.cuda().contiguous(),
        projmatrix=cam.full_proj_transform.cuda().contiguous(), levels=g.levels, S=g.S,
        base_resolution=g.base_resolution, channels=g.channels, level_dim=g.level_dim,
        table_fp16=g.table.dtype == torch.float16)
    args = (inp["means3D"].cuda().contiguous(), None, None, inp["opacities"].cuda().reshape(-1).contiguous(),
            inp["homotrans"].cuda().reshape(-1, 16).contiguous(), inp["ap_level"].cuda().reshape(-1).contiguous(),
            g.table.cuda().contiguous(), g.offsets.cuda().contiguous(), g.gridrange.cuda().contiguous())
    Td = Ts.cuda().contiguous()
    n, _, _, radii, _, _, scratch = raster.rasterize_forward(cfg, *args, transmat_precomp=Td)
    got = raster.rasterize_backward(cfg, *args, radii, n, scratch, gc.cuda(), go.cuda(), transmat_precomp=Td)
    torch.cuda.synchronize()
    got = {k: v.cpu().numpy() for k, v in got.items()}
    assert not got["means3D"].any() and not got["scales"].any() and not got["rotations"].any()
    W, H = cam.width, cam.height
    vm, pm = cam.world_view_transform.numpy(), cam.full_proj_transform.numpy()
    pre = oracle.preprocess(inp["means3D"].numpy(), None, None, inp["opacities"].numpy(), vm, pm, W, H,
                            transmat_precomp=Ts.numpy())
    np.testing.assert_array_equal(radii.cpu().numpy(), pre["radii"])
    _, vals, ranges = oracle.bin_surfels(pre, W, H)
    common = (inp["homotrans"].numpy(), inp["ap_level"].numpy(), g.table.float().numpy(), g.offsets.numpy(),
              g.gridrange.numpy(), W, H, g.channels, g.level_dim, g.levels, g.S, g.base_resolution)
    fwd = oracle.render(pre, vals, ranges, *common)
    refs = []
    for f64 in (False, True):
        gr = oracle.render_backward(pre, vals, ranges, fwd, *common, gc.numpy(), go.numpy(), f64=f64)
        pg = oracle.preprocess_backward(None, None, None, pre, gr, vm, pm, W, H, cam.tanfovx, cam.tanfovy,
                                        f64=f64, precomp=True)
        refs.append(dict(g=gr, pg=pg))
    keys = {"transmat_precomp": ("pg", "dL_dtransMat"), "opacity": ("g", "dL_dopacity"),
            "table": ("g", "dL_dtable"), "gradsum": ("g", "dL_gradsum"), "means2D": ("pg", "dL_dmean2D")}
    check_all(got, refs[0], refs[1], keys=keys)


def test_precomputed_transforms_dropin_gradient_in_cov3d_slot():
    """The drop-in returns the transforms' gradient in cov3D_precomp's slot."""
    from test_gpu_backward import upstream
    sc, inp, Ts = precomp_case(132)
    cam, g = sc.camera, sc.grid
    dev = "cuda"
    gc, go = upstream(sc, seed=7)
    rs = dsr.GaussianRasterizationSettings(
        image_height=cam.height, image_width=cam.width, tanfovx=cam.tanfovx, tanfovy=cam.tanfovy,
        bg=torch.zeros(3, device=dev), scale_modifier=1.0, viewmatrix=cam.world_view_transform.to(dev),
        projmatrix=cam.full_proj_transform.to(dev), sh_degree=0, campos=cam.camera_center.to(dev),
        prefiltered=False, debug=False, beta=0.0, if_contract=False, record_transmittance=False,
        max_intersections=0)
    hs = dsr.HashGridSettings(L=g.levels, S=g.S, H=g.base_resolution, align_corners=False, interpolation=0,
                              shape_dims=torch.tensor([0, g.channels, g.channels], dtype=torch.int32, device=dev))
    r = dsr.GaussianRasterizer(rs, hs)
    P = sc.P
    T_leaf = Ts.to(dev).clone().requires_grad_(True)
    color, _, allmap, _, _ = r(
        means3D=inp["means3D"].to(dev), means2D=torch.zeros(P, 3, device=dev), shs=None,
        colors_precomp=torch.zeros(P, 3, device=dev), opacities=inp["opacities"].to(dev), cov3D_precomp=T_leaf,
        homotrans=inp["homotrans"].to(dev), ap_level=inp["ap_level"].to(dev), features=g.table.to(dev),
        offsets=g.offsets.to(dev), gridrange=g.gridrange.to(dev), render_mode=0)
    ((color * gc.to(dev)).sum() + (allmap * go.to(dev)).sum()).backward()
    got = T_leaf.grad
    assert got is not None and got.shape == Ts.shape and torch.isfinite(got).all()
    assert float(got.abs().max()) > 0
    # the same gradient through the C-ABI path directly
    cfg = raster.RasterConfig(
        image_height=cam.height, image_width=cam.width, tanfovx=cam.tanfovx, tanfovy=cam.tanfovy,
        viewmatrix=cam.world_view_transform.cuda().contiguous(),
        projmatrix=cam.full_proj_transform.cuda().contiguous(), levels=g.levels, S=g.S,
        base_resolution=g.base_resolution, channels=g.channels, level_dim=g.level_dim,
        table_fp16=g.table.dtype == torch.float16)
    args = (inp["means3D"].cuda().contiguous(), None, None, inp["opacities"].cuda().reshape(-1).contiguous(),
            inp["homotrans"].cuda().reshape(-1, 16).contiguous(), inp["ap_level"].cuda().reshape(-1).contiguous(),
            g.table.cuda().contiguous(), g.offsets.cuda().contiguous(), g.gridrange.cuda().contiguous())
    n, _, _, radii, _, _, scratch = raster.rasterize_forward(cfg, *args, transmat_precomp=Ts.cuda().contiguous())
    want = raster.rasterize_backward(cfg, *args, radii, n, scratch, gc.cuda(), go.cuda(),
                                     transmat_precomp=Ts.cuda().contiguous())["transmat_precomp"]
    assert float((got - want).norm() / want.norm()) < 1e-3
