"""GPU parity of level 0 with SH coefficients (the reference's warm-up renders:
render mode 0 without a hash grid, colours from computeColorFromSH in the
preprocess, forward.cu:21-74, 414-423; backward.cu:21-140, 2266-2267) against
the oracle (oracle.sh_color, pinned to the reference's utils/sh_utils.py
eval_sh in test_golden.py, and its backward, pinned to float64 autograd in
test_oracle_backward.py), through the drop-in module and the C-ABI."""
import numpy as np
import pytest
import torch

import diff_surfel_rasterization as dsr
from helpers import api_inputs, compare, small_scene
from nest_b200 import raster
from oracle import oracle

pytestmark = pytest.mark.gpu


def sh_scene(seed, M=16):
    sc = small_scene(n=1500, seed=seed)
    inp = api_inputs(sc)
    g = torch.Generator().manual_seed(seed)
    shs = (torch.randn(sc.P, M, 3, generator=g) * 0.5).contiguous()
    return sc, inp, shs


def oracle_colours(sc, inp, shs, deg):
    cam = sc.camera
    return oracle.sh_color(inp["means3D"].numpy(), cam.camera_center.numpy(), shs.numpy(), deg)


@pytest.mark.parametrize("deg", [0, 1, 3])
def test_level0_sh_forward_matches_oracle(deg):
    sc, inp, shs = sh_scene(100 + deg)
    cam = sc.camera
    dev = "cuda"
    rgb = oracle_colours(sc, inp, shs, deg)
    dummy = np.zeros((1, 2), np.float32)
    out, _, _ = oracle.forward(inp["means3D"].numpy(), inp["scales"].numpy(), inp["rotations"].numpy(),
                               inp["opacities"].numpy(), inp["homotrans"].numpy(), inp["ap_level"].numpy(),
                               dummy, np.zeros(1, np.int32), np.array([-1.0, 1.0], np.float32),
                               cam.world_view_transform.numpy(), cam.full_proj_transform.numpy(), cam.width,
                               cam.height, 3, 2, 0, 0.0, 16, render_mode=0, gauss=rgb)
    rs = dsr.GaussianRasterizationSettings(
        image_height=cam.height, image_width=cam.width, tanfovx=cam.tanfovx, tanfovy=cam.tanfovy,
        bg=torch.zeros(3, device=dev), scale_modifier=1.0, viewmatrix=cam.world_view_transform.to(dev),
        projmatrix=cam.full_proj_transform.to(dev), sh_degree=deg, campos=cam.camera_center.to(dev),
        prefiltered=False, debug=False, beta=0.0, if_contract=False, record_transmittance=False,
        max_intersections=0)
    hs = dsr.HashGridSettings(L=0, S=0.0, H=16, align_corners=False, interpolation=0,
                              shape_dims=torch.tensor([0, 0, 3], dtype=torch.int32, device=dev))
    r = dsr.GaussianRasterizer(rs, hs)
    P = sc.P
    with torch.no_grad():
        color, _, allmap, _, _ = r(
            means3D=inp["means3D"].to(dev), means2D=torch.zeros(P, 3, device=dev), shs=shs.to(dev),
            colors_precomp=None, opacities=inp["opacities"].to(dev), scales=inp["scales"].to(dev),
            rotations=inp["rotations"].to(dev), homotrans=inp["homotrans"].to(dev),
            ap_level=inp["ap_level"].to(dev), render_mode=0)
    torch.cuda.synchronize()
    color, allmap = color.cpu().numpy(), allmap.cpu().numpy()
    assert color.shape[0] == 3 and np.abs(out["out_color"]).max() > 0.1
    compare(out, color, allmap)


def gpu_and_oracle_grads(sc, inp, shs, deg, gc, go):
    from test_gpu_backward import GRAD_KEYS
    cam = sc.camera
    dev = "cuda"
    cfg = raster.RasterConfig(
        image_height=cam.height, image_width=cam.width, tanfovx=cam.tanfovx, tanfovy=cam.tanfovy,
        viewmatrix=cam.world_view_transform.cuda().contiguous(),
        projmatrix=cam.full_proj_transform.cuda().contiguous(), levels=0, S=0.0, base_resolution=16, channels=3,
        level_dim=2, table_fp16=False, sh_degree=deg, campos=cam.camera_center.to(dev).float().contiguous())
    table = torch.zeros((1, 2), device=dev)
    args = (inp["means3D"].cuda().contiguous(), inp["scales"].cuda().contiguous(),
            inp["rotations"].cuda().contiguous(), inp["opacities"].cuda().reshape(-1).contiguous(),
            inp["homotrans"].cuda().reshape(-1, 16).contiguous(), inp["ap_level"].cuda().reshape(-1).contiguous(),
            table, torch.zeros(1, dtype=torch.int32, device=dev), torch.tensor([-1.0, 1.0], device=dev))
    shs_d = shs.cuda().contiguous()
    n, color, others, radii, _, _, scratch = raster.rasterize_forward(cfg, *args, shs=shs_d)
    got = raster.rasterize_backward(cfg, *args, radii, n, scratch, gc.cuda(), go.cuda(), shs=shs_d)
    torch.cuda.synchronize()
    got = {k: v.cpu().numpy() for k, v in got.items()}
    vm, pm = cam.world_view_transform.numpy(), cam.full_proj_transform.numpy()
    W, H = cam.width, cam.height
    rgb = oracle_colours(sc, inp, shs, deg)
    pre = oracle.preprocess(inp["means3D"].numpy(), inp["scales"].numpy(), inp["rotations"].numpy(),
                            inp["opacities"].numpy(), vm, pm, W, H)
    _, vals, ranges = oracle.bin_surfels(pre, W, H)
    common = (inp["homotrans"].numpy(), inp["ap_level"].numpy(), np.zeros((1, 2), np.float32),
              np.zeros(1, np.int32), np.array([-1.0, 1.0], np.float32), W, H, 3, 2, 0, 0.0, 16)
    fwd = oracle.render(pre, vals, ranges, *common, render_mode=0, gauss=rgb)
    refs = []
    for f64 in (False, True):
        gr = oracle.render_backward(pre, vals, ranges, fwd, *common, gc.numpy(), go.numpy(), f64=f64, render_mode=0,
                                    gauss=rgb)
        pg = oracle.preprocess_backward(inp["means3D"].numpy(), inp["scales"].numpy(), inp["rotations"].numpy(),
                                        pre, gr, vm, pm, W, H, cam.tanfovx, cam.tanfovy, f64=f64)
        dsh, dmean = oracle.sh_color_backward(inp["means3D"].numpy(), cam.camera_center.numpy(), shs.numpy(), deg,
                                              pre["radii"], gr["dL_dcolors"], f64=f64)
        pg = dict(pg)
        pg["dL_dmeans3D"] = pg["dL_dmeans3D"] + dmean
        gr = dict(gr)
        gr["dL_dshs"] = dsh
        refs.append(dict(g=gr, pg=pg))
    np.testing.assert_array_equal(radii.cpu().numpy(), pre["radii"])
    keys = {k: v for k, v in GRAD_KEYS.items() if k not in ("table", "gradsum")}
    keys["shs"] = ("g", "dL_dshs")
    return got, refs[0], refs[1], keys


@pytest.mark.parametrize("deg", [0, 2, 3])
def test_level0_sh_backward_matches_oracle(deg):
    """Every gradient, dL/dshs and the colour's part of dL/dmeans included,
    against the oracle's level-0 backward followed by its SH backward."""
    from test_gpu_backward import check_all, upstream
    sc, inp, shs = sh_scene(110 + deg)
    g = torch.Generator().manual_seed(deg)
    gc = torch.randn(3, sc.camera.height, sc.camera.width, generator=g)
    _, go = upstream(sc, seed=5)
    got, ref, exact, keys = gpu_and_oracle_grads(sc, inp, shs, deg, gc, go)
    assert not got["gradsum"].any()  # level 0 adds nothing to the densification sum
    check_all(got, ref, exact, keys=keys)


def test_level0_sh_dropin_gradient_in_sh_slot():
    """The drop-in Function returns dL/dshs in sh's slot and the SH colour's
    part of the mean gradient in means3D's."""
    from test_gpu_backward import upstream
    deg = 3
    sc, inp, shs = sh_scene(120)
    cam = sc.camera
    dev = "cuda"
    g = torch.Generator().manual_seed(7)
    gc = torch.randn(3, cam.height, cam.width, generator=g)
    _, go = upstream(sc, seed=5)
    _, ref, _, _ = gpu_and_oracle_grads(sc, inp, shs, deg, gc, go)
    rs = dsr.GaussianRasterizationSettings(
        image_height=cam.height, image_width=cam.width, tanfovx=cam.tanfovx, tanfovy=cam.tanfovy,
        bg=torch.zeros(3, device=dev), scale_modifier=1.0, viewmatrix=cam.world_view_transform.to(dev),
        projmatrix=cam.full_proj_transform.to(dev), sh_degree=deg, campos=cam.camera_center.to(dev),
        prefiltered=False, debug=False, beta=0.0, if_contract=False, record_transmittance=False,
        max_intersections=0)
    hs = dsr.HashGridSettings(L=0, S=0.0, H=16, align_corners=False, interpolation=0,
                              shape_dims=torch.tensor([0, 0, 3], dtype=torch.int32, device=dev))
    r = dsr.GaussianRasterizer(rs, hs)
    P = sc.P
    sh_leaf = shs.to(dev).clone().requires_grad_(True)
    means = inp["means3D"].to(dev).clone().requires_grad_(True)
    color, _, allmap, _, _ = r(
        means3D=means, means2D=torch.zeros(P, 3, device=dev), shs=sh_leaf, colors_precomp=None,
        opacities=inp["opacities"].to(dev), scales=inp["scales"].to(dev), rotations=inp["rotations"].to(dev),
        homotrans=inp["homotrans"].to(dev), ap_level=inp["ap_level"].to(dev), render_mode=0)
    loss = (color * gc.to(dev)).sum() + (allmap * go.to(dev)).sum()
    loss.backward()
    got_sh = sh_leaf.grad.cpu().numpy()
    want_sh = ref["g"]["dL_dshs"]
    assert got_sh.shape == want_sh.shape
    assert np.linalg.norm(got_sh - want_sh) / np.linalg.norm(want_sh) < 1e-3
    got_m = means.grad.cpu().numpy()
    want_m = ref["pg"]["dL_dmeans3D"]
    assert np.linalg.norm(got_m - want_m) / np.linalg.norm(want_m) < 1e-2
