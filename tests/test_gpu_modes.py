"""GPU parity of the render modes that combine per-surfel features with the hash
grid (forward.cu:1218-1282 mode 4 cat, :1283-1325 mode 6 adaptive, :1326-1377
mode 7 adaptive_add, :1593-1700 mode 12 adaptive_cat, :1701-1790 mode 14
adaptive_zero; the inference flag 256 of 12 and 14) and of level 0
(:1093-1096, per-surfel colours without a hash grid) through
the drop-in module, against the oracle's restatement (oracle/nest_oracle.cpp
mode_feature). The level word and the feature rows are built as the
reference's renderer builds them (gaussian_renderer/__init__.py:216-241,
334-447): hashgrid_settings.L = total << 16 | active << 8 | hybrid,
colors_precomp = per-surfel features (+ the blend weight for 12 / 14), offsets
padded to 17 entries for mode 4."""
import numpy as np
import pytest
import torch

import diff_surfel_rasterization as dsr
from helpers import api_inputs, small_scene
from nest_b200 import synth
from oracle import oracle
from test_gpu_raster import compare

pytestmark = pytest.mark.gpu


def mode_case(mode, total, hybrid, active, seed, weights="uniform"):
    sc = small_scene(n=1500, seed=seed)
    inp = api_inputs(sc)
    g = torch.Generator().manual_seed(seed)
    LD = 2
    grid = synth.hash_grid(g, levels=max(active, 1), log2_T=13, lo=-1.0, hi=1.0, base_resolution=64,
                           per_level_scale=1.5)
    P = sc.P
    base = mode & 0xFF
    if base == 4:
        gauss = torch.rand(P, hybrid * LD, generator=g) * 2 - 1
    elif base in (0, 6):  # level 0 / adaptive: rows of C = total LD channels
        gauss = torch.rand(P, total * LD, generator=g) * 2 - 1
    else:
        width = total * LD if base in (7, 12, 13) else hybrid * LD
        feats = torch.rand(P, width, generator=g) * 2 - 1
        if weights == "uniform":
            wgt = torch.rand(P, 1, generator=g)
        else:  # thresholds of the inference rules and exact zeros / ones
            wgt = torch.tensor([0.0, 1e-7, 0.05, 0.1, 0.5, 0.89, 0.9, 0.95, 1.0])[
                torch.randint(0, 9, (P, 1), generator=g)]
        gauss = torch.cat([feats, wgt], 1)
    return sc, inp, grid, gauss.float().contiguous()


def level_word(mode, total, hybrid, active):
    """hashgrid_settings.L as the reference's renderer sets it: the level count
    for mode 6 and for mode 0 (0: per-surfel colours), total << 16 | active << 8
    for mode 7, and total << 16 | active << 8 | hybrid for 4 and 12-14."""
    base = mode & 0xFF
    if base in (0, 6):
        return active
    if base == 7:
        return (total << 16) | (active << 8)
    return (total << 16) | (active << 8) | hybrid


def run_mode(sc, inp, grid, gauss, mode, total, hybrid, active):
    cam = sc.camera
    dev = "cuda"
    base = mode & 0xFF
    C = total * 2
    hash_levels = grid.levels if base == 4 else active
    offsets = grid.offsets
    if base == 4 and offsets.numel() < 17:
        offsets = torch.cat([offsets, torch.zeros(17 - offsets.numel(), dtype=offsets.dtype)])
    rs = dsr.GaussianRasterizationSettings(
        image_height=cam.height, image_width=cam.width, tanfovx=cam.tanfovx, tanfovy=cam.tanfovy,
        bg=torch.zeros(3, device=dev), scale_modifier=1.0, viewmatrix=cam.world_view_transform.to(dev),
        projmatrix=cam.full_proj_transform.to(dev), sh_degree=0, campos=cam.camera_center.to(dev),
        prefiltered=False, debug=False, beta=0.0, if_contract=False, record_transmittance=False,
        max_intersections=0)
    hs = dsr.HashGridSettings(L=level_word(mode, total, hybrid, active), S=grid.S, H=grid.base_resolution,
                              align_corners=False, interpolation=0,
                              shape_dims=torch.tensor([hybrid * 2, active * 2, C], dtype=torch.int32, device=dev))
    r = dsr.GaussianRasterizer(rs, hs)
    P = sc.P
    with torch.no_grad():
        color, radii, allmap, _, _ = r(
            means3D=inp["means3D"].to(dev), means2D=torch.zeros(P, 3, device=dev), shs=None,
            colors_precomp=gauss.to(dev), opacities=inp["opacities"].to(dev), scales=inp["scales"].to(dev),
            rotations=inp["rotations"].to(dev), homotrans=inp["homotrans"].to(dev),
            ap_level=inp["ap_level"].to(dev), features=grid.table.to(dev), offsets=offsets.to(dev),
            gridrange=grid.gridrange.to(dev), render_mode=mode)
    torch.cuda.synchronize()
    out, pre, n = oracle.forward(inp["means3D"].numpy(), inp["scales"].numpy(), inp["rotations"].numpy(),
                                 inp["opacities"].numpy(), inp["homotrans"].numpy(), inp["ap_level"].numpy(),
                                 grid.table.float().numpy(), grid.offsets.numpy(), grid.gridrange.numpy(),
                                 cam.world_view_transform.numpy(), cam.full_proj_transform.numpy(), cam.width,
                                 cam.height, C, 2, hash_levels, grid.S, grid.base_resolution, render_mode=mode,
                                 hybrid_levels=hybrid, total_levels=total, gauss=gauss.numpy())
    return out, color.cpu().numpy(), allmap.cpu().numpy()


@pytest.mark.parametrize("mode,total,hybrid,active,weights", [
    (4, 16, 6, 10, "uniform"),
    (4, 12, 4, 8, "uniform"),
    (12, 16, 6, 10, "uniform"),
    (12, 16, 6, 10, "thresholds"),
    (12 | 256, 16, 6, 10, "thresholds"),
    (12, 14, 5, 7, "uniform"),
    (14, 16, 6, 10, "thresholds"),
    (14 | 256, 16, 6, 10, "thresholds"),
    (14, 16, 16, 0, "uniform"),
    (13, 16, 6, 10, "uniform"),
    (13 | 256, 16, 6, 10, "thresholds"),
    (6, 16, 0, 10, "uniform"),
    (6, 12, 0, 12, "uniform"),
    (7, 16, 0, 10, "uniform"),
    (7, 16, 0, 10, "thresholds"),
    (7, 12, 0, 0, "uniform"),
    (0, 16, 0, 0, "uniform"),
])
def test_render_modes_match_oracle(mode, total, hybrid, active, weights):
    sc, inp, grid, gauss = mode_case(mode, total, hybrid, active, seed=50 + (mode & 0xFF), weights=weights)
    out, color, allmap = run_mode(sc, inp, grid, gauss, mode, total, hybrid, active)
    assert allmap[7].sum() > 100
    assert np.abs(out["out_color"]).max() > 0.1
    compare(out, color, allmap)


def test_render_mode_4_channels_split():
    """Mode 4: the first hybrid * LD channels are the blended per-surfel features
    alone (an all-zero table leaves them unchanged and zeroes the hash channels)."""
    sc, inp, grid, gauss = mode_case(4, 16, 6, 10, seed=61)
    grid.table = torch.zeros_like(grid.table)
    out, color, allmap = run_mode(sc, inp, grid, gauss, 4, 16, 6, 10)
    assert np.abs(color[:12]).max() > 0.1
    assert not color[12:].any()
    compare(out, color, allmap)


def mode_grads(sc, inp, grid, gauss, mode, total, hybrid, active, gc, go):
    """GPU gradients of modes 4 / 12 / 14 through raster.rasterize_forward /
    rasterize_backward, and the oracle's (float32 and float64) on the same lists."""
    from nest_b200 import raster
    from test_gpu_backward import GRAD_KEYS
    cam = sc.camera
    base = mode & 0xFF
    hash_levels = grid.levels if base == 4 else active
    C = total * 2
    cfg = raster.RasterConfig(
        image_height=cam.height, image_width=cam.width, tanfovx=cam.tanfovx, tanfovy=cam.tanfovy,
        viewmatrix=cam.world_view_transform.cuda().contiguous(),
        projmatrix=cam.full_proj_transform.cuda().contiguous(), levels=hash_levels, S=grid.S,
        base_resolution=grid.base_resolution, channels=C, level_dim=2, table_fp16=True, render_mode=mode,
        hybrid_levels=hybrid, total_levels=total)
    args = (inp["means3D"].cuda().contiguous(), inp["scales"].cuda().contiguous(),
            inp["rotations"].cuda().contiguous(), inp["opacities"].cuda().reshape(-1).contiguous(),
            inp["homotrans"].cuda().reshape(-1, 16).contiguous(), inp["ap_level"].cuda().reshape(-1).contiguous(),
            grid.table.cuda().contiguous(), grid.offsets.cuda().contiguous(), grid.gridrange.cuda().contiguous())
    gcol = gauss.cuda().contiguous()
    n, color, others, radii, _, _, scratch = raster.rasterize_forward(cfg, *args, colors_precomp=gcol)
    got = raster.rasterize_backward(cfg, *args, radii, n, scratch, gc.cuda(), go.cuda(), colors_precomp=gcol)
    torch.cuda.synchronize()
    got = {k: v.cpu().numpy() for k, v in got.items()}
    vm, pm = cam.world_view_transform.numpy(), cam.full_proj_transform.numpy()
    W, H = cam.width, cam.height
    pre = oracle.preprocess(inp["means3D"].numpy(), inp["scales"].numpy(), inp["rotations"].numpy(),
                            inp["opacities"].numpy(), vm, pm, W, H)
    _, vals, ranges = oracle.bin_surfels(pre, W, H)
    common = (inp["homotrans"].numpy(), inp["ap_level"].numpy(), grid.table.float().numpy(), grid.offsets.numpy(),
              grid.gridrange.numpy(), W, H, C, 2, hash_levels, grid.S, grid.base_resolution)
    mkw = dict(render_mode=mode, hybrid_levels=hybrid, total_levels=total, gauss=gauss.numpy())
    fwd = oracle.render(pre, vals, ranges, *common, **mkw)
    refs = []
    for f64 in (False, True):
        gr = oracle.render_backward(pre, vals, ranges, fwd, *common, gc.numpy(), go.numpy(), f64=f64, **mkw)
        pg = oracle.preprocess_backward(inp["means3D"].numpy(), inp["scales"].numpy(), inp["rotations"].numpy(),
                                        pre, gr, vm, pm, W, H, cam.tanfovx, cam.tanfovy, f64=f64)
        refs.append(dict(g=gr, pg=pg))
    np.testing.assert_array_equal(radii.cpu().numpy(), pre["radii"])
    return got, refs[0], refs[1], {**GRAD_KEYS, "colors_precomp": ("g", "dL_dcolors")}


@pytest.mark.parametrize("mode,total,hybrid,active,seed", [
    (4, 16, 6, 10, 19), (12, 16, 6, 10, 19), (14, 16, 6, 10, 19), (12, 14, 5, 7, 18), (14, 16, 16, 0, 18),
    (6, 16, 0, 10, 19), (7, 16, 0, 10, 19), (7, 12, 0, 0, 18), (0, 16, 0, 0, 19), (0, 2, 0, 0, 18)])
def test_render_modes_backward_match_oracle(mode, total, hybrid, active, seed):
    """Every gradient, the per-surfel rows' (blend weight included) among them,
    against the oracle's restatement of backward.cu:987-1033, 1425-1606 (itself
    pinned to float64 autograd in test_oracle_backward.py); table U(-1e-4, 1e-4)
    as in the benchmark."""
    from test_gpu_backward import check_all, upstream
    sc, inp, grid, gauss = mode_case(mode, total, hybrid, active, seed=seed)
    grid.table = (grid.table.float() * 1e-4).half()
    g = torch.Generator().manual_seed(seed)
    gc = torch.randn(total * 2, sc.camera.height, sc.camera.width, generator=g)
    _, go = upstream(sc, seed=5)
    got, ref, exact, keys = mode_grads(sc, inp, grid, gauss, mode, total, hybrid, active, gc, go)
    if active == 0:
        keys = {k: v for k, v in keys.items() if k != "table"}
        assert not got["table"].any()
    if mode == 0:  # level 0 adds nothing to the densification sum (backward.cu:833-849)
        keys = {k: v for k, v in keys.items() if k != "gradsum"}
        assert not got["gradsum"].any() and not ref["g"]["dL_gradsum"].any()
    check_all(got, ref, exact, keys=keys)


def test_dropin_mode_gradients_in_colors_precomp_slot():
    """The drop-in Function returns the per-surfel rows' gradient in
    colors_precomp's slot (mode 14); the inference flag has no backward."""
    from test_gpu_backward import upstream
    mode, total, hybrid, active = 14, 16, 6, 10
    sc, inp, grid, gauss = mode_case(mode, total, hybrid, active, seed=19)
    cam = sc.camera
    dev = "cuda"
    g = torch.Generator().manual_seed(19)
    gc = torch.randn(total * 2, cam.height, cam.width, generator=g)
    _, go = upstream(sc, seed=5)
    _, ref, _, _ = mode_grads(sc, inp, grid, gauss, mode, total, hybrid, active, gc, go)
    for flag in (0, 256):
        rs = dsr.GaussianRasterizationSettings(
            image_height=cam.height, image_width=cam.width, tanfovx=cam.tanfovx, tanfovy=cam.tanfovy,
            bg=torch.zeros(3, device=dev), scale_modifier=1.0, viewmatrix=cam.world_view_transform.to(dev),
            projmatrix=cam.full_proj_transform.to(dev), sh_degree=0, campos=cam.camera_center.to(dev),
            prefiltered=False, debug=False, beta=0.0, if_contract=False, record_transmittance=False,
            max_intersections=0)
        hs = dsr.HashGridSettings(L=(total << 16) | (active << 8) | hybrid, S=grid.S, H=grid.base_resolution,
                                  align_corners=False, interpolation=0,
                                  shape_dims=torch.tensor([12, 20, 32], dtype=torch.int32, device=dev))
        r = dsr.GaussianRasterizer(rs, hs)
        P = sc.P
        feats = gauss.to(dev).clone().requires_grad_(True)
        color, _, allmap, _, _ = r(
            means3D=inp["means3D"].to(dev), means2D=torch.zeros(P, 3, device=dev), shs=None, colors_precomp=feats,
            opacities=inp["opacities"].to(dev), scales=inp["scales"].to(dev), rotations=inp["rotations"].to(dev),
            homotrans=inp["homotrans"].to(dev), ap_level=inp["ap_level"].to(dev), features=grid.table.to(dev),
            offsets=grid.offsets.to(dev), gridrange=grid.gridrange.to(dev), render_mode=mode | flag)
        loss = (color * gc.to(dev)).sum() + (allmap * go.to(dev)).sum()
        if flag:
            with pytest.raises(NotImplementedError):
                loss.backward()
            continue
        loss.backward()
        got = feats.grad.cpu().numpy()
        want = ref["g"]["dL_dcolors"]
        assert got.shape == want.shape
        assert np.linalg.norm(got - want) / np.linalg.norm(want) < 1e-3
