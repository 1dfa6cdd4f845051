"""GPU parity of the spherical-harmonic hybrid render modes against the oracle:
8 hybrid_SH (forward.cu:1378-1437), 9 hybrid_SH_post (:1438-1482), 10
hybrid_SH_raw (:1483-1526) with one 3-wide hash level and the decompose flag,
and 11 residual_hybrid (:1527-1592, :1918-1943, :2039-2045: hash features in
out_color, the rows' degree-3 SH colour in out_others channels 14-16); the
backward of each (backward.cu:1191-1424). The level words and rows are built as
the reference's renderer builds them (gaussian_renderer/__init__.py:570-686):
decompose << 24 | SH degree << 16 | 1 << 8 with rows of 3 raw SH colours (48
SH coefficients for 9), and total << 16 | hash levels << 8 | hybrid with rows
of 48 SH coefficients for 11. The oracle's restatement of these modes is
pinned to float64 autograd in test_oracle_backward.py."""
import numpy as np
import pytest
import torch

import diff_surfel_rasterization as dsr
from helpers import api_inputs, compare, small_scene
from nest_b200 import _lib, raster, synth
from oracle import oracle

pytestmark = pytest.mark.gpu


def sh_case(mode, seed, fp16=False, levels=3):
    """A small scene, a table (one 3-wide level U(-2, 2) for modes 8-10; the
    scene's 2-wide levels for 11) and the per-surfel rows."""
    sc = small_scene(n=1500, seed=seed)
    inp = api_inputs(sc)
    g = torch.Generator().manual_seed(seed)
    if mode == 11:
        grid = synth.hash_grid(g, levels=levels, log2_T=13, lo=-1.0, hi=1.0, base_resolution=64,
                               per_level_scale=1.5)
        table = grid.table.float()
    else:
        grid = synth.hash_grid(g, levels=1, log2_T=13, lo=-1.0, hi=1.0, base_resolution=64, per_level_scale=1.5)
        table = torch.rand(int(grid.offsets[-1]), 3, generator=g) * 4 - 2
    table = table.half() if fp16 else table
    width = 3 if mode in (8, 10) else 48
    rows = (torch.rand(sc.P, width, generator=g) * 2 - 1).contiguous()
    return sc, inp, grid, table.contiguous(), rows


def dims(mode, levels):
    """(C, level_dim, hash levels) of a mode."""
    if mode == 11:
        return 2 * levels, 2, levels
    return (48 if mode == 9 else 3), 3, 1


def oracle_forward(sc, inp, grid, table, rows, mode, decompose, levels):
    cam = sc.camera
    C, LD, L = dims(mode, levels)
    out, _, _ = oracle.forward(inp["means3D"].numpy(), inp["scales"].numpy(), inp["rotations"].numpy(),
                               inp["opacities"].numpy(), inp["homotrans"].numpy(), inp["ap_level"].numpy(),
                               table.float().numpy(), grid.offsets.numpy(), grid.gridrange.numpy(),
                               cam.world_view_transform.numpy(), cam.full_proj_transform.numpy(), cam.width,
                               cam.height, C, LD, L, grid.S, grid.base_resolution, render_mode=mode,
                               hybrid_levels=decompose, total_levels=3 if mode != 11 else levels,
                               gauss=rows.numpy())
    return out


def dropin_forward(sc, inp, grid, table, rows, mode, decompose, levels):
    cam = sc.camera
    dev = "cuda"
    rs = dsr.GaussianRasterizationSettings(
        image_height=cam.height, image_width=cam.width, tanfovx=cam.tanfovx, tanfovy=cam.tanfovy,
        bg=torch.zeros(3, device=dev), scale_modifier=1.0, viewmatrix=cam.world_view_transform.to(dev),
        projmatrix=cam.full_proj_transform.to(dev), sh_degree=3, campos=cam.camera_center.to(dev),
        prefiltered=False, debug=False, beta=0.0, if_contract=False, record_transmittance=False,
        max_intersections=0)
    if mode == 11:
        word = (levels << 16) | (levels << 8) | 0
        shape_dims = torch.tensor([48, 2 * levels, 0], dtype=torch.int32, device=dev)
    else:
        word = (decompose << 24) | (3 << 16) | (1 << 8)
        shape_dims = torch.tensor([0, 3, 3], dtype=torch.int32, device=dev)
    hs = dsr.HashGridSettings(L=word, S=grid.S, H=grid.base_resolution, align_corners=False, interpolation=0,
                              shape_dims=shape_dims)
    r = dsr.GaussianRasterizer(rs, hs)
    P = sc.P
    with torch.no_grad():
        color, _, allmap, _, _ = r(
            means3D=inp["means3D"].to(dev), means2D=torch.zeros(P, 3, device=dev), shs=None,
            colors_precomp=rows.to(dev), opacities=inp["opacities"].to(dev), scales=inp["scales"].to(dev),
            rotations=inp["rotations"].to(dev), homotrans=inp["homotrans"].to(dev),
            ap_level=inp["ap_level"].to(dev), features=table.to(dev), offsets=grid.offsets.to(dev),
            gridrange=grid.gridrange.to(dev), render_mode=mode)
    torch.cuda.synchronize()
    return color.cpu().numpy(), allmap.cpu().numpy()


@pytest.mark.parametrize("mode,decompose,fp16", [
    (8, 0, False), (8, 1, False), (8, 2, False), (8, 0, True),
    (10, 0, False), (10, 1, False), (10, 2, True),
    (9, 0, False), (9, 1, False), (9, 2, True),
    (11, 0, False), (11, 0, True),
])
def test_sh_modes_forward_match_oracle(mode, decompose, fp16):
    levels = 3
    sc, inp, grid, table, rows = sh_case(mode, seed=70 + mode + 3 * decompose, fp16=fp16, levels=levels)
    out = oracle_forward(sc, inp, grid, table, rows, mode, decompose, levels)
    color, allmap = dropin_forward(sc, inp, grid, table, rows, mode, decompose, levels)
    C = dims(mode, levels)[0]
    assert color.shape[0] == C and allmap.shape[0] == (17 if mode == 11 else 14)
    assert allmap[7].sum() > 100
    assert np.abs(out["out_color"]).max() > 0.1
    compare(out, color, allmap)
    if mode == 11:
        sh_ref = out["out_others"][14:17]
        assert np.abs(sh_ref).max() > 0.1
        err = np.abs(allmap[14:17] - sh_ref).max(axis=0)
        assert (err > 2e-3).mean() <= 1e-3, ((err > 2e-3).mean(), err.max())


def sh_grads(sc, inp, grid, table, rows, mode, decompose, levels, gc, go):
    """GPU gradients through raster.rasterize_forward / rasterize_backward and
    the oracle's (float32 and float64) on the same lists."""
    from test_gpu_backward import GRAD_KEYS
    cam = sc.camera
    C, LD, L = dims(mode, levels)
    total = 3 if mode != 11 else levels
    cfg = raster.RasterConfig(
        image_height=cam.height, image_width=cam.width, tanfovx=cam.tanfovx, tanfovy=cam.tanfovy,
        viewmatrix=cam.world_view_transform.cuda().contiguous(),
        projmatrix=cam.full_proj_transform.cuda().contiguous(), levels=L, S=grid.S,
        base_resolution=grid.base_resolution, channels=C, level_dim=LD, table_fp16=table.dtype == torch.float16,
        render_mode=mode, hybrid_levels=decompose, total_levels=total)
    args = (inp["means3D"].cuda().contiguous(), inp["scales"].cuda().contiguous(),
            inp["rotations"].cuda().contiguous(), inp["opacities"].cuda().reshape(-1).contiguous(),
            inp["homotrans"].cuda().reshape(-1, 16).contiguous(), inp["ap_level"].cuda().reshape(-1).contiguous(),
            table.cuda().contiguous(), grid.offsets.cuda().contiguous(), grid.gridrange.cuda().contiguous())
    gcol = rows.cuda().contiguous()
    n, color, others, radii, _, _, scratch = raster.rasterize_forward(cfg, *args, colors_precomp=gcol)
    got = raster.rasterize_backward(cfg, *args, radii, n, scratch, gc.cuda(), go.cuda(), colors_precomp=gcol)
    torch.cuda.synchronize()
    got = {k: v.cpu().numpy() for k, v in got.items()}
    vm, pm = cam.world_view_transform.numpy(), cam.full_proj_transform.numpy()
    W, H = cam.width, cam.height
    pre = oracle.preprocess(inp["means3D"].numpy(), inp["scales"].numpy(), inp["rotations"].numpy(),
                            inp["opacities"].numpy(), vm, pm, W, H)
    _, vals, ranges = oracle.bin_surfels(pre, W, H)
    common = (inp["homotrans"].numpy(), inp["ap_level"].numpy(), table.float().numpy(), grid.offsets.numpy(),
              grid.gridrange.numpy(), W, H, C, LD, L, grid.S, grid.base_resolution)
    mkw = dict(render_mode=mode, hybrid_levels=decompose, total_levels=total, gauss=rows.numpy())
    fwd = oracle.render(pre, vals, ranges, *common, **mkw)
    refs = []
    for f64 in (False, True):
        gr = oracle.render_backward(pre, vals, ranges, fwd, *common, gc.numpy(), go.numpy(), f64=f64, **mkw)
        pg = oracle.preprocess_backward(inp["means3D"].numpy(), inp["scales"].numpy(), inp["rotations"].numpy(),
                                        pre, gr, vm, pm, W, H, cam.tanfovx, cam.tanfovy, f64=f64)
        refs.append(dict(g=gr, pg=pg))
    np.testing.assert_array_equal(radii.cpu().numpy(), pre["radii"])
    return got, refs[0], refs[1], {**GRAD_KEYS, "colors_precomp": ("g", "dL_dcolors")}


@pytest.mark.parametrize("mode,decompose,seed", [
    (8, 0, 80), (8, 1, 81), (8, 2, 82), (10, 0, 83), (10, 2, 84), (9, 0, 85), (9, 1, 86), (11, 0, 87)])
def test_sh_modes_backward_match_oracle(mode, decompose, seed):
    """Every gradient against the oracle's restatement of backward.cu:1191-1424
    (the reference's alpha T applied twice to the row and table gradients of
    modes 8-10 included; no row gradient in mode 11)."""
    from test_gpu_backward import check_all, upstream
    levels = 3
    sc, inp, grid, table, rows = sh_case(mode, seed=seed, levels=levels)
    if mode == 11:
        table = table * 1e-2
    C = dims(mode, levels)[0]
    g = torch.Generator().manual_seed(seed)
    gc = torch.randn(C, sc.camera.height, sc.camera.width, generator=g)
    _, go = upstream(sc, seed=5)
    if mode == 11:
        go = torch.cat([go, torch.randn(3, *go.shape[1:], generator=g)], 0)  # SH maps: no gradient
    got, ref, exact, keys = sh_grads(sc, inp, grid, table, rows, mode, decompose, levels, gc, go)
    if decompose == 1:  # the surfel only: the grid is not read
        keys = {k: v for k, v in keys.items() if k != "table"}
        assert not got["table"].any()
    if decompose == 2 or mode == 11:  # the grid only (or mode 11): no row gradient
        keys = {k: v for k, v in keys.items() if k != "colors_precomp"}
        assert not got["colors_precomp"].any()
    check_all(got, ref, exact, keys=keys)


def test_sh_modes_deterministic_table_gradient():
    """Mode 8's table gradient in 64-bit fixed point: bit-identical over two runs
    and within rounding of the float-atomic one."""
    from test_gpu_backward import upstream
    sc, inp, grid, table, rows = sh_case(8, seed=88)
    g = torch.Generator().manual_seed(88)
    gc = torch.randn(3, sc.camera.height, sc.camera.width, generator=g)
    _, go = upstream(sc, seed=5)
    cam = sc.camera
    outs = []
    for det in (True, True, False):
        cfg = raster.RasterConfig(
            image_height=cam.height, image_width=cam.width, tanfovx=cam.tanfovx, tanfovy=cam.tanfovy,
            viewmatrix=cam.world_view_transform.cuda().contiguous(),
            projmatrix=cam.full_proj_transform.cuda().contiguous(), levels=1, S=grid.S,
            base_resolution=grid.base_resolution, channels=3, level_dim=3, table_fp16=False, render_mode=8,
            hybrid_levels=0, total_levels=3, deterministic=det)
        args = (inp["means3D"].cuda().contiguous(), inp["scales"].cuda().contiguous(),
                inp["rotations"].cuda().contiguous(), inp["opacities"].cuda().reshape(-1).contiguous(),
                inp["homotrans"].cuda().reshape(-1, 16).contiguous(),
                inp["ap_level"].cuda().reshape(-1).contiguous(), table.cuda().contiguous(),
                grid.offsets.cuda().contiguous(), grid.gridrange.cuda().contiguous())
        gcol = rows.cuda().contiguous()
        n, _, _, radii, _, _, scratch = raster.rasterize_forward(cfg, *args, colors_precomp=gcol)
        got = raster.rasterize_backward(cfg, *args, radii, n, scratch, gc.cuda(), go.cuda(), colors_precomp=gcol)
        outs.append(got["table"].cpu().numpy())
    assert np.array_equal(outs[0], outs[1])
    assert np.abs(outs[0]).max() > 0
    assert np.linalg.norm(outs[0] - outs[2]) / np.linalg.norm(outs[2]) < 1e-5


def test_sh_modes_reject_bad_shapes():
    """Modes 8-10 take one 3-wide level and C = 3 (48 for mode 9); mode 11 needs
    three accumulators after its C channels."""
    sc, inp, grid, table, rows = sh_case(8, seed=89)
    cam = sc.camera
    base = dict(image_height=cam.height, image_width=cam.width, tanfovx=cam.tanfovx, tanfovy=cam.tanfovy,
                viewmatrix=cam.world_view_transform.cuda().contiguous(),
                projmatrix=cam.full_proj_transform.cuda().contiguous(), S=grid.S,
                base_resolution=grid.base_resolution, table_fp16=False, total_levels=3)
    args = (inp["means3D"].cuda().contiguous(), inp["scales"].cuda().contiguous(),
            inp["rotations"].cuda().contiguous(), inp["opacities"].cuda().reshape(-1).contiguous(),
            inp["homotrans"].cuda().reshape(-1, 16).contiguous(), inp["ap_level"].cuda().reshape(-1).contiguous(),
            table.cuda().contiguous(), grid.offsets.cuda().contiguous(), grid.gridrange.cuda().contiguous())
    bad = [dict(levels=1, channels=3, level_dim=2, render_mode=8),     # 2-wide table
           dict(levels=2, channels=6, level_dim=3, render_mode=8),     # two levels
           dict(levels=1, channels=3, level_dim=3, render_mode=9),     # mode 9 wants 48
           dict(levels=1, channels=3, level_dim=3, render_mode=10, hybrid_levels=3),  # decompose 3
           dict(levels=15, channels=30, level_dim=2, render_mode=11)]  # 30 + 3 > 32
    for kw in bad:
        cfg = raster.RasterConfig(**base, **kw)
        with pytest.raises(_lib.NestError):
            raster.rasterize_forward(cfg, *args, colors_precomp=rows.cuda().contiguous())
