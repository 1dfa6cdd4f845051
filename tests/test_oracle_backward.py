"""Pins the CPU oracle's backward (oracle/nest_oracle_bw.cpp) to float64 autograd.

The model in bw_model.py renders the same tile lists in float64 with torch and
is differentiated by autograd; the oracle restates the reference's hand-written
backward in float32. Agreement of every gradient (means, scales, rotations,
opacities, hash table) to 1e-4 relative L2 shows that the restatement computes
the reference's gradient formulas, not just something self-consistent.
"""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

import bw_model
from nest_b200 import camera, synth
from oracle import oracle


def rel_l2(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def tiny_case(seed, n=40, W=48, H=40, interp=0):
    g = torch.Generator().manual_seed(seed)
    base = synth.surfel_base(n, -1.8, 0.3, g)
    means = base[:, 0:3].contiguous()
    scales = torch.exp(base[:, 3:5]).contiguous()
    rots = F.normalize(base[:, 5:9], dim=-1).contiguous()
    opac = (0.05 + 0.9 * torch.sigmoid(base[:, 9])).contiguous()
    grid = synth.hash_grid(g, levels=4, log2_T=12, lo=-1.0, hi=1.0, base_resolution=4, per_level_scale=2.0)
    table = grid.table.float().contiguous()
    ap = (torch.randint(1, 6, (n,), generator=g).float() + 0.5).contiguous()
    R = synth.build_rotation(rots)
    homo = torch.zeros(n, 4, 4)
    homo[:, :3, 0] = R[:, :, 0] * scales[:, 0:1]
    homo[:, :3, 1] = R[:, :, 1] * scales[:, 1:2]
    homo[:, :3, 3] = means
    homo[:, 3, 3] = 1.0
    cam = camera.orbit_camera(W, H, 50.0)
    gc = torch.randn(grid.levels * grid.level_dim, H, W, generator=g)
    go = torch.randn(14, H, W, generator=g)
    go[7:] = 0.0  # count, position and level-vis maps carry no gradient in the reference
    return dict(means=means, scales=scales, rots=rots, opac=opac, table=table, grid=grid, ap=ap,
                homo=homo.reshape(n, 16), cam=cam, gc=gc, go=go, W=W, H=H, interp=interp)


def oracle_grads(c):
    cam, grid = c["cam"], c["grid"]
    vm, pm = cam.world_view_transform.numpy(), cam.full_proj_transform.numpy()
    W, H = c["W"], c["H"]
    pre = oracle.preprocess(c["means"].numpy(), c["scales"].numpy(), c["rots"].numpy(), c["opac"].numpy(), vm, pm,
                            W, H)
    _, vals, ranges = oracle.bin_surfels(pre, W, H)
    kw = dict(interp=c["interp"])
    if c.get("kernel_type"):
        kw.update(kernel_type=c["kernel_type"], shapes=c["shapes"].numpy())
    if "mode" in c:
        kw.update(render_mode=c["mode"], hybrid_levels=c["hybrid"], total_levels=c["total"], gauss=c["gauss"].numpy())
    C = c.get("C", c["total"] * grid.level_dim) if "mode" in c else grid.channels
    L = c.get("levels", grid.levels)
    fwd = oracle.render(pre, vals, ranges, c["homo"].numpy(), c["ap"].numpy(), c["table"].numpy(),
                        grid.offsets.numpy(), grid.gridrange.numpy(), W, H, C, grid.level_dim,
                        L, grid.S, grid.base_resolution, **kw)
    g = oracle.render_backward(pre, vals, ranges, fwd, c["homo"].numpy(), c["ap"].numpy(), c["table"].numpy(),
                               grid.offsets.numpy(), grid.gridrange.numpy(), W, H, C, grid.level_dim,
                               L, grid.S, grid.base_resolution, c["gc"].numpy(), c["go"].numpy(), **kw)
    pg = oracle.preprocess_backward(c["means"].numpy(), c["scales"].numpy(), c["rots"].numpy(), pre, g, vm, pm, W,
                                    H, cam.tanfovx, cam.tanfovy)
    return pre, vals, ranges, fwd, g, pg


def model_grads(c, pre, vals, ranges):
    cam, grid = c["cam"], c["grid"]
    names = ("means", "scales", "rots", "opac", "table") + (("shapes",) if c.get("kernel_type") else ())
    names = names + (("gauss",) if "mode" in c else ())
    leaves = [c[k].double().clone().requires_grad_(True) for k in names]
    means, scales, rots, opac, table = leaves[:5]
    info = dict(L=c.get("levels", grid.levels), LD=grid.level_dim, S=grid.S, H=grid.base_resolution,
                offsets=grid.offsets.numpy(), vmin=float(grid.gridrange[0]), vmax=float(grid.gridrange[1]),
                interp=c["interp"])
    rows = None
    if "mode" in c:
        rows = leaves[-1]
        if c["mode"] == 7:
            # mode 7's weight slot is differentiated as the pre-sigmoid parameter
            # (backward.cu:1183-1186): the leaf holds logit(weight)
            td = c["total"] * grid.level_dim
            rows = torch.cat([rows[:, :td], torch.sigmoid(rows[:, td:td + 1])], 1)
    visible = torch.as_tensor(pre["radii"] > 0)
    modes = None if "mode" not in c else dict(
        mode=c["mode"], gauss=rows, pg=c["hybrid"] * grid.level_dim, td=c["total"] * grid.level_dim,
        C=c.get("C", c["total"] * grid.level_dim), decompose=c["hybrid"])
    c["model_modes"] = modes
    color, others, margin, _ = bw_model.render(
        means, scales, rots, opac, table,
        dict(viewmatrix=cam.world_view_transform.numpy(), projmatrix=cam.full_proj_transform.numpy()),
        (ranges, vals), info, np.floor(c["ap"].numpy()).astype(np.int64), c["W"], c["H"],
        kernel_type=c.get("kernel_type", 0), shapes=leaves[5] if c.get("kernel_type") else None,
        modes=modes)
    loss = (color * c["gc"].double()).sum() + (others * c["go"][:7].double()).sum()
    loss.backward()
    grads = {k: (v.grad if v.grad is not None else torch.zeros_like(v)).detach().numpy()
             for k, v in zip(names, leaves)}
    for k in ("means", "scales", "rots", "opac"):
        grads[k][~visible.numpy()] = 0.0
    return color.detach().numpy(), others.detach().numpy(), margin, grads


@pytest.mark.parametrize("seed,interp", [(5, 0), (6, 0), (7, 1)])
def test_oracle_backward_matches_autograd(seed, interp):
    c = tiny_case(seed, interp=interp)
    pre, vals, ranges, fwd, g, pg = oracle_grads(c)
    color, others, margin, mg = model_grads(c, pre, vals, ranges)
    assert margin > 1e-5, "a branch sits on its threshold; pick another seed"
    # The float64 model renders what the float32 oracle renders.
    assert np.max(np.abs(color - fwd["out_color"])) < 2e-5
    assert np.max(np.abs(others - fwd["out_others"][:7])) < 2e-4
    checks = {"means": pg["dL_dmeans3D"], "scales": pg["dL_dscales"], "rots": pg["dL_drots"],
              "opac": g["dL_dopacity"], "table": g["dL_dtable"]}
    for k, got in checks.items():
        assert np.linalg.norm(mg[k]) > 0, k
        assert rel_l2(got, mg[k]) < 1e-4, (k, rel_l2(got, mg[k]))


def test_oracle_backward_gradsum_and_mean2d_statistic():
    c = tiny_case(8)
    pre, vals, ranges, fwd, g, pg = oracle_grads(c)
    # dL_gradsum: per sample alpha*T*sum|dL/dcolor| (backward.cu:1780-1784), so it is
    # zero exactly for surfels no pixel blends and positive otherwise.
    blended = fwd["out_others"][7].sum() > 0
    assert blended and np.all(g["dL_gradsum"] >= 0) and g["dL_gradsum"].sum() > 0
    # The means2D gradient returned to Python is the densification statistic
    # dL/dT[2] * depth * W/2 (backward.cu:2268-2272) with W = int(focal * tan * 2).
    cam = c["cam"]
    fx = np.float32(c["W"]) / (np.float32(2.0) * np.float32(cam.tanfovx))
    Wq = int(np.float32(np.float32(fx * np.float32(cam.tanfovx)) * np.float32(2)))
    vis = pre["radii"] > 0
    expect = (g["dL_dtransMat"][:, 2] * pre["transMat"][:, 8]).astype(np.float64) * 0.5 * Wq
    np.testing.assert_allclose(pg["dL_dmean2D"][vis, 0], expect[vis].astype(np.float32), rtol=1e-6, atol=0)


@pytest.mark.parametrize("kernel_type,lo,hi,seed", [(1, 0.5, 3.0, 11), (2, 0.2, 2.0, 12), (2, -1.0, 0.0, 5),
                                                    (3, 2.0, 6.0, 14)])
def test_oracle_backward_splat_kernels_match_autograd(kernel_type, lo, hi, seed):
    """The splat kernels' gradients (backward.cu:1862-2045), dL/dshape included,
    against autograd of the same forward (kernel 1 with the reference's halved
    rho derivative, stated in bw_model)."""
    c = tiny_case(seed)
    g = torch.Generator().manual_seed(seed)
    c["kernel_type"] = kernel_type
    c["shapes"] = (torch.rand(c["means"].shape[0], generator=g) * (hi - lo) + lo).float()
    pre, vals, ranges, fwd, gr, pg = oracle_grads(c)
    color, others, margin, mg = model_grads(c, pre, vals, ranges)
    assert margin > 1e-5, "a branch sits on its threshold; pick another seed"
    assert np.max(np.abs(color - fwd["out_color"])) < 2e-5
    assert np.max(np.abs(others - fwd["out_others"][:7])) < 2e-4
    checks = {"means": pg["dL_dmeans3D"], "scales": pg["dL_dscales"], "rots": pg["dL_drots"],
              "opac": gr["dL_dopacity"], "table": gr["dL_dtable"], "shapes": gr["dL_dshapes"]}
    if hi <= 0:  # flex kernel with shape <= 0: the plain Gaussian, no shape gradient
        assert not gr["dL_dshapes"].any()
        checks.pop("shapes")
    for k, got in checks.items():
        assert np.linalg.norm(mg[k]) > 0, k
        assert rel_l2(got, mg[k]) < 1e-4, (k, rel_l2(got, mg[k]))


@pytest.mark.parametrize("mode,seed", [(4, 21), (12, 22), (14, 23), (6, 24), (7, 27), (0, 26)])
def test_oracle_backward_render_modes_match_autograd(mode, seed):
    """Render modes 4 / 6 / 7 / 12 / 14 (training rules) and level 0 (mode 0
    without hash levels): every gradient, the per-surfel rows' (colors_precomp,
    blend weight included) among them, against autograd of the same forward.
    The colour term of dL/dalpha uses the forward's feature vector (the
    reference's cases 12 and 14 read an unwritten array there); mode 7's weight
    slot is the pre-sigmoid parameter's gradient, as the reference returns it."""
    c = tiny_case(seed)
    g = torch.Generator().manual_seed(seed)
    n = c["means"].shape[0]
    total = 4
    hybrid = 1 if mode in (4, 12, 14) else 0
    grid = synth.hash_grid(g, levels=3, log2_T=12, lo=-1.0, hi=1.0, base_resolution=8, per_level_scale=2.0)
    LD = grid.level_dim
    c.update(grid=grid, table=grid.table.float().contiguous(), mode=mode, hybrid=hybrid, total=total)
    if mode == 0:
        c["levels"] = 0
    c["gc"] = torch.randn(total * LD, c["H"], c["W"], generator=g)
    width = {4: hybrid * LD, 12: total * LD + 1, 14: hybrid * LD + 1, 6: total * LD, 7: total * LD + 1,
             0: total * LD}[mode]
    gauss = torch.rand(n, width, generator=g) * 2 - 1
    if mode in (7, 12, 14):
        gauss[:, -1] = torch.rand(n, generator=g) * 0.8 + 0.1
    c["gauss"] = gauss.contiguous()
    pre, vals, ranges, fwd, gr, pg = oracle_grads(c)
    if mode == 7:  # the model's leaf for the weight slot is logit(weight)
        c["gauss"] = torch.cat([gauss[:, :-1].double(), torch.logit(gauss[:, -1:].double())], 1)
    color, others, margin, mg = model_grads(c, pre, vals, ranges)
    assert margin > 1e-5, "a branch sits on its threshold; pick another seed"
    assert np.max(np.abs(color - fwd["out_color"])) < 2e-5
    checks = {"means": pg["dL_dmeans3D"], "scales": pg["dL_dscales"], "rots": pg["dL_drots"],
              "opac": gr["dL_dopacity"], "gauss": gr["dL_dcolors"]}
    if mode != 0:  # level 0 reads no table
        checks["table"] = gr["dL_dtable"]
    for k, got in checks.items():
        assert np.linalg.norm(mg[k]) > 0, k
        assert rel_l2(got, mg[k]) < 1e-4, (k, rel_l2(got, mg[k]))


def sh_grid(g, levels=1):
    """A single-level hash grid with 3-wide rows U(-2, 2) (modes 8-10 query one
    3-channel level, query_feature<false, 3, 3>)."""
    from types import SimpleNamespace
    base = synth.hash_grid(g, levels=levels, log2_T=12, lo=-1.0, hi=1.0, base_resolution=8, per_level_scale=2.0)
    rows = int(base.offsets[-1])
    table = (torch.rand(rows, 3, generator=g) * 4 - 2).contiguous()
    return SimpleNamespace(table=table, offsets=base.offsets, gridrange=base.gridrange, S=base.S,
                           base_resolution=base.base_resolution, level_dim=3, levels=levels, channels=3)


@pytest.mark.parametrize("mode,decompose,seed", [(8, 0, 31), (8, 1, 42), (8, 2, 33), (10, 0, 34), (10, 1, 38),
                                                 (10, 2, 44), (9, 0, 36), (9, 2, 39)])
def test_oracle_backward_sh_hybrid_modes_match_autograd(mode, decompose, seed):
    """Render modes 8 (hybrid_SH), 9 (hybrid_SH_post) and 10 (hybrid_SH_raw):
    one 3-wide hash level and per-surfel rows (3 raw SH colours; 48 SH
    coefficients for 9), with each decompose flag. The reference's backward
    multiplies the row and table gradients (and so dL/dxyz) by alpha T once more
    than the derivative of its forward; the model reproduces that by scaling
    the gradient through the feature by the detached weight."""
    c = tiny_case(seed)
    g = torch.Generator().manual_seed(seed)
    n = c["means"].shape[0]
    grid = sh_grid(g)
    C = 48 if mode == 9 else 3
    c.update(grid=grid, table=grid.table, mode=mode, hybrid=decompose, total=3, levels=1, C=C)
    c["gc"] = torch.randn(C, c["H"], c["W"], generator=g)
    c["gauss"] = (torch.rand(n, C, generator=g) * 2 - 1).contiguous()
    pre, vals, ranges, fwd, gr, pg = oracle_grads(c)
    color, others, margin, mg = model_grads(c, pre, vals, ranges)
    assert margin > 1e-5, "a branch sits on its threshold; pick another seed"
    assert np.max(np.abs(color - fwd["out_color"])) < 2e-5
    checks = {"means": pg["dL_dmeans3D"], "scales": pg["dL_dscales"], "rots": pg["dL_drots"],
              "opac": gr["dL_dopacity"]}
    if decompose != 2:
        checks["gauss"] = gr["dL_dcolors"]
    else:
        assert not np.any(gr["dL_dcolors"])
    if decompose != 1:
        checks["table"] = gr["dL_dtable"]
    else:
        assert not np.any(gr["dL_dtable"])
    for k, got in checks.items():
        assert np.linalg.norm(mg[k]) > 0, k
        assert rel_l2(got, mg[k]) < 1e-4, (k, rel_l2(got, mg[k]))


def test_oracle_residual_hybrid_mode_11():
    """Render mode 11 (residual_hybrid): the hash levels from channel 0 with
    mode 0's gradients and no gradient for the SH rows; the rows' degree-3 SH
    colour (48 coefficients read interleaved, along hit - centre) blended into
    out_others channels 14-16, against the float64 model."""
    seed = 41
    c = tiny_case(seed)
    g = torch.Generator().manual_seed(seed)
    n = c["means"].shape[0]
    grid = synth.hash_grid(g, levels=3, log2_T=12, lo=-1.0, hi=1.0, base_resolution=8, per_level_scale=2.0)
    c.update(grid=grid, table=grid.table.float().contiguous(), mode=11, hybrid=0, total=3, levels=3, C=6)
    c["gc"] = torch.randn(6, c["H"], c["W"], generator=g)
    c["gauss"] = (torch.rand(n, 48, generator=g) * 2 - 1).contiguous()
    pre, vals, ranges, fwd, gr, pg = oracle_grads(c)
    assert fwd["out_others"].shape[0] == 17
    color, others, margin, mg = model_grads(c, pre, vals, ranges)
    assert margin > 1e-5
    assert np.max(np.abs(color - fwd["out_color"])) < 2e-5
    sh = c["model_modes"]["sh_rgb"].numpy()
    assert np.abs(sh).max() > 0.1
    assert np.max(np.abs(sh - fwd["out_others"][14:17])) < 2e-5
    assert not np.any(gr["dL_dcolors"])
    checks = {"means": pg["dL_dmeans3D"], "scales": pg["dL_dscales"], "rots": pg["dL_drots"],
              "opac": gr["dL_dopacity"], "table": gr["dL_dtable"]}
    for k, got in checks.items():
        assert np.linalg.norm(mg[k]) > 0, k
        assert rel_l2(got, mg[k]) < 1e-4, (k, rel_l2(got, mg[k]))


@pytest.mark.parametrize("deg", [0, 1, 2, 3])
def test_oracle_sh_color_backward_matches_autograd(deg):
    """computeColorFromSH's backward (backward.cu:21-140, dnormvdv): dL/dsh and
    the mean's view-direction gradient against float64 autograd of the SH
    colour (clamped channels pass no gradient); culled surfels get zeros."""
    g = torch.Generator().manual_seed(90 + deg)
    P, M = 50, 16
    shs = (torch.randn(P, M, 3, generator=g) * 0.6).float()
    means = torch.randn(P, 3, generator=g).float()
    campos = torch.tensor([0.3, -4.0, 0.8])
    radii = np.ones(P, np.int32)
    radii[::7] = 0
    up = torch.randn(P, 3, generator=g).double()
    m = means.double().requires_grad_(True)
    sh = shs.double().reshape(P, -1).requires_grad_(True)
    d = m - campos.double()
    d = d / d.norm(dim=1, keepdim=True)
    rgb = bw_model.eval_sh_interleaved(sh, d, deg)
    assert np.abs(rgb.detach().numpy() - oracle.sh_color(means.numpy(), campos.numpy(), shs.numpy(), deg)).max() < 1e-5
    (rgb * up).sum().backward()
    dsh, dmean = oracle.sh_color_backward(means.numpy(), campos.numpy(), shs.numpy(), deg, radii, up.numpy())
    on = radii > 0
    want_sh = sh.grad.numpy().reshape(P, M, 3)
    assert not dsh[~on].any() and not dmean[~on].any()
    assert rel_l2(dsh[on], want_sh[on]) < 1e-5, rel_l2(dsh[on], want_sh[on])
    if deg > 0:
        assert rel_l2(dmean[on], m.grad.numpy()[on]) < 1e-4, rel_l2(dmean[on], m.grad.numpy()[on])
    else:
        assert np.abs(dmean).max() < 1e-6
    d64, m64 = oracle.sh_color_backward(means.numpy(), campos.numpy(), shs.numpy(), deg, radii, up.numpy(), f64=True)
    assert rel_l2(d64[on], want_sh[on]) < 1e-7  # the constants are the reference's float values


def test_oracle_precomputed_transforms_match_autograd():
    """The reference's transMat_precomp path (pipe.compute_cov3D_python;
    forward.cu:366-380, backward.cu:2082-2088, 2128-2158): transforms given per
    surfel, the normal the view axis, the hit point from the given homotrans.
    The transforms' gradient (render pass plus the centre's mean2D term),
    opacity and table against float64 autograd of the same forward with the
    transforms as leaves; means, scales and rotations get nothing."""
    c = tiny_case(52)
    cam, grid = c["cam"], c["grid"]
    vm, pm = cam.world_view_transform.numpy(), cam.full_proj_transform.numpy()
    W, H = c["W"], c["H"]
    g = torch.Generator().manual_seed(52)
    pre0 = oracle.preprocess(c["means"].numpy(), c["scales"].numpy(), c["rots"].numpy(), c["opac"].numpy(), vm,
                             pm, W, H)
    Ts = (pre0["transMat"] * (1 + 1e-2 * torch.randn(pre0["transMat"].shape, generator=g).numpy())).astype(
        np.float32)
    pre = oracle.preprocess(c["means"].numpy(), None, None, c["opac"].numpy(), vm, pm, W, H, transmat_precomp=Ts)
    assert (pre["radii"] > 0).sum() > 10
    assert np.allclose(pre["normal_opacity"][pre["radii"] > 0, 2], -1.0)
    _, vals, ranges = oracle.bin_surfels(pre, W, H)
    common = (c["homo"].numpy(), c["ap"].numpy(), c["table"].numpy(), grid.offsets.numpy(), grid.gridrange.numpy(),
              W, H, grid.channels, grid.level_dim, grid.levels, grid.S, grid.base_resolution)
    fwd = oracle.render(pre, vals, ranges, *common)
    gr = oracle.render_backward(pre, vals, ranges, fwd, *common, c["gc"].numpy(), c["go"].numpy())
    pg = oracle.preprocess_backward(None, None, None, pre, gr, vm, pm, W, H, cam.tanfovx, cam.tanfovy,
                                    precomp=True)
    assert not pg["dL_dmeans3D"].any() and not pg["dL_dscales"].any() and not pg["dL_drots"].any()

    Tl = torch.tensor(Ts, dtype=torch.float64).requires_grad_(True)
    opac = c["opac"].double().clone().requires_grad_(True)
    table = c["table"].double().clone().requires_grad_(True)
    info = dict(L=grid.levels, LD=grid.level_dim, S=grid.S, H=grid.base_resolution, offsets=grid.offsets.numpy(),
                vmin=float(grid.gridrange[0]), vmax=float(grid.gridrange[1]), interp=0)
    color, others, margin, _ = bw_model.render(
        c["means"].double(), None, None, opac, table,
        dict(viewmatrix=vm, projmatrix=pm), (ranges, vals), info, np.floor(c["ap"].numpy()).astype(np.int64), W, H,
        Ts=Tl, homo=c["homo"].numpy())
    assert margin > 1e-5
    assert np.max(np.abs(color.detach().numpy() - fwd["out_color"])) < 2e-5
    ((color * c["gc"].double()).sum() + (others * c["go"][:7].double()).sum()).backward()
    on = pre["radii"] > 0
    checks = {"transMat": (pg["dL_dtransMat"][on], Tl.grad.numpy()[on]),
              "opac": (gr["dL_dopacity"], opac.grad.numpy()), "table": (gr["dL_dtable"], table.grad.numpy())}
    for k, (got, want) in checks.items():
        assert np.linalg.norm(want) > 0, k
        assert rel_l2(got, want) < 1e-4, (k, rel_l2(got, want))
