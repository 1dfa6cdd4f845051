"""The fused depth-normal error (ns_normal_error / ns_normal_error_backward)
against the plain fp32 torch restatement of the reference's expressions
(nest_b200.train.decode_allmap: gaussian_renderer/__init__.py:763-792,
utils/point_utils.py:10-30,48-60, train.py:674) and its torch autograd.

Tolerances: error map max-abs 2e-3 (the image tolerance); gradients rel L2
1e-3 over pixels where alpha > 0 (torch's autograd gives 0 / 0 = NaN for D and
alpha at alpha == 0; the kernel gives 0 there, checked separately).
"""
import pytest
import torch

from nest_b200 import camera, train


def synthetic_allmap(W, H, seed, zero_alpha_frac=0.05):
    """An allmap of a smooth surface: expected depth 3-5 along the rays with a
    ripple, alpha in (0.2, 1] with some exact zeros (D = 0 there), unit-ish
    view-space normals scaled by alpha."""
    g = torch.Generator().manual_seed(seed)
    ys, xs = torch.meshgrid(torch.linspace(0, 1, H), torch.linspace(0, 1, W), indexing="ij")
    depth = 4.0 + 0.6 * xs - 0.4 * ys + 0.05 * torch.sin(9 * xs) * torch.cos(7 * ys)
    alpha = 0.2 + 0.8 * torch.rand(H, W, generator=g)
    alpha[torch.rand(H, W, generator=g) < zero_alpha_frac] = 0.0
    n = torch.randn(3, H, W, generator=g)
    n[2] = -n[2].abs() - 1.0
    n = n / n.norm(dim=0, keepdim=True)
    allmap = torch.zeros(14, H, W)
    allmap[0] = depth * alpha
    allmap[1] = alpha
    allmap[2:5] = n * alpha
    allmap[5] = depth
    allmap[6] = torch.rand(H, W, generator=g)
    return allmap


def kernel_and_torch(allmap_cpu, cam, up=None):
    dev = "cuda"
    a1 = allmap_cpu.to(dev).requires_grad_(True)
    err = train.normal_error(a1, cam)
    a2 = allmap_cpu.to(dev).requires_grad_(True)
    ref = train.normal_error_torch(a2, cam)
    if up is None:
        err.mean().backward()
        ref.mean().backward()
    else:
        (err * up).sum().backward()
        (ref * up).sum().backward()
    return err.detach(), ref.detach(), a1.grad, a2.grad


def check_grads(got, ref, alpha):
    on = (alpha > 0)[None].expand_as(got).clone()
    on[5:] = False
    g, r = got[on], ref[on]
    assert torch.isfinite(g).all()
    rel = float((g - r).norm() / r.norm().clamp_min(1e-30))
    assert rel < 1e-3, rel
    assert torch.all(got[5:] == 0)
    off = alpha == 0
    assert torch.all(got[0][off] == 0) and torch.all(got[1][off] == 0)


@pytest.mark.gpu
@pytest.mark.parametrize("W,H,seed", [(128, 96, 1), (97, 61, 2), (333, 17, 3)])
def test_normal_error_forward_and_mean_backward(W, H, seed):
    cam = camera.orbit_camera(W, H, 55.0, azimuth_deg=20.0 * seed, elevation_deg=10.0)
    allmap = synthetic_allmap(W, H, seed)
    err, ref, g, gr = kernel_and_torch(allmap, cam)
    assert err.shape == (H, W)
    assert float((err - ref).abs().max()) < 2e-3
    assert torch.all(err[0] == 1) and torch.all(err[:, -1] == 1)
    check_grads(g, gr, allmap[1].cuda())


@pytest.mark.gpu
def test_normal_error_per_pixel_upstream():
    W, H = 160, 120
    cam = camera.orbit_camera(W, H, 60.0, azimuth_deg=-35.0)
    allmap = synthetic_allmap(W, H, 7, zero_alpha_frac=0.2)
    up = torch.randn(H, W, generator=torch.Generator().manual_seed(8)).cuda()
    err, ref, g, gr = kernel_and_torch(allmap, cam, up)
    assert float((err - ref).abs().max()) < 2e-3
    check_grads(g, gr, allmap[1].cuda())


@pytest.mark.gpu
@pytest.mark.parametrize("W,H", [(1, 1), (2, 2), (3, 3), (1, 50), (50, 1), (3, 40)])
def test_normal_error_tiny_images(W, H):
    cam = camera.orbit_camera(W, H, 50.0)
    allmap = synthetic_allmap(W, H, 11, zero_alpha_frac=0.0)
    err, ref, g, gr = kernel_and_torch(allmap, cam)
    assert float((err - ref).abs().max()) < 2e-3
    if W < 3 or H < 3:  # no interior pixel: error 1 everywhere, no gradient
        assert torch.all(err == 1) and torch.all(g == 0)
    else:
        check_grads(g, gr, allmap[1].cuda())


@pytest.mark.gpu
def test_normal_error_on_rasterized_allmap():
    """A real allmap (the rasterizer's out_others) of the small test scene."""
    from helpers import small_scene
    import diff_surfel_rasterization as dsr

    sc = small_scene(seed=5)
    state = train.make_state(sc)
    cam, grid = sc.camera, sc.grid
    dev = "cuda"
    rs = dsr.GaussianRasterizationSettings(
        image_height=cam.height, image_width=cam.width, tanfovx=cam.tanfovx, tanfovy=cam.tanfovy,
        bg=torch.zeros(3, device=dev), scale_modifier=1.0, viewmatrix=cam.world_view_transform.to(dev),
        projmatrix=cam.full_proj_transform.to(dev), sh_degree=0, campos=cam.camera_center.to(dev),
        prefiltered=False, debug=False, beta=0.0, if_contract=False, record_transmittance=False,
        max_intersections=0)
    hs = dsr.HashGridSettings(L=grid.levels, S=grid.S, H=grid.base_resolution, align_corners=False,
                              interpolation=0,
                              shape_dims=torch.tensor([0, grid.channels, grid.channels], dtype=torch.int32,
                                                      device=dev))
    rast = dsr.GaussianRasterizer(rs, hs)
    with torch.no_grad():
        _, _, allmap, _, _ = rast(
            means3D=state.means3D, means2D=torch.zeros(sc.P, 3, device=dev), opacities=state.opacities,
            shs=torch.zeros(sc.P, 1, 3, device=dev), scales=state.scales, rotations=state.rotations,
            homotrans=None, ap_level=state.ap_level, features=state.table, offsets=state.offsets,
            gridrange=state.gridrange, render_mode=0)
    allmap = allmap.cpu()
    alpha = allmap[1]
    assert (alpha == 0).any() and (alpha > 0.5).any()
    err, ref, g, gr = kernel_and_torch(allmap, cam)
    assert float((err - ref).abs().max()) < 2e-3
    check_grads(g, gr, alpha.cuda())


@pytest.mark.gpu
@pytest.mark.parametrize("ratio", [0.0, 1.0, 0.3])
def test_render_maps_match_torch(ratio):
    """ns_allmap_decode (the render_pkg maps) against the reference's torch
    expressions, including NaN / +inf median depths (nan_to_num -> 0)."""
    from nest_b200 import maps

    W, H = 120, 90
    cam = camera.orbit_camera(W, H, 55.0, azimuth_deg=15.0, elevation_deg=5.0)
    allmap = synthetic_allmap(W, H, 4)
    allmap[5, 0, 3] = float("nan")
    allmap[5, 0, 4] = float("inf")
    allmap[5, 40, 50] = float("nan")
    a = allmap.cuda()
    got = maps.render_maps(a, cam, ratio)
    ref = maps.render_maps_torch(a, cam, ratio)
    assert set(got) == set(ref)
    for k in ref:
        g, r = got[k], ref[k]
        assert g.shape == r.shape, k
        assert torch.isfinite(g).all(), k
        err = float((g - r).abs().max())
        assert err < 2e-3, (k, err)


@pytest.mark.gpu
@pytest.mark.parametrize("i", [0, 1])
def test_render_maps_surf_normal_matches_reference_point_utils(i):
    """surf_normal of ns_allmap_decode against utils/point_utils.py:48-60 run
    unmodified (tests/golden/reference_utils.npz): alpha 1, expected depth the
    golden surface. Same fp32 expressions, different evaluation order (the
    kernel forms rays and differences per pixel): max-abs 1e-4 on unit normals,
    the zero border exact."""
    import pathlib

    import numpy as np

    from nest_b200 import maps

    gold = np.load(pathlib.Path(__file__).resolve().parent / "golden" / "reference_utils.npz")
    W, H, fovx, fovy = gold[f"pu{i}_meta"][:4]
    W, H = int(W), int(H)
    cam = camera.make_camera(gold[f"pu{i}_R"], gold[f"pu{i}_t"], W, H, float(fovx), float(fovy))
    allmap = torch.zeros(14, H, W)
    allmap[0] = torch.tensor(gold[f"pu{i}_depth"][0])
    allmap[1] = 1.0
    allmap[5] = allmap[0]
    got = maps.render_maps(allmap.cuda(), cam, 0.0)["surf_normal"].permute(1, 2, 0).cpu().numpy()
    ref = gold[f"pu{i}_normal"]
    assert np.array_equal(got[0], ref[0]) and np.array_equal(got[-1], ref[-1])
    assert np.array_equal(got[:, 0], ref[:, 0]) and np.array_equal(got[:, -1], ref[:, -1])
    err = float(np.abs(got - ref).max())
    assert err < 1e-4, err
