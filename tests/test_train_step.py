"""Config 4 (one training step): the host glue on CPU, and on the GPU the whole
step's rasterizer gradients against the CPU oracle fed with the same upstream
gradients, plus the MLP backward against torch autograd of the same network."""
import numpy as np
import pytest
import torch

import diff_surfel_rasterization as dsr
from nest_b200 import camera, train


def test_depth_to_normal_recovers_a_plane():
    cam = camera.orbit_camera(64, 48, 60.0)
    # Points of the world plane y = 0 (the camera sits at y = -4 looking along +y):
    # depth along each pixel ray d with o + t d on the plane.
    wv = cam.world_view_transform
    c2w = wv.T.inverse()
    ndc2pix = torch.tensor([[32.0, 0, 0, 32.0], [0, 24.0, 0, 24.0], [0, 0, 0, 1]]).T
    intr = ((c2w.T @ cam.full_proj_transform) @ ndc2pix)[:3, :3].T
    gx, gy = torch.meshgrid(torch.arange(64.0), torch.arange(48.0), indexing="xy")
    pix = torch.stack([gx, gy, torch.ones_like(gx)], -1).reshape(-1, 3)
    d = pix @ intr.inverse().T @ c2w[:3, :3].T
    o = c2w[:3, 3]
    t = (0.0 - o[1]) / d[:, 1]
    depth = t.reshape(1, 48, 64)
    n = train.depth_to_normal(cam, depth)
    inner = n[1:-1, 1:-1].reshape(-1, 3)
    assert torch.allclose(inner.abs(), torch.tensor([0.0, 1.0, 0.0]).expand_as(inner), atol=1e-3)
    assert torch.all(n[0] == 0) and torch.all(n[:, -1] == 0)


def test_decode_allmap_expected_depth_and_world_normal():
    cam = camera.orbit_camera(32, 24, 60.0)
    allmap = torch.zeros(14, 24, 32)
    allmap[1] = 0.5
    allmap[0] = 1.5  # depth * alpha
    allmap[2:5] = torch.tensor([0.0, 0.0, -0.5]).view(3, 1, 1)  # view-space normal * alpha
    alpha, rn, sn, depth = train.decode_allmap(allmap, cam)
    assert torch.allclose(depth, torch.full_like(depth, 3.0))
    # view -z (towards the camera) is world -y for the orbit camera at azimuth 0
    assert torch.allclose(rn[:, 5, 5], torch.tensor([0.0, -0.5, 0.0]), atol=1e-6)
    allmap[1] = 0.0
    _, _, _, depth0 = train.decode_allmap(allmap, cam)
    assert torch.all(depth0 == 0)  # NaN / inf from 0 / 0 -> 0


@pytest.mark.gpu
def test_train_step_gradients_match_oracle():
    from helpers import small_scene
    from test_gpu_backward import check_all, oracle_grads

    sc = small_scene(seed=21, table_range=1e-4)
    state = train.make_state(sc)
    cam, g = sc.camera, sc.grid
    dev = "cuda"
    rs = dsr.GaussianRasterizationSettings(
        image_height=cam.height, image_width=cam.width, tanfovx=cam.tanfovx, tanfovy=cam.tanfovy,
        bg=torch.zeros(3, device=dev), scale_modifier=1.0, viewmatrix=cam.world_view_transform.to(dev),
        projmatrix=cam.full_proj_transform.to(dev), sh_degree=0, campos=cam.camera_center.to(dev),
        prefiltered=False, debug=False, beta=0.0, if_contract=False, record_transmittance=False,
        max_intersections=0)
    hs = dsr.HashGridSettings(L=g.levels, S=g.S, H=g.base_resolution, align_corners=False, interpolation=0,
                              shape_dims=torch.tensor([0, g.channels, g.channels], dtype=torch.int32, device=dev))
    rast = dsr.GaussianRasterizer(rs, hs)
    for t in state.leaves():
        t.grad = None
    loss, rgb, allmap = train.forward(state, rast, cam, keep_upstream=True)
    loss.backward()
    assert np.isfinite(float(loss.detach()))
    for t in state.leaves():
        assert t.grad is not None and torch.isfinite(t.grad).all()

    # The rasterizer's gradients vs the oracle fed with the same upstream gradients.
    up_color = state.extra["color"].grad.detach().cpu()
    up_allmap = state.extra["allmap"].grad.detach().cpu()
    assert up_color.abs().sum() > 0 and up_allmap[2:5].abs().sum() > 0
    from nest_b200 import synth
    inputs = dict(means3D=state.means3D.detach().cpu(), scales=state.scales.detach().cpu(),
                  rotations=state.rotations.detach().cpu(), opacities=state.opacities.detach().cpu().reshape(-1, 1),
                  ap_level=state.ap_level.cpu())
    R = synth.build_rotation(inputs["rotations"])
    homo = torch.zeros(sc.P, 4, 4)
    homo[:, :3, 0] = R[:, :, 0] * inputs["scales"][:, 0:1]
    homo[:, :3, 1] = R[:, :, 1] * inputs["scales"][:, 1:2]
    homo[:, :3, 3] = inputs["means3D"]
    homo[:, 3, 3] = 1
    inputs["homotrans"] = homo.reshape(-1, 16)
    sc.grid.table = state.table.detach().cpu().half()  # the fp32 leaf holds the fp16 values
    ref, _ = oracle_grads(sc, inputs, up_color, up_allmap)
    exact, _ = oracle_grads(sc, inputs, up_color, up_allmap, f64=True)
    got = {"means3D": state.means3D.grad, "scales": state.scales.grad, "rotations": state.rotations.grad,
           "opacity": state.opacities.grad, "table": state.table.grad, "means2D": state.extra["means2D"].grad}
    got = {k: v.detach().cpu().numpy() for k, v in got.items()}
    got["gradsum"] = ref["g"]["dL_gradsum"]  # returned in ap_level's slot; ap_level is not a leaf here
    check_all(got, ref, exact)


@pytest.mark.gpu
@pytest.mark.parametrize("H,W,scale", [(40, 56, 1.0), (37, 53, 1e-7), (2, 5, 1.0)])
def test_mlp_backward_matches_torch_autograd(H, W, scale):
    """The fused MLP backward (ns_mlp_backward) against torch autograd of the same
    network on fp16-rounded operands, in fp32; scale 1e-7 is the size of a mean
    loss's per-pixel gradient over a megapixel image (below fp16's normal range)."""
    g = torch.Generator().manual_seed(3)
    feat = (torch.rand(32, H, W, generator=g) * 2 - 1).cuda().requires_grad_(True)
    alpha = (torch.rand(H, W, generator=g)).cuda()
    alpha[::7] = 0.0
    ws = [((torch.rand(o, i, generator=g) * 2 - 1) * (6 / (i + o)) ** 0.5).cuda().requires_grad_(True)
          for i, o in ((32, 64), (64, 64), (64, 3))]
    up = torch.randn(3, H, W, generator=g).cuda() * scale
    rgb = train.mlp(feat, *ws, alpha)
    (rgb * up).sum().backward()
    got = [feat.grad] + [w.grad for w in ws]
    # torch fp32 reference of the same network on fp16-rounded operands; the
    # roundings pass gradients through unchanged (autograd through .half() would
    # round the gradients to fp16 too, and flush the 1e-7-scale case to zero)
    def r16(t):
        return t + (t.half().float() - t).detach()

    f2 = feat.detach().clone().requires_grad_(True)
    w2 = [w.detach().clone().requires_grad_(True) for w in ws]
    x = r16(f2.reshape(32, -1).T)
    h = x
    for i, w in enumerate(w2):
        h = h @ r16(w).T
        h = r16(h) if i == 2 else r16(torch.relu(h))
    ref_rgb = torch.sigmoid(h[:, :3]).T.reshape(3, H, W) * (alpha > 0).float()
    assert torch.allclose(ref_rgb, rgb, atol=2e-3)
    (ref_rgb * up).sum().backward()
    for a, b in zip(got, [f2.grad] + [w.grad for w in w2]):
        rel = (a - b).norm() / b.norm()
        assert rel < 1e-2, float(rel)
