"""Camera and homotrans construction against golden vectors produced by the
reference's own Python code (tests/golden/make_golden.py imports
utils/graphics_utils.py and utils/general_utils.py unmodified)."""
import pathlib

import numpy as np
import torch

from nest_b200 import camera as camlib
from nest_b200 import synth

GOLD = np.load(pathlib.Path(__file__).resolve().parent / "golden" / "reference_utils.npz")


def test_camera_matrices_match_reference():
    for i in range(3):
        W, H, fovx, fovy = GOLD[f"cam{i}_meta"][:4]
        R, t = GOLD[f"cam{i}_R"], GOLD[f"cam{i}_t"]
        cam = camlib.make_camera(R, t, int(W), int(H), float(fovx), float(fovy))
        assert np.array_equal(cam.world_view_transform.numpy(), GOLD[f"cam{i}_view"])
        assert np.array_equal(cam.full_proj_transform.numpy(), GOLD[f"cam{i}_full"])
        assert np.allclose(cam.camera_center.numpy(), GOLD[f"cam{i}_center"], atol=1e-6)


def test_orbit_camera_matches_reference_look_at():
    # config-3 style orbit view (azimuth 45, elevation 20) and config 2's camera
    cam = camlib.orbit_camera(1920, 1080, 60.0, 4.0, 45.0, 20.0)
    assert np.allclose(cam.world_view_transform.numpy(), GOLD["cam2_view"], atol=1e-6)
    assert np.allclose(cam.full_proj_transform.numpy(), GOLD["cam2_full"], atol=1e-5)
    cam = camlib.orbit_camera(1297, 840, 60.0)
    assert np.allclose(cam.full_proj_transform.numpy(), GOLD["cam1_full"], atol=1e-6)
    assert abs(cam.fovy - GOLD["cam1_meta"][3]) < 1e-12


def test_homotrans_matches_reference_build_H():
    raw = torch.cat([torch.tensor(GOLD["homo_xyz"]), torch.tensor(GOLD["homo_log_s"]),
                     torch.tensor(GOLD["homo_q"]), torch.zeros(64, 1)], 1)
    H = synth.build_homotrans(raw).numpy()
    assert np.array_equal(H, GOLD["homo_H"])


def _pu_camera(i):
    W, H, fovx, fovy = GOLD[f"pu{i}_meta"][:4]
    return camlib.make_camera(GOLD[f"pu{i}_R"], GOLD[f"pu{i}_t"], int(W), int(H), float(fovx), float(fovy))


def test_depth_to_normal_matches_reference_point_utils():
    """nest_b200.train's rays, world points and normals against utils/point_utils.py:10-30,48-60
    run unmodified (fp32 on CPU): the same expressions in the same order, so bit-equal."""
    from nest_b200 import train
    for i in range(2):
        cam = _pu_camera(i)
        depth = torch.tensor(GOLD[f"pu{i}_depth"])
        rays_d, rays_o = train._camera_rays(cam, depth.device)
        assert np.array_equal(rays_d.numpy(), GOLD[f"pu{i}_rays_d"])
        assert np.array_equal(rays_o.numpy(), GOLD[f"pu{i}_rays_o"])
        assert np.array_equal(train.depths_to_points(cam, depth).numpy(), GOLD[f"pu{i}_points"])
        assert np.array_equal(train.depth_to_normal(cam, depth).numpy(), GOLD[f"pu{i}_normal"])


def test_oracle_sh_color_matches_reference_eval_sh():
    """The oracle's computeColorFromSH (forward.cu:21-74) against the reference's
    own utils/sh_utils.py eval_sh (tests/golden/make_golden.py), degrees 0-3:
    the same basis and sum, then + 0.5 and the clamp at 0."""
    from oracle import oracle
    shs, means, campos = GOLD["sh_shs"], GOLD["sh_means"], GOLD["sh_campos"]
    for deg in range(4):
        got = oracle.sh_color(means, campos, shs, deg)
        want = np.maximum(GOLD[f"sh_eval_deg{deg}"] + 0.5, 0.0)
        assert np.abs(got - want).max() < 2e-6, (deg, np.abs(got - want).max())
        assert (GOLD[f"sh_eval_deg{deg}"] + 0.5 < 0).any() or deg == 0  # the clamp is exercised
