"""Generates tests/golden/reference_utils.npz from the reference's own Python code.

Run in a container where the reference checkout is importable:
    python tests/golden/make_golden.py /path/to/nest-splatting

It imports, unmodified:
  * utils/graphics_utils.py: getWorld2View2, getProjectionMatrix, focal2fov,
    fov2focal -> camera matrices exactly as scene/cameras.py:63-66 builds them;
  * utils/general_utils.py: build_rotation, build_H -> homotrans of
    gaussian_model.py:312-317 (get_homotrans);
  * utils/point_utils.py: depths_to_points, depth_to_normal -> the per-pixel
    rays, world points and surf_normal of the render_pkg decode
    (gaussian_renderer/__init__.py:789-792), on two small cameras;
  * utils/sh_utils.py: eval_sh -> the SH colour basis (degrees 0-3) of 64
    surfels seen from one camera centre, the sum the rasterizer's
    computeColorFromSH forms before its + 0.5 and clamp.
These functions hard-code device='cuda'; with no GPU in the generating
container they are run on CPU by redirecting torch.zeros / torch.arange
(device='cuda') and Tensor.cuda() to CPU for the duration of the call
(arithmetic unchanged). point_utils imports matplotlib for its plotting
helpers only; where matplotlib is absent an empty module stands in for it.
The fixture is committed; tests never import the reference.
"""
from __future__ import annotations

import math
import sys
from pathlib import Path

import numpy as np
import torch

OUT = Path(__file__).resolve().parent / "reference_utils.npz"


def _cpu_cuda_shim():
    real_zeros = torch.zeros
    real_arange = torch.arange
    real_cuda = torch.Tensor.cuda

    def zeros(*a, **k):
        k.pop("device", None)
        return real_zeros(*a, **k)

    def arange(*a, **k):
        k.pop("device", None)
        return real_arange(*a, **k)

    torch.zeros = zeros
    torch.arange = arange
    torch.Tensor.cuda = lambda self, *a, **k: self

    def undo():
        torch.zeros = real_zeros
        torch.arange = real_arange
        torch.Tensor.cuda = real_cuda

    return undo


def look_at(eye):
    eye = np.asarray(eye, dtype=np.float64)
    f = -eye / np.linalg.norm(eye)
    right = np.cross(f, np.array([0.0, 0.0, 1.0]))
    right /= np.linalg.norm(right)
    down = np.cross(f, right)
    R_w2c = np.stack([right, down, f], 0)
    return R_w2c.T, -R_w2c @ eye


def main(ref_root: str) -> None:
    sys.path.insert(0, ref_root)
    from utils import general_utils as gu  # noqa: E402
    from utils import graphics_utils as gr  # noqa: E402

    data = {}
    # Cameras: config 1 (800x800, 50 deg), config 2 (1297x840, fovx 60), one config-3 orbit view.
    cams = [
        (800, 800, math.radians(50.0), math.radians(50.0), (0.0, -4.0, 0.0)),
        (1297, 840, math.radians(60.0), None, (0.0, -4.0, 0.0)),
        (1920, 1080, math.radians(60.0), None,
         (4 * math.cos(math.radians(20)) * math.sin(math.radians(45)),
          -4 * math.cos(math.radians(20)) * math.cos(math.radians(45)), 4 * math.sin(math.radians(20)))),
    ]
    for i, (W, H, fovx, fovy, eye) in enumerate(cams):
        if fovy is None:
            fovy = gr.focal2fov(gr.fov2focal(fovx, W), H)
        R, t = look_at(eye)
        wv = torch.tensor(gr.getWorld2View2(R, t, np.array([0.0, 0.0, 0.0]), 1.0)).transpose(0, 1)
        proj = gr.getProjectionMatrix(znear=0.2, zfar=100.0, fovX=fovx, fovY=fovy).transpose(0, 1)
        full = wv.unsqueeze(0).bmm(proj.unsqueeze(0)).squeeze(0)
        center = wv.inverse()[3, :3]
        data[f"cam{i}_meta"] = np.array([W, H, fovx, fovy, *eye], np.float64)
        data[f"cam{i}_R"] = R
        data[f"cam{i}_t"] = t
        data[f"cam{i}_view"] = wv.numpy()
        data[f"cam{i}_full"] = full.numpy()
        data[f"cam{i}_center"] = center.numpy()

    # homotrans of 64 random surfels (raw quaternion, log-scale, mean).
    g = torch.Generator().manual_seed(123)
    raw_q = torch.randn(64, 4, generator=g)
    log_s = torch.randn(64, 2, generator=g) * 0.5 - 4.0
    xyz = torch.randn(64, 3, generator=g)
    undo = _cpu_cuda_shim()
    try:
        rots = gu.build_rotation(raw_q)
        H = gu.build_H(rots, torch.exp(log_s), xyz)
    finally:
        undo()
    data["homo_q"] = raw_q.numpy()
    data["homo_log_s"] = log_s.numpy()
    data["homo_xyz"] = xyz.numpy()
    data["homo_H"] = H.reshape(64, 16).numpy()

    # point_utils on two small cameras (one odd-sized) and a smooth depth surface.
    try:
        import matplotlib.pyplot  # noqa: F401
    except ImportError:
        import types
        mpl = types.ModuleType("matplotlib")
        mpl.pyplot = types.ModuleType("matplotlib.pyplot")
        sys.modules["matplotlib"] = mpl
        sys.modules["matplotlib.pyplot"] = mpl.pyplot
    from utils import point_utils as pu  # noqa: E402
    from types import SimpleNamespace

    for i, (W, H, fovx, eye) in enumerate([(64, 48, math.radians(50.0), (0.3, -4.0, 0.8)),
                                            (37, 23, math.radians(70.0), (2.5, -2.0, 1.5))]):
        fovy = gr.focal2fov(gr.fov2focal(fovx, W), H)
        R, t = look_at(eye)
        wv = torch.tensor(gr.getWorld2View2(R, t, np.array([0.0, 0.0, 0.0]), 1.0)).transpose(0, 1)
        proj = gr.getProjectionMatrix(znear=0.2, zfar=100.0, fovX=fovx, fovY=fovy).transpose(0, 1)
        full = wv.unsqueeze(0).bmm(proj.unsqueeze(0)).squeeze(0)
        view = SimpleNamespace(world_view_transform=wv, full_proj_transform=full, image_width=W, image_height=H)
        ys, xs = torch.meshgrid(torch.linspace(0, 1, H), torch.linspace(0, 1, W), indexing="ij")
        depth = (3.5 + 0.7 * xs - 0.5 * ys + 0.08 * torch.sin(11 * xs) * torch.cos(5 * ys))[None].float()
        undo = _cpu_cuda_shim()
        try:
            points, rays_d, rays_o = pu.depths_to_points(view, depth)
            normal = pu.depth_to_normal(view, depth)
        finally:
            undo()
        data[f"pu{i}_meta"] = np.array([W, H, fovx, fovy, *eye], np.float64)
        data[f"pu{i}_R"] = R
        data[f"pu{i}_t"] = t
        data[f"pu{i}_depth"] = depth.numpy()
        data[f"pu{i}_rays_d"] = rays_d.numpy()
        data[f"pu{i}_rays_o"] = rays_o.numpy()
        data[f"pu{i}_points"] = points.numpy()
        data[f"pu{i}_normal"] = normal.numpy()
    # SH colours: GaussianModel's features [N, 16, 3] (DC then rest), viewed as the
    # renderer does for eval_sh ([N, 3, 16]), along the unit direction camera -> mean.
    from utils import sh_utils  # noqa: E402
    g = torch.Generator().manual_seed(321)
    shs = torch.randn(64, 16, 3, generator=g) * 0.6
    means = torch.randn(64, 3, generator=g)
    campos = torch.tensor([0.3, -4.0, 0.8])
    dirs = means - campos
    dirs = dirs / dirs.norm(dim=1, keepdim=True)
    data["sh_shs"] = shs.numpy()
    data["sh_means"] = means.numpy()
    data["sh_campos"] = campos.numpy()
    for deg in range(4):
        data[f"sh_eval_deg{deg}"] = sh_utils.eval_sh(deg, shs.transpose(1, 2), dirs).numpy()
    np.savez(OUT, **data)
    print("wrote", OUT)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python make_golden.py <path to the reference repository checkout>")
    main(sys.argv[1])
