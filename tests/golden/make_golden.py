"""Generates tests/golden/reference_utils.npz from the reference's own Python code.

Run in a container where the reference checkout is importable:
    python tests/golden/make_golden.py /path/to/nest-splatting

It imports, unmodified:
  * utils/graphics_utils.py: getWorld2View2, getProjectionMatrix, focal2fov,
    fov2focal -> camera matrices exactly as scene/cameras.py:63-66 builds them;
  * utils/general_utils.py: build_rotation, build_H -> homotrans of
    gaussian_model.py:312-317 (get_homotrans).
build_rotation / build_H hard-code device='cuda'; with no GPU in the generating
container they are run on CPU by redirecting torch.zeros(device='cuda') and
Tensor.cuda() to CPU for the duration of the call (arithmetic unchanged).
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
    real_cuda = torch.Tensor.cuda

    def zeros(*a, **k):
        k.pop("device", None)
        return real_zeros(*a, **k)

    torch.zeros = zeros
    torch.Tensor.cuda = lambda self, *a, **k: self

    def undo():
        torch.zeros = real_zeros
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
    np.savez(OUT, **data)
    print("wrote", OUT)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python make_golden.py <path to the reference repository checkout>")
    main(sys.argv[1])
