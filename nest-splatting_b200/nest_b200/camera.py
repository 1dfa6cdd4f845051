"""Pinhole cameras in the reference's conventions.

Restates utils/graphics_utils.py:38-71 (getWorld2View2, getProjectionMatrix,
fov2focal, focal2fov) and scene/cameras.py:17-83 (Camera / MiniCam tensors):
world_view_transform and full_proj_transform are stored transposed
("row-vector" layout), which is what the rasterizer kernels index.
Camera axes follow COLMAP/OpenCV: x right, y down, z forward.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np
import torch


def fov2focal(fov: float, pixels: int) -> float:
    return pixels / (2 * math.tan(fov / 2))


def focal2fov(focal: float, pixels: int) -> float:
    return 2 * math.atan(pixels / (2 * focal))


def world_to_view(R: np.ndarray, t: np.ndarray) -> np.ndarray:
    """getWorld2View2 with translate 0 and scale 1: R is camera-to-world rotation."""
    Rt = np.zeros((4, 4))
    Rt[:3, :3] = R.transpose()
    Rt[:3, 3] = t
    Rt[3, 3] = 1.0
    C2W = np.linalg.inv(Rt)
    Rt = np.linalg.inv(C2W)
    return np.float32(Rt)


def projection_matrix(znear: float, zfar: float, fovx: float, fovy: float) -> torch.Tensor:
    """getProjectionMatrix (column-vector convention, z in [0, 1])."""
    tan_y = math.tan(fovy / 2)
    tan_x = math.tan(fovx / 2)
    top = tan_y * znear
    bottom = -top
    right = tan_x * znear
    left = -right
    P = torch.zeros(4, 4)
    P[0, 0] = 2.0 * znear / (right - left)
    P[1, 1] = 2.0 * znear / (top - bottom)
    P[0, 2] = (right + left) / (right - left)
    P[1, 2] = (top + bottom) / (top - bottom)
    P[3, 2] = 1.0
    P[2, 2] = zfar / (zfar - znear)
    P[2, 3] = -(zfar * znear) / (zfar - znear)
    return P


@dataclass
class Camera:
    width: int
    height: int
    fovx: float
    fovy: float
    znear: float
    zfar: float
    world_view_transform: torch.Tensor  # [4,4] float32, transposed W2C
    full_proj_transform: torch.Tensor   # [4,4] float32
    camera_center: torch.Tensor         # [3]

    @property
    def tanfovx(self) -> float:
        return math.tan(self.fovx * 0.5)

    @property
    def tanfovy(self) -> float:
        return math.tan(self.fovy * 0.5)

    def to(self, device) -> "Camera":
        return Camera(self.width, self.height, self.fovx, self.fovy, self.znear, self.zfar,
                      self.world_view_transform.to(device), self.full_proj_transform.to(device),
                      self.camera_center.to(device))


def make_camera(R_c2w: np.ndarray, t: np.ndarray, width: int, height: int, fovx: float,
                fovy: float, znear: float = 0.2, zfar: float = 100.0) -> Camera:
    """Camera tensors exactly as scene/cameras.py:63-66 builds them."""
    wv = torch.tensor(world_to_view(R_c2w, t)).transpose(0, 1)
    proj = projection_matrix(znear, zfar, fovx, fovy).transpose(0, 1)
    full = wv.unsqueeze(0).bmm(proj.unsqueeze(0)).squeeze(0)
    center = wv.inverse()[3, :3]
    return Camera(width, height, fovx, fovy, znear, zfar, wv.contiguous(), full.contiguous(), center)


def look_at(eye, target=(0.0, 0.0, 0.0), up=(0.0, 0.0, 1.0)):
    """(R_c2w, t) of a camera at `eye` looking at `target` (x right, y down, z forward)."""
    eye = np.asarray(eye, dtype=np.float64)
    f = np.asarray(target, dtype=np.float64) - eye
    f /= np.linalg.norm(f)
    right = np.cross(f, np.asarray(up, dtype=np.float64))
    right /= np.linalg.norm(right)
    down = np.cross(f, right)
    R_w2c = np.stack([right, down, f], axis=0)
    t = -R_w2c @ eye
    return R_w2c.T, t


def orbit_camera(width: int, height: int, fovx_deg: float, radius: float = 4.0,
                 azimuth_deg: float = 0.0, elevation_deg: float = 0.0, fovy_deg: float | None = None,
                 znear: float = 0.2, zfar: float = 100.0) -> Camera:
    """Camera on a sphere around the origin, world up +z; azimuth 0 is the -y axis.

    fovy defaults to the value with the same focal length as fovx (square pixels).
    """
    az, el = math.radians(azimuth_deg), math.radians(elevation_deg)
    eye = (radius * math.cos(el) * math.sin(az), -radius * math.cos(el) * math.cos(az),
           radius * math.sin(el))
    R, t = look_at(eye)
    fovx = math.radians(fovx_deg)
    fovy = math.radians(fovy_deg) if fovy_deg is not None else focal2fov(fov2focal(fovx, width), height)
    return make_camera(R, t, width, height, fovx, fovy, znear, zfar)
