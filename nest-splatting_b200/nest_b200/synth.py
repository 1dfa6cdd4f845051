"""Seeded synthetic scenes for the benchmark configurations.

No dataset or trained checkpoint exists on this machine, so every benchmark and
parity case runs on scenes drawn here. Draw order (one torch.Generator per
scene, CPU): surfel radii, directions, log-scales, quaternions, opacity logits,
hash table, MLP weights, then (RVQ scenes) codebooks and indices.

Surfels (benchmark config 1): means uniform in volume in the shell
0.8 <= r <= 1.2 (r = cbrt(U(0.8^3, 1.2^3)), direction = normalised N(0, I3)),
log-scales N(mean, std) on two axes, quaternions normalise(N(0, I4)), opacity
= sigmoid(N(0, 1.5)). Hash grid: L levels x 2^log2_T rows x LD features, rows
U(lo, hi) rounded to fp16, offsets 2^log2_T * l (gridencoder/grid.py:120-130),
base resolution 16, per-level scale 1.447. MLP: Xavier-uniform, no bias.
RVQ (config 0): codebook stage k ~ N(0, 1) * 0.5^k (0.5^k read as the standard
deviation), indices uniform u8.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch
import torch.nn.functional as F

from .camera import Camera, orbit_camera

ATTR_DIMS = 59  # mean 3 + log-scale 2 + quaternion 4 + opacity logit 1 + SH 48 + texture scale 1
BASE_DIMS = 10  # the geometric attributes the rasterizer consumes


@dataclass
class HashGrid:
    table: torch.Tensor        # [L*T, LD] fp16
    offsets: torch.Tensor      # [L+1] int32
    levels: int
    level_dim: int
    per_level_scale: float
    base_resolution: int
    align_corners: bool = False
    interpolation: int = 0
    gridrange: torch.Tensor = field(default_factory=lambda: torch.tensor([-1.5, 1.5]))

    @property
    def S(self) -> float:
        return math.log2(self.per_level_scale)

    @property
    def channels(self) -> int:
        return self.levels * self.level_dim


@dataclass
class Scene:
    base: torch.Tensor         # [P,10] raw attributes (xyz, log-scale, quaternion, opacity logit)
    grid: HashGrid
    mlp: list                  # fp16 weights [64,32], [64,64], [3,64]
    camera: Camera
    ap_level: torch.Tensor     # [P,1]
    codebooks: torch.Tensor | None = None  # [K,E,59] fp32
    rvq_idx: torch.Tensor | None = None    # [P,K] uint8
    mix: float = 0.0           # raw = base + mix * decoded[:, :10]

    @property
    def P(self) -> int:
        return self.base.shape[0]


def surfel_base(n: int, log_scale_mean: float, log_scale_std: float, g: torch.Generator) -> torch.Tensor:
    u = torch.rand(n, generator=g) * (1.2 ** 3 - 0.8 ** 3) + 0.8 ** 3
    r = u.pow(1.0 / 3.0)
    d = torch.randn(n, 3, generator=g)
    d = d / d.norm(dim=1, keepdim=True)
    xyz = d * r[:, None]
    log_scale = torch.randn(n, 2, generator=g) * log_scale_std + log_scale_mean
    quat = torch.randn(n, 4, generator=g)
    opacity_logit = torch.randn(n, 1, generator=g) * 1.5
    return torch.cat([xyz, log_scale, quat, opacity_logit], dim=1).float().contiguous()


def activate(raw: torch.Tensor):
    """gaussian_model.py:231-281 activations on raw [P,10] attributes."""
    means = raw[:, 0:3].contiguous()
    scales = torch.exp(raw[:, 3:5]).contiguous()
    rotations = F.normalize(raw[:, 5:9], dim=-1).contiguous()
    opacities = torch.sigmoid(raw[:, 9:10]).contiguous()
    return means, scales, rotations, opacities


def build_rotation(r: torch.Tensor) -> torch.Tensor:
    """general_utils.py:78-99 (device-agnostic restatement)."""
    norm = torch.sqrt(r[:, 0] * r[:, 0] + r[:, 1] * r[:, 1] + r[:, 2] * r[:, 2] + r[:, 3] * r[:, 3])
    q = r / norm[:, None]
    R = torch.zeros((q.size(0), 3, 3), device=r.device)
    w, x, y, z = q[:, 0], q[:, 1], q[:, 2], q[:, 3]
    R[:, 0, 0] = 1 - 2 * (y * y + z * z)
    R[:, 0, 1] = 2 * (x * y - w * z)
    R[:, 0, 2] = 2 * (x * z + w * y)
    R[:, 1, 0] = 2 * (x * y + w * z)
    R[:, 1, 1] = 1 - 2 * (x * x + z * z)
    R[:, 1, 2] = 2 * (y * z - w * x)
    R[:, 2, 0] = 2 * (x * z - w * y)
    R[:, 2, 1] = 2 * (y * z + w * x)
    R[:, 2, 2] = 1 - 2 * (x * x + y * y)
    return R


def build_homotrans(raw: torch.Tensor) -> torch.Tensor:
    """gaussian_model.py:312-317 get_homotrans -> general_utils.py:101-113 build_H, as [P,16]."""
    rots = build_rotation(raw[:, 5:9])
    scales = torch.exp(raw[:, 3:5])
    n = raw.shape[0]
    s = torch.zeros(n, 1, 3, device=raw.device)
    s[:, 0, :2] = scales
    h = torch.zeros(n, 4, 4, device=raw.device)
    h[:, :3, :3] = s * rots
    h[:, :3, 3] = raw[:, 0:3]
    h[:, 3, 3] = 1.0
    return h.reshape(n, 16).contiguous()


def hash_grid(g: torch.Generator, levels: int = 16, log2_T: int = 19, level_dim: int = 2,
              lo: float = -1e-4, hi: float = 1e-4, base_resolution: int = 16,
              per_level_scale: float = 1.447) -> HashGrid:
    T = 1 << log2_T
    table = (torch.rand(levels * T, level_dim, generator=g) * (hi - lo) + lo).half().contiguous()
    offsets = (torch.arange(levels + 1, dtype=torch.int64) * T).to(torch.int32)
    return HashGrid(table, offsets, levels, level_dim, per_level_scale, base_resolution)


def xavier_mlp(g: torch.Generator, dims=(32, 64, 64, 3)) -> list:
    ws = []
    for fan_in, fan_out in zip(dims[:-1], dims[1:]):
        b = math.sqrt(6.0 / (fan_in + fan_out))
        ws.append(((torch.rand(fan_out, fan_in, generator=g) * 2 - 1) * b).half().contiguous())
    return ws


def rvq_codebooks(g: torch.Generator, stages: int = 6, entries: int = 256, dims: int = ATTR_DIMS) -> torch.Tensor:
    cb = torch.randn(stages, entries, dims, generator=g)
    scale = torch.tensor([0.5 ** k for k in range(stages)]).view(stages, 1, 1)
    return (cb * scale).float().contiguous()


def rvq_indices(g: torch.Generator, n: int, stages: int = 6, entries: int = 256) -> torch.Tensor:
    return torch.randint(0, entries, (n, stages), generator=g, dtype=torch.int64).to(torch.uint8).contiguous()


def config0(n: int = 200_000, seed: int = 0):
    """RVQ decode workload: (codebooks [6,256,59] fp32, idx [n,6] u8)."""
    g = torch.Generator().manual_seed(seed)
    cb = rvq_codebooks(g)
    idx = rvq_indices(g, n)
    return cb, idx


def make_scene(n: int, log_scale_mean: float, log_scale_std: float, width: int, height: int,
               fovx_deg: float, seed: int, rvq: bool = False, table_range: float = 1e-4,
               fovy_deg: float | None = None, levels: int = 16, log2_T: int = 19,
               mix: float = 1e-3) -> Scene:
    g = torch.Generator().manual_seed(seed)
    base = surfel_base(n, log_scale_mean, log_scale_std, g)
    grid = hash_grid(g, levels=levels, log2_T=log2_T, lo=-table_range, hi=table_range)
    mlp = xavier_mlp(g, (levels * 2, 64, 64, 3))
    cam = orbit_camera(width, height, fovx_deg, fovy_deg=fovy_deg)
    ap = torch.full((n, 1), 24.0)
    sc = Scene(base, grid, mlp, cam, ap)
    if rvq:
        sc.codebooks = rvq_codebooks(g)
        sc.rvq_idx = rvq_indices(g, n)
        sc.mix = mix
    return sc


def config1(n: int = 200_000, width: int = 800, height: int = 800, table_range: float = 1e-4,
            seed: int = 1) -> Scene:
    return make_scene(n, -4.0, 0.5, width, height, 50.0, seed, fovy_deg=50.0 if width == height else None,
                      table_range=table_range)


def config2(n: int = 1_000_000, width: int = 1297, height: int = 840, table_range: float = 1e-4,
            seed: int = 2) -> Scene:
    return make_scene(n, -4.6, 0.5, width, height, 60.0, seed, rvq=True, table_range=table_range)


def config3_cameras(count: int = 64, width: int = 1920, height: int = 1080, elevation_deg: float = 20.0):
    return [orbit_camera(width, height, 60.0, 4.0, 360.0 * i / count, elevation_deg) for i in range(count)]


def config3(n: int = 3_000_000, table_range: float = 1e-4, seed: int = 3) -> Scene:
    return make_scene(n, -5.0, 0.6, 1920, 1080, 60.0, seed, rvq=True, table_range=table_range)
