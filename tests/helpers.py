"""Shared helpers: scene -> rasterizer inputs, oracle runs, comparisons."""
from __future__ import annotations

import numpy as np
import torch

from nest_b200 import synth
from oracle import oracle


def raw_attributes(scene: synth.Scene, decoded: torch.Tensor | None = None) -> torch.Tensor:
    """raw [P,10] = base + mix * decoded[:, :10] (RVQ scenes) or base."""
    if decoded is None:
        return scene.base
    return (scene.base + np.float32(scene.mix) * decoded[:, :10].cpu()).float()


def api_inputs(scene: synth.Scene, raw: torch.Tensor | None = None):
    """Activated tensors as render() passes them to the rasterizer (CPU float32)."""
    raw = scene.base if raw is None else raw
    means, scales, rots, opac = synth.activate(raw)
    homo = synth.build_homotrans(raw)
    return dict(means3D=means, scales=scales, rotations=rots, opacities=opac, homotrans=homo,
                ap_level=scene.ap_level)


def oracle_render(scene: synth.Scene, inputs: dict, **kw):
    g = scene.grid
    cam = scene.camera
    out, pre, n = oracle.forward(inputs["means3D"].numpy(), inputs["scales"].numpy(), inputs["rotations"].numpy(),
                                 inputs["opacities"].numpy(), inputs["homotrans"].numpy(),
                                 inputs["ap_level"].numpy(), g.table.float().numpy(), g.offsets.numpy(),
                                 g.gridrange.numpy(), cam.world_view_transform.numpy(),
                                 cam.full_proj_transform.numpy(), cam.width, cam.height, g.channels,
                                 g.level_dim, g.levels, g.S, g.base_resolution, **kw)
    return out, pre, n


def small_scene(n=2000, width=100, height=70, table_range=1.0, seed=11, log_scale=-2.6, rvq=False):
    return synth.make_scene(n, log_scale, 0.5, width, height, 50.0, seed, rvq=rvq, table_range=table_range,
                            log2_T=14, mix=1e-3)


def psnr(a: np.ndarray, b: np.ndarray, peak: float = 1.0) -> float:
    mse = float(np.mean((np.asarray(a, np.float64) - np.asarray(b, np.float64)) ** 2))
    return float("inf") if mse == 0 else 10 * np.log10(peak * peak / mse)
