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


def compare(out, got_color, got_allmap, tol=2e-3, max_bad_frac=1e-3, rows=None, feat_tol=None):
    """max-abs <= tol per channel (features, depth, alpha, normal, median depth,
    distortion, position) on at least 99.9% of the pixels, and PSNR >= 60 dB.

    The remaining pixels are threshold decisions that flip between the CPU and
    GPU float evaluation (FMA contraction and expf ulps differ): a sample at
    alpha = 1/255 or T = 1e-4 kept on one side and dropped on the other (the
    count channel differs there), or the hit point switching between the
    surfel plane and its centre at rho3d == rho2d (forward.cu:855-857, 1102-1109),
    which moves the hash lookup to another position. Both are discrete events
    of probability ~1e-4 per pixel; a systematic error fails the 99.9% bound.

    rows: optional pixel-row selection (e.g. the tile rows a sampled oracle
    render covered); only those rows are compared. feat_tol: tolerance of the
    feature channels when it must differ from tol (a table of small entries
    needs one scaled to its magnitude, or any error would pass)."""
    ref_c, ref_o = out["out_color"], out["out_others"]
    if rows is not None:
        ref_c, ref_o = ref_c[:, rows], ref_o[:, rows]
        got_color, got_allmap = got_color[:, rows], got_allmap[:, rows]
    npx = ref_c.shape[1] * ref_c.shape[2]
    flips = got_allmap[7] != ref_o[7]
    assert flips.mean() <= max_bad_frac, ("count flips", flips.mean())
    err_c = np.abs(got_color - ref_c).max(axis=0)
    ft = tol if feat_tol is None else feat_tol
    assert (err_c > ft).sum() <= max(1, int(max_bad_frac * npx)), ("features", (err_c > ft).sum(), err_c.max())
    for ch in range(14):
        if ch == 7:
            continue
        err = np.abs(got_allmap[ch] - ref_o[ch])
        scale = max(1.0, np.abs(ref_o[ch]).max())
        assert (err > tol * scale).sum() <= max(1, int(max_bad_frac * npx)), (ch, err.max())
    assert psnr(got_color, ref_c, peak=max(1.0, np.abs(ref_c).max())) >= 60
    assert psnr(got_allmap[1], ref_o[1]) >= 60
