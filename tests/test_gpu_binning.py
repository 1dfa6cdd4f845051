"""Tile binning, checked instance by instance.

The reference emits one instance per tile of a surfel's getRect rectangle
(rasterizer_impl.cu:70-111, auxiliary.h:72-82), key (tile << 32 | depth bits),
sorts the keys stably (:381-386) and records each tile's [start, end)
(:173-195). This build emits only the tiles that meet the surfel's alpha >=
1/255 box (pixels outside it can only see alpha < 1/255 and skip the surfel).
So, exactly:
  * the GPU point list equals the reference list restricted to the instances
    whose tile lies in the surfel's cut rectangle, in the reference's order,
    and the tile ranges are that list's ranges (the reference's emission and
    stable sort are run here in numpy / the C++ oracle on the GPU's own
    centres, radii and depths, so the check is integer-exact);
  * the cut rectangle is inside the getRect rectangle and covers the alpha
    box;
  * every pixel of a reference tile where the reference arithmetic gives a
    surfel alpha >= 1/255 lies inside the surfel's alpha box (checked with the
    oracle's preprocess values), so no blended sample is lost.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from helpers import api_inputs, small_scene
from nest_b200 import raster, synth
from oracle import oracle

pytestmark = pytest.mark.gpu
TILE = 16


def _forward(scene, inputs):
    cam, g = scene.camera, scene.grid
    dev = "cuda"
    cfg = raster.RasterConfig(image_height=cam.height, image_width=cam.width, tanfovx=cam.tanfovx,
                              tanfovy=cam.tanfovy, viewmatrix=cam.world_view_transform.to(dev),
                              projmatrix=cam.full_proj_transform.to(dev), levels=g.levels, S=g.S,
                              base_resolution=g.base_resolution, channels=g.channels, level_dim=g.level_dim)
    t = {k: v.to(dev).contiguous() for k, v in inputs.items()}
    n, color, others, radii, _, _, scratch = raster.rasterize_forward(
        cfg, t["means3D"], t["scales"], t["rotations"], t["opacities"], t["homotrans"], t["ap_level"],
        g.table.to(dev), g.offsets.to(dev), g.gridrange.to(dev))
    b = raster.read_binning(scratch, scene.P, cam.width, cam.height, n)
    torch.cuda.synchronize()
    b = {k: v.cpu().numpy() for k, v in b.items()}
    b["radii"] = radii.cpu().numpy()
    b["num_rendered"] = n
    return b


def _get_rect(means2D, radii, gx, gy):
    """auxiliary.h:72-82 (getRect), in float32 as the reference evaluates it."""
    px, py = means2D[:, 0].astype(np.float32), means2D[:, 1].astype(np.float32)
    r = radii.astype(np.float32)
    x0 = np.clip(((px - r) / np.float32(TILE)).astype(np.int32), 0, gx)
    y0 = np.clip(((py - r) / np.float32(TILE)).astype(np.int32), 0, gy)
    # p + max_radius + BLOCK - 1 evaluates left to right: ((p + r) + 16) - 1
    x1 = np.clip(((px + r + np.float32(TILE) - np.float32(1)) / np.float32(TILE)).astype(np.int32), 0, gx)
    y1 = np.clip(((py + r + np.float32(TILE) - np.float32(1)) / np.float32(TILE)).astype(np.int32), 0, gy)
    return x0, y0, x1, y1


def check_binning(b, W, H):
    gx, gy = (W + TILE - 1) // TILE, (H + TILE - 1) // TILE
    rects = b["tile_rects"].astype(np.int64)
    live = (rects[:, 2] > rects[:, 0]) & (rects[:, 3] > rects[:, 1])
    # The reference emission + stable sort on the GPU's centres, radii and depths
    # (surfels whose cut rectangle is empty keep no instance either way).
    radii = np.where(live, b["radii"], 0).astype(np.int32)
    x0, y0, x1, y1 = _get_rect(b["means2D"], radii, gx, gy)
    assert np.all(rects[live, 0] >= x0[live]) and np.all(rects[live, 1] >= y0[live])
    assert np.all(rects[live, 2] <= x1[live]) and np.all(rects[live, 3] <= y1[live])
    touched = np.where(radii > 0, (x1 - x0) * (y1 - y0), 0).astype(np.uint32)
    pre = dict(means2D=np.ascontiguousarray(b["means2D"], np.float32),
               depths=np.ascontiguousarray(b["depths"], np.float32), radii=radii, tiles_touched=touched)
    keys, vals, _ = oracle.bin_surfels(pre, W, H)
    tile = (keys >> np.uint64(32)).astype(np.int64)
    tx, ty = tile % gx, tile // gx
    r = rects[vals]
    keep = (tx >= r[:, 0]) & (tx < r[:, 2]) & (ty >= r[:, 1]) & (ty < r[:, 3])
    want = vals[keep].astype(np.int64)
    assert b["num_rendered"] == len(want)
    assert np.array_equal(b["point_list"].astype(np.int64), want)
    kt = tile[keep]
    ranges = np.zeros((gx * gy, 2), np.int64)
    bounds = np.flatnonzero(np.diff(kt)) + 1
    starts = np.concatenate([[0], bounds]) if len(kt) else np.zeros(0, np.int64)
    ends = np.concatenate([bounds, [len(kt)]]) if len(kt) else np.zeros(0, np.int64)
    ranges[kt[starts], 0] = starts
    ranges[kt[starts], 1] = ends
    assert np.array_equal(b["ranges"].astype(np.int64), ranges)
    # the cut rectangle covers the pixel box
    box = b["pixel_boxes"][live]
    bx0 = np.floor(np.maximum(box[:, 0], 0) / TILE).astype(np.int64)
    bx1 = np.floor(box[:, 1] / TILE).astype(np.int64) + 1
    by0 = np.floor(np.maximum(box[:, 2], 0) / TILE).astype(np.int64)
    by1 = np.floor(box[:, 3] / TILE).astype(np.int64) + 1
    lr = rects[live]
    assert np.all(lr[:, 0] == np.maximum(x0[live], bx0)) and np.all(lr[:, 2] == np.minimum(x1[live], bx1))
    assert np.all(lr[:, 1] == np.maximum(y0[live], by0)) and np.all(lr[:, 3] == np.minimum(y1[live], by1))
    return len(vals), len(want)


def alpha_pixels_inside_box(scene, inputs, b):
    """Every (pixel, surfel) pair of the reference's tile lists with alpha >=
    1/255 on the reference path (forward.cu:839-929, oracle preprocess values,
    float32) lies inside the GPU's pixel box of the surfel."""
    cam = scene.camera
    W, H = cam.width, cam.height
    pre = oracle.preprocess(inputs["means3D"].numpy(), inputs["scales"].numpy(), inputs["rotations"].numpy(),
                            inputs["opacities"].numpy(), cam.world_view_transform.numpy(),
                            cam.full_proj_transform.numpy(), W, H)
    keys, vals, _ = oracle.bin_surfels(pre, W, H)
    gx = (W + TILE - 1) // TILE
    tile = (keys >> np.uint64(32)).astype(np.int64)
    f32 = np.float32
    checked = 0
    for lo in range(0, len(vals), 4096):
        v = vals[lo:lo + 4096].astype(np.int64)
        t = tile[lo:lo + 4096]
        off = np.arange(TILE * TILE)
        px = ((t % gx)[:, None] * TILE + off[None] % TILE).astype(f32)
        py = ((t // gx)[:, None] * TILE + off[None] // TILE).astype(f32)
        inside_img = (px < W) & (py < H)
        T9 = pre["transMat"][v].astype(f32)
        Tu, Tv, Tw = T9[:, 0:3, None], T9[:, 3:6, None], T9[:, 6:9, None]
        k = px[:, None, :] * Tw - Tu
        l_ = py[:, None, :] * Tw - Tv
        p = np.cross(k, l_, axis=1)
        with np.errstate(divide="ignore", invalid="ignore"):
            sx, sy = p[:, 0] / p[:, 2], p[:, 1] / p[:, 2]
        rho3d = sx * sx + sy * sy
        m2 = pre["means2D"][v].astype(f32)
        dx, dy = m2[:, 0:1] - px, m2[:, 1:2] - py
        rho2d = f32(2.0) * (dx * dx + dy * dy)
        rho = np.minimum(rho3d, rho2d)
        depth = np.where(rho3d <= rho2d, sx * Tw[:, 0] + sy * Tw[:, 1] + Tw[:, 2], Tw[:, 2])
        op = pre["normal_opacity"][v, 3].astype(f32)[:, None]
        alpha = np.minimum(f32(0.99), op * np.exp(f32(-0.5) * rho).astype(f32))
        hit = inside_img & (alpha >= f32(1.0 / 255.0)) & (depth >= f32(0.2)) & (p[:, 2] != 0)
        box = b["pixel_boxes"][v]
        rect = b["tile_rects"][v].astype(np.int64)
        live = ((rect[:, 2] > rect[:, 0]) & (rect[:, 3] > rect[:, 1]))[:, None]
        in_box = live & (px >= box[:, 0:1]) & (px <= box[:, 1:2]) & (py >= box[:, 2:3]) & (py <= box[:, 3:4])
        assert not np.any(hit & ~in_box), np.argwhere(hit & ~in_box)[:4]
        checked += int(hit.sum())
    return checked


def test_binning_small_scene_exact_and_conservative():
    sc = small_scene()
    inp = api_inputs(sc)
    b = _forward(sc, inp)
    ref_n, n = check_binning(b, sc.camera.width, sc.camera.height)
    assert n < ref_n  # the cut removes instances
    assert alpha_pixels_inside_box(sc, inp, b) > 1000


def test_binning_large_tilted_surfels_exact_and_conservative():
    """Surfels whose alpha-cutoff disc reaches the camera plane keep the full
    reference rectangle; the others take the ellipse box."""
    sc = small_scene(seed=19, log_scale=-0.5)
    inp = api_inputs(sc)
    b = _forward(sc, inp)
    check_binning(b, sc.camera.width, sc.camera.height)
    assert alpha_pixels_inside_box(sc, inp, b) > 10000


def test_binning_config1_exact():
    """benchmark config 1 (200k surfels, 800x800)."""
    sc = synth.config1()
    b = _forward(sc, api_inputs(sc))
    ref_n, n = check_binning(b, sc.camera.width, sc.camera.height)
    assert 0 < n < ref_n


def test_binning_config2_exact():
    """benchmark config 2 geometry (1M surfels at 1297x840, RVQ-mixed attributes)."""
    from helpers import raw_attributes

    sc = synth.config2()
    decoded = torch.from_numpy(oracle.rvq_decode_np(sc.rvq_idx.numpy(), sc.codebooks.numpy()))
    b = _forward(sc, api_inputs(sc, raw_attributes(sc, decoded)))
    ref_n, n = check_binning(b, sc.camera.width, sc.camera.height)
    assert n > 4_000_000 and ref_n > n
