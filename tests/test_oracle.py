"""Known-answer tests that pin the CPU oracle (no GPU).

The reference ships no tests or golden vectors for this path, so these cases
fix the restatement to hand-derived answers of the reference algorithm:
  (i)   dense level-0 grid index x + 17 y + 289 z (hashgrid.h:22-31, res 16);
  (ii)  hashed index (x*1 ^ y*2654435761 ^ z*805459861) mod T (hashgrid.h:7-20,35-39);
  (iii) one surfel facing the camera: alpha = min(0.99, opacity) at its centre
        pixel (forward.cu:839-929), depth = view z;
  (iv)  early termination on a stack of opacity-0.99 surfels, simulated in fp32
        (forward.cu:921-929: T*(1-a) < 1e-4 stops before blending);
  (v)   RVQ decode of one-hot codebooks (benchmark config 0 definition);
plus stability of the tile/depth ordering (rasterizer_impl.cu:381-386).
"""
import math

import numpy as np
import pytest
import torch

from helpers import api_inputs, small_scene
from nest_b200 import camera as camlib
from nest_b200 import synth
from oracle import oracle

T19 = 1 << 19


def _u32(x):
    return int(x) & 0xFFFFFFFF


@pytest.mark.parametrize("x,y,z", [(0, 0, 0), (1, 2, 3), (16, 16, 16), (5, 0, 11)])
def test_dense_level0_index(x, y, z):
    # level 0: scale = 16 - 1 = 15, resolution 16, stride 17, dense since 17^3 <= 2^19
    assert oracle.grid_index(False, T19, 16, x, y, z) == x + 17 * y + 289 * z


@pytest.mark.parametrize("x,y,z", [(0, 0, 0), (7, 3, 1), (101, 102, 55), (4085, 17, 4000)])
def test_hashed_index(x, y, z):
    res = 102  # level 5 at H=16, growth 1.447: 103^3 > 2^19 -> hashed
    h = _u32(x * 1) ^ _u32(y * 2654435761) ^ _u32(z * 805459861)
    assert oracle.grid_index(False, T19, res, x, y, z) == h % T19


def test_level_resolutions_and_dense_levels():
    # scale = exp2(l*S)*16 - 1, res = ceil(scale) + 1; dense iff (res+1)^3 <= 2^19
    S = math.log2(1.447)
    res = [math.ceil(np.float32(2.0 ** (l * S)) * 16 - 1) + 1 for l in range(16)]
    assert res[:6] == [16, 24, 34, 49, 71, 102]
    assert [((r + 1) ** 3 <= T19) for r in res[:6]] == [True] * 5 + [False]


def _facing_surfels(depths, opac, W=65, H=65):
    """Surfels on the optical axis of a camera at (0,-4,0), facing it."""
    cam = camlib.orbit_camera(W, H, 50.0, fovy_deg=50.0)
    n = len(depths)
    xyz = np.zeros((n, 3), np.float32)
    xyz[:, 1] = -4.0 + np.asarray(depths, np.float32)
    # rotation of +90 deg about x maps the surfel normal (local z) onto -y
    q = np.tile(np.array([math.cos(math.pi / 4), math.sin(math.pi / 4), 0, 0], np.float32), (n, 1))
    ls = np.full((n, 2), math.log(0.05), np.float32)
    ol = np.log(np.asarray(opac, np.float32) / (1 - np.asarray(opac, np.float32)))
    base = torch.tensor(np.concatenate([xyz, ls, q, ol[:, None]], 1), dtype=torch.float32)
    return cam, base


def _oracle_on(cam, base, table_range=0.0):
    g = torch.Generator().manual_seed(0)
    grid = synth.hash_grid(g, levels=2, log2_T=12, lo=-table_range, hi=table_range)
    sc = synth.Scene(base, grid, [], cam, torch.full((base.shape[0], 1), 24.0))
    inp = api_inputs(sc)
    out, pre, n = oracle.forward(inp["means3D"].numpy(), inp["scales"].numpy(), inp["rotations"].numpy(),
                                 inp["opacities"].numpy(), inp["homotrans"].numpy(), inp["ap_level"].numpy(),
                                 grid.table.float().numpy(), grid.offsets.numpy(), grid.gridrange.numpy(),
                                 cam.world_view_transform.numpy(), cam.full_proj_transform.numpy(),
                                 cam.width, cam.height, 4, 2, 2, grid.S, 16)
    return out, pre, n


def test_single_surfel_alpha_at_centre():
    cam, base = _facing_surfels([4.0], [0.7])
    out, pre, n = _oracle_on(cam, base)
    c = 32  # principal point of a 65-pixel image: (W-1)/2
    alpha = out["out_others"][1, c, c]
    assert abs(alpha - 0.7) < 1e-6
    assert abs(out["out_others"][0, c, c] - 4.0 * 0.7) < 1e-5  # depth * weight
    assert out["out_others"][7, c, c] == 1.0  # one blended sample
    assert pre["radii"][0] >= 3


def test_opaque_stack_terminates_in_fp32():
    depths = [3.0, 3.5, 4.0, 4.5]
    cam, base = _facing_surfels(depths, [0.99] * 4)
    out, _, _ = _oracle_on(cam, base)
    c = 32
    # simulate the termination rule in float32
    T = np.float32(1.0)
    blended = 0
    for _ in depths:
        a = np.float32(0.99)
        tt = np.float32(T * (np.float32(1) - a))
        if tt < np.float32(1e-4):
            break
        blended += 1
        T = tt
    assert out["out_others"][7, c, c] == blended
    assert blended == 1  # 0.01 * 0.01 rounds below 1e-4 in fp32
    assert abs(out["final_T"][0, c, c] - T) < 1e-9


def test_rvq_one_hot_decode():
    K, E, D = 6, 256, 59
    cb = np.zeros((K, E, D), np.float32)
    for k in range(K):
        for e in range(E):
            cb[k, e, (7 * k + e) % D] = 2.0 ** k
    rng = np.random.default_rng(0)
    idx = rng.integers(0, E, size=(300, K), dtype=np.uint8)
    expect = np.zeros((300, D), np.float32)
    for k in range(K):
        expect[np.arange(300), (7 * k + idx[:, k].astype(int)) % D] += 2.0 ** k
    assert np.array_equal(oracle.rvq_decode_np(idx, cb), expect)
    assert np.array_equal(oracle.rvq_decode_c(idx, cb), expect)


def test_rvq_torch_matches_numpy_bitwise():
    cb, idx = synth.config0(n=5000)
    a = oracle.rvq_decode_torch(idx, cb).numpy()
    b = oracle.rvq_decode_np(idx.numpy(), cb.numpy())
    c = oracle.rvq_decode_c(idx.numpy(), cb.numpy())
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    assert np.array_equal(b.view(np.uint32), c.view(np.uint32))


def test_binning_order_is_tile_then_depth_then_index():
    sc = small_scene(n=400, width=64, height=48)
    inp = api_inputs(sc)
    cam = sc.camera
    pre = oracle.preprocess(inp["means3D"].numpy(), inp["scales"].numpy(), inp["rotations"].numpy(),
                            inp["opacities"].numpy(), cam.world_view_transform.numpy(),
                            cam.full_proj_transform.numpy(), cam.width, cam.height)
    # force depth ties to exercise stability
    pre["depths"][::2] = 3.0
    keys, vals, ranges = oracle.bin_surfels(pre, cam.width, cam.height)
    order = np.lexsort((vals, keys))
    assert np.array_equal(order, np.arange(len(keys)))
    tiles = (keys >> np.uint64(32)).astype(np.int64)
    for t in np.unique(tiles):
        sel = np.nonzero(tiles == t)[0]
        assert ranges[t, 0] == sel[0] and ranges[t, 1] == sel[-1] + 1


def test_mlp_oracle_shapes_and_mask():
    g = torch.Generator().manual_seed(3)
    ws = synth.xavier_mlp(g)
    feat = np.random.default_rng(1).normal(size=(32, 4, 5)).astype(np.float32)
    alpha = np.ones((4, 5), np.float32)
    alpha[0, 0] = 0
    rgb = oracle.mlp_oracle(feat, ws, alpha, bg=np.array([0.0, 0.0, 0.0]))
    assert rgb.shape == (3, 4, 5)
    assert np.all(rgb[:, 0, 0] == 0)
    assert np.all((rgb[:, 1:, :] > 0) & (rgb[:, 1:, :] < 1))


def _oracle_kernels(cam, base, kernel_type, shapes, beta=0.0):
    g = torch.Generator().manual_seed(0)
    grid = synth.hash_grid(g, levels=2, log2_T=12, lo=0.0, hi=0.0)
    sc = synth.Scene(base, grid, [], cam, torch.full((base.shape[0], 1), 24.0))
    inp = api_inputs(sc)
    out, pre, n = oracle.forward(inp["means3D"].numpy(), inp["scales"].numpy(), inp["rotations"].numpy(),
                                 inp["opacities"].numpy(), inp["homotrans"].numpy(), inp["ap_level"].numpy(),
                                 grid.table.float().numpy(), grid.offsets.numpy(), grid.gridrange.numpy(),
                                 cam.world_view_transform.numpy(), cam.full_proj_transform.numpy(),
                                 cam.width, cam.height, 4, 2, 2, grid.S, 16, kernel_type=kernel_type,
                                 shapes=np.asarray(shapes, np.float32), beta=beta)
    return out


@pytest.mark.parametrize("kernel_type,shape", [(1, 2.0), (1, 0.0), (2, 1.5), (3, 4.0)])
def test_splat_kernels_alpha_at_centre(kernel_type, shape):
    """Every splat kernel has G = 1 at the surfel centre (forward.cu:864-902):
    alpha = opacity there."""
    cam, base = _facing_surfels([4.0], [0.6])
    out = _oracle_kernels(cam, base, kernel_type, [shape])
    assert abs(out["out_others"][1, 32, 32] - 0.6) < 1e-5


def test_beta_kernel_shape_zero_is_flat_disc():
    """Kernel 1 with shape 0: G = (1 - rho)^0 = 1 inside the unit circle and no
    sample outside it, so every covered pixel has alpha = opacity exactly."""
    cam, base = _facing_surfels([4.0], [0.6])
    base[:, 3:5] = math.log(0.3)  # a disc a few pixels wide
    out = _oracle_kernels(cam, base, 1, [0.0])
    a = out["out_others"][1]
    covered = a > 0
    assert covered.sum() > 20
    assert np.all(np.abs(a[covered] - 0.6) < 1e-6)


def test_flex_kernel_equals_global_beta():
    """Kernel 2 with per-surfel shape b renders what kernel 0 renders with the
    global beta b (forward.cu:873-885 against :903-915)."""
    cam, base = _facing_surfels([3.0, 3.5, 4.0], [0.5, 0.4, 0.3])
    base[:, 3:5] = math.log(0.2)
    flex = _oracle_kernels(cam, base, 2, [0.7, 0.7, 0.7])
    glob = _oracle_kernels(cam, base, 0, [0.0, 0.0, 0.0], beta=0.7)
    assert np.abs(flex["out_others"][:7] - glob["out_others"][:7]).max() < 1e-5
    assert flex["out_others"][1].max() > 0.1


@pytest.mark.parametrize("mode", [4, 12, 14, 13 | 256])
def test_render_modes_single_surfel_features(mode):
    """One facing surfel and a zero hash table: the features at its centre are
    alpha times the surfel's row as each mode combines it (forward.cu:964-1091,
    1218-1282, 1593-1790): mode 4 and 14 copy the coarse channels, mode 12
    copies them and scales the fine ones by the blend weight, mode 13 with the
    inference flag and weight > 0.5 copies every channel."""
    cam, base = _facing_surfels([4.0], [0.6])
    g = torch.Generator().manual_seed(0)
    total, hybrid, L = 2, 1, 1
    grid = synth.hash_grid(g, levels=L, log2_T=12, lo=0.0, hi=0.0)
    sc = synth.Scene(base, grid, [], cam, torch.full((1, 1), 24.0))
    inp = api_inputs(sc)
    base_mode = mode & 0xFF
    row = {4: [0.5, -0.25], 12: [0.5, -0.25, 0.75, 1.5, 0.8], 14: [0.5, -0.25, 0.8],
           13: [0.5, -0.25, 0.75, 1.5, 0.8]}[base_mode]
    gauss = np.asarray([row], np.float32)
    out, _, _ = oracle.forward(inp["means3D"].numpy(), inp["scales"].numpy(), inp["rotations"].numpy(),
                               inp["opacities"].numpy(), inp["homotrans"].numpy(), inp["ap_level"].numpy(),
                               grid.table.float().numpy(), grid.offsets.numpy(), grid.gridrange.numpy(),
                               cam.world_view_transform.numpy(), cam.full_proj_transform.numpy(),
                               cam.width, cam.height, 2 * total, 2, L, grid.S, 16, render_mode=mode,
                               hybrid_levels=hybrid, total_levels=total, gauss=gauss)
    f = out["out_color"][:, 32, 32] / 0.6
    want = {4: [0.5, -0.25, 0, 0], 12: [0.5, -0.25, 0.8 * 0.75, 0.8 * 1.5], 14: [0.5, -0.25, 0, 0],
            13: [0.5, -0.25, 0.75, 1.5]}[base_mode]
    assert np.allclose(f, want, atol=1e-5), f
